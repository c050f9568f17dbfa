"""bench.py's JSON-line contract, checked on the CPU.

The reference arm (`--impl reference`) runs the reference's own CPU decode
(compiled in place) and needs no GPU, so its line is checked here on a tiny
preset; the B200 arm must fail loudly (non-zero exit, no JSON line) where
no GPU is present instead of falling back to a CPU path.
"""
import json
import os
import subprocess
import sys

import pytest
import torch

from oracle import RefLib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_bench(tmp_path, *args):
    env = dict(os.environ, AF_BENCH_DIR=str(tmp_path))
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                          env=env, cwd=str(tmp_path), timeout=600)


def json_lines(out: str):
    return [json.loads(l) for l in out.splitlines() if l.startswith("{")]


@pytest.mark.skipif(not RefLib.available(), reason="reference library not built")
def test_reference_arm_line(tmp_path):
    r = run_bench(tmp_path, "--impl", "reference", "--model", "tiny", "--steps", "4", "--warmup", "1")
    assert r.returncode == 0, r.stderr
    lines = json_lines(r.stdout)
    assert len(lines) == 1, r.stdout
    d = lines[0]
    assert d["impl"] == "reference"
    assert d["metric"] == "bs=1 decode tok/s" and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["steps"] == 4 and d["warmup"] == 3  # fewer than 3 warm-up steps are raised to 3
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["model"] == "tiny-llama" and d["config"]["seq_len"] == 128
    lo, hi = (int(v) for v in d["config"]["context"].split(".."))
    assert hi - lo == 4 and lo >= 128
    assert d["config"]["l2"].startswith("weights fit in L2")
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == d["value"] and cb["cores"] == len(os.sched_getaffinity(0))
    assert cb["cpu_model"] and cb["affinity"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour without a GPU")
def test_b200_arm_fails_loudly_without_gpu(tmp_path):
    r = run_bench(tmp_path, "--model", "tiny", "--steps", "3", "--warmup", "3", "--no-cpu-baseline")
    assert r.returncode != 0
    assert not json_lines(r.stdout)
