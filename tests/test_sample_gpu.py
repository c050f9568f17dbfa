"""Device sampling against the reference's own sampler.

The reference samples with apply_rep_penalty + sample()
(src/models/llama_model.cpp:1466-1498, 1586-1598) and std::mt19937(42).
af_sample_f32 gets the same logits and the draw the reference's rng would
make; the picks must be identical (inputs are seeded, so a pick that sat
within expf rounding of a cumulative boundary would show on every run, not
intermittently).  Whole generations are compared on a small random-init model
with the reference forward in F32-activation mode."""
import ctypes as C

import numpy as np
import pytest

from helpers import dev, model_path
from llm_core_b200 import _lib
from llm_core_b200.engine import LlamaConfig, LlamaCudaModel, mt19937_uniform
from oracle import RefLib

pytestmark = pytest.mark.gpu

CASES = [
    # (vocab, temperature, top_k, top_p, rep_penalty, window)
    (32000, 0.0, 40, 1.0, 1.0, 0),     # greedy
    (32000, 0.0, 40, 1.0, 1.3, 64),    # greedy after the penalty
    (32000, 1.0, 40, 0.95, 1.0, 0),    # the reference CLI defaults
    (32000, 0.7, 40, 1.0, 1.1, 64),
    (32000, 1.5, 1, 1.0, 1.0, 0),      # top-1
    (32000, 0.8, 1024, 0.9, 1.0, 0),   # the largest k the device sorts
    (151936, 1.0, 40, 0.95, 1.2, 16),  # Qwen2.5 vocabulary
    (1000, 2.0, 999, 0.5, 1.0, 0),
]


def _sample_dev(lib, logits, window, s, r):
    import torch
    d_lg = dev(logits)
    d_w = dev(np.asarray(window, np.int32)) if len(window) else None
    d_out = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.af_sample_f32(d_lg.data_ptr(), logits.size, d_w.data_ptr() if d_w is not None else None, len(window),
                           C.byref(s), r, d_out.data_ptr(), None)
    _lib.check(rc, "af_sample_f32")
    torch.cuda.synchronize()
    return int(d_out.item()), d_lg.cpu().numpy()


@pytest.mark.parametrize("case", CASES)
def test_sampler_matches_reference(gpu, case):
    if not RefLib.available():
        pytest.skip("reference library not built")
    V, T, k, p, pen, nw = case
    ref = RefLib()
    rng = np.random.default_rng(V + nw)
    for trial in range(24):
        logits = (rng.standard_normal(V) * 3.0).astype(np.float32)
        # repeated ids in the window are penalised once per occurrence
        window = rng.integers(0, V, nw).astype(np.int32)
        if nw:
            window[nw // 2:] = window[: nw - nw // 2]
        seed = 1000 + trial
        r = float(mt19937_uniform(1, seed)[0])
        s = _lib.Sampling(T, k, p, pen, nw)
        got, penalised = _sample_dev(gpu, logits, window, s, r)
        want = ref.sample(logits, window, pen, k, p, T, seed)
        assert got == want, f"trial {trial}: device {got} reference {want}"
        # the penalty is applied in place, as the reference's lambda does
        exp = logits.copy()
        for i in window:
            exp[i] = exp[i] / pen if exp[i] > 0 else exp[i] * pen
        np.testing.assert_array_equal(penalised, exp)


def test_sampler_rejects_unsupported_k(gpu):
    import torch
    logits = np.zeros(4096, np.float32)
    d = dev(logits)
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = _lib.Sampling(1.0, 0, 1.0, 1.0, 0)  # top_k 0 keeps 4096 > 1024 candidates
    assert gpu.af_sample_f32(d.data_ptr(), 4096, None, 0, C.byref(s), 0.5, out.data_ptr(), None) != 0
    assert b"top_k" in gpu.af_last_error()


@pytest.mark.parametrize("preset,cfg", [
    ("tiny", LlamaConfig(max_new_tokens=48, temperature=0.8, top_k=40, top_p=0.95, rep_penalty=1.1)),
    ("tiny", LlamaConfig(max_new_tokens=48, temperature=0.0, rep_penalty=1.3, rep_penalty_last_n=16)),
    ("tiny-qwen", LlamaConfig(max_new_tokens=32, temperature=1.0, top_k=40, top_p=1.0)),
])
def test_generate_sampled_matches_reference(gpu, preset, cfg):
    if not RefLib.available():
        pytest.skip("reference library not built")
    path = model_path(preset, 11)
    prompt = [5, 17, 99, 3, 250, 7]
    ref = RefLib().open(path, threads=4, f32_mode=True)
    want = ref.generate_sampled(prompt, cfg.max_new_tokens, cfg.temperature, cfg.top_k, cfg.top_p,
                                cfg.rep_penalty, cfg.rep_penalty_last_n)
    ref.close()
    m = LlamaCudaModel(path)
    got = m.generate(prompt, cfg)
    m.close()
    assert got == want
