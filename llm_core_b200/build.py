"""Build the sm_100a shared library llm_core_b200/libaf_b200.so in-tree with nvcc.

    python -m llm_core_b200.build        (or __graft_entry__.build())
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libaf_b200.so")
SOURCES = ["af_gemv.cu", "af_ops.cu", "af_attention.cu", "af_step.cu", "af_prefill.cu", "af_bgemv.cu", "af_sample.cu", "af_engine.cu",
           "af_gguf.cpp"]
HEADERS = ["af_common.cuh", "af_gemv.cuh", "af_gemv_dev.cuh", "af_ops.cuh", "af_step.cuh", "af_gguf.h"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", f"-I{os.path.join(ROOT, 'include')}"]


def _stale(obj: str, deps) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, jobs: int = 8) -> str:
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "af_b200.h")]
    objs, procs = [], []
    for src in SOURCES:
        sp = os.path.join(CSRC, src)
        obj = os.path.join(objdir, src + ".o")
        objs.append(obj)
        if _stale(obj, [sp] + hdrs):
            cmd = [NVCC, *GENCODE, *FLAGS, "-dc" if src.endswith(".cu") else "-c", sp, "-o", obj]
            if src.endswith(".cpp"):
                cmd = [NVCC, *FLAGS, "-x", "c++", "-c", sp, "-o", obj]
            if verbose:
                print(" ".join(cmd))
            procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
            if len(procs) >= jobs:
                _wait(procs)
    _wait(procs)
    if _stale(LIB, objs):
        cmd = [NVCC, *GENCODE, "-shared", "-o", LIB, *objs, "-L/usr/lib/x86_64-linux-gnu", "-lnccl",
               "-lcudart"]
        if verbose:
            print(" ".join(cmd))
        subprocess.check_call(cmd)
    return LIB


def _wait(procs):
    errs = []
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            errs.append(f"--- {src}\n{out.decode(errors='replace')}")
        elif out.strip():
            sys.stderr.write(out.decode(errors="replace"))
    procs.clear()
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
