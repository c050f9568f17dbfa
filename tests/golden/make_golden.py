"""Generate the committed golden fixtures from the reference's own CPU code.

Run in the build container (where the reference sources are present):

    python tests/golden/make_golden.py

It compiles oracle/_ref/libaxref.so from the unmodified reference sources
(oracle/ref.mk) and records, for seeded inputs:

* gemv_*.npz   — Q4_K / Q6_K blocks, x, and y from gemv_q4k_avx2_range /
                 gemv_q6k_avx2_range (F32 activations) plus the production
                 Q8_0-activation y (for reporting only);
* model_tiny.npz / model_tiny_qwen.npz — per-position logits of
                 llama_forward_token (F32 mode) for a fixed token sequence on the
                 seeded random-init GGUF written by llm_core_b200.gguf, the greedy
                 continuation from the reference decode loop, and a SHA-256 of
                 the GGUF so the fixture is tied to the exact bytes.
"""
from __future__ import annotations

import hashlib
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from llm_core_b200 import gguf  # noqa: E402
from oracle import RefLib, build_ref  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))

GEMV_CASES = [
    # (name, ggml_type, rows, cols, seed)
    ("gemv_q4k_256x2048", gguf.GGML_Q4_K, 256, 2048, 11),
    ("gemv_q4k_40x11008", gguf.GGML_Q4_K, 40, 11008, 12),
    ("gemv_q4k_37x256", gguf.GGML_Q4_K, 37, 256, 13),
    ("gemv_q6k_256x2048", gguf.GGML_Q6_K, 256, 2048, 21),
    ("gemv_q6k_40x11008", gguf.GGML_Q6_K, 40, 11008, 22),
    ("gemv_q6k_37x256", gguf.GGML_Q6_K, 37, 256, 23),
]

MODEL_CASES = [
    # (fixture, preset, seed, tokens, greedy steps)
    ("model_tiny", "tiny", 1, [1, 5, 77, 300, 2, 9, 511, 0], 24),
    ("model_tiny_qwen", "tiny-qwen", 2, [1, 17, 999, 4, 250], 24),
]


def sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def main():
    if build_ref() is None:
        raise SystemExit("reference sources not found; fixtures can only be generated where they are")
    ref = RefLib()
    for name, t, rows, cols, seed in GEMV_CASES:
        rng = np.random.default_rng(seed)
        blocks = rows * cols // gguf.QK_K
        W = (gguf.random_q4k if t == gguf.GGML_Q4_K else gguf.random_q6k)(rng, blocks).reshape(-1)
        x = rng.standard_normal(cols).astype(np.float32)
        y = ref.gemv_f32(W, t, x, rows)
        y8 = ref.gemv_q8(W, t, x, rows)
        np.savez_compressed(os.path.join(OUT, name + ".npz"), W=W, x=x, y=y, y_q8=y8,
                            ggml_type=t, rows=rows, cols=cols)
        print(name, float(np.linalg.norm(y8 - y) / np.linalg.norm(y)))
    with tempfile.TemporaryDirectory() as td:
        for fx, preset, seed, toks, steps in MODEL_CASES:
            path = os.path.join(td, fx + ".gguf")
            cfg = gguf.write_random_model(path, preset, seed)
            ref.open(path, threads=2, f32_mode=True)
            logits = np.stack([ref.forward_token(tk, p) for p, tk in enumerate(toks)])
            ref.open(path, threads=2, f32_mode=True)
            prompt = toks[1:5]
            gen, glog = ref.generate_greedy(prompt, steps, want_logits=True)
            np.savez_compressed(os.path.join(OUT, fx + ".npz"), tokens=np.array(toks, np.int32),
                                logits=logits, prompt=np.array(prompt, np.int32),
                                greedy=np.array(gen, np.int32), greedy_logits=glog,
                                preset=preset, seed=seed, sha256=sha256(path))
            print(fx, cfg.name, logits.shape, gen[:8])
            ref.close()


if __name__ == "__main__":
    main()
