"""Shared test helpers: device buffers through torch (plumbing only), rel-L2."""
from __future__ import annotations

import os
import tempfile

import numpy as np

GEMV_TOL = 2e-3     # per-GEMV relative L2 bound (north star)
LOGITS_TOL = 5e-3   # final-logits relative L2 bound (north star)
TOP1_MIN = 0.99     # greedy top-1 agreement over 256 steps (north star)


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def dev(a: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ptr(t) -> int:
    return t.data_ptr()


_MODEL_CACHE = {}


def model_path(preset: str, seed: int) -> str:
    """Seeded random-init GGUF for a preset, written once per session."""
    from llm_core_b200 import gguf
    key = (preset, seed)
    if key not in _MODEL_CACHE:
        d = os.environ.get("AF_TEST_MODEL_DIR") or tempfile.gettempdir()
        p = os.path.join(d, f"af_{preset}_{seed}.gguf")
        if not os.path.exists(p):
            gguf.write_random_model(p, preset, seed)
        _MODEL_CACHE[key] = p
    return _MODEL_CACHE[key]
