"""Batched dequant GEMV (af_gemv_batched_f32) through the C ABI against the C
oracle: every vector's row of Y must equal the reference-order F32 GEMV of
that vector (oracle/af_oracle.c, pinned to gemv_q4k_avx2_range /
gemv_q6k_avx2_range), within the GEMV bar of 2e-3 relative L2 per vector.

The inputs are quantised to a 16-bit grid per token and 256 values, so the
error is of the order 1e-5; 1e-4 is asserted as the tighter check."""
import ctypes

import numpy as np
import pytest

from helpers import GEMV_TOL, dev, rel_l2
from llm_core_b200 import gguf
from oracle import COracle

pytestmark = pytest.mark.gpu


def packed(lib, W, t, rows, cols):
    import torch
    src = dev(W)
    Wd = torch.empty(lib.af_weight_bytes(t, rows, cols), dtype=torch.uint8, device="cuda")
    assert lib.af_weight_pack(Wd.data_ptr(), src.data_ptr(), t, rows, cols, None) == 0
    return Wd


def run_bgemv(lib, Wd, t, X, rows):
    import torch
    B, cols = X.shape
    xd = dev(np.ascontiguousarray(X, dtype=np.float32))
    y = torch.full((B, rows), float("nan"), dtype=torch.float32, device="cuda")
    rc = lib.af_gemv_batched_f32(y.data_ptr(), Wd.data_ptr(), t, xd.data_ptr(), rows, cols, B, None)
    assert rc == 0, lib.af_last_error()
    torch.cuda.synchronize()
    code = ctypes.c_int()
    lib.af_device_error(ctypes.byref(code), 1)
    assert code.value == 0
    return y.cpu().numpy()


def oracle_rows(W, t, X, rows):
    D = COracle().dequant_rows(W, t, rows, X.shape[1]).astype(np.float64)
    return (X.astype(np.float64) @ D.T).astype(np.float32)


@pytest.mark.parametrize("t", [gguf.GGML_Q4_K, gguf.GGML_Q6_K])
@pytest.mark.parametrize("rows,cols,B", [
    (2048, 4096, 4), (4096, 2048, 16),     # the sweep's batches
    (1000, 2048, 2),                        # rows not a multiple of 16
    (256, 2048, 5),                         # fewer tiles than SMs: sub-block parts per warp
    (5632, 2048, 8), (2048, 5632, 9),       # 22 super-blocks; a partial token octet
    (300, 768, 31), (4096, 512, 32),        # the largest batch
    (40, 11008, 16),                        # 43 super-blocks: a partial last entry
    (32000, 256, 3),                        # groups of 8 tiles, one super-block
])
def test_batched_gemv_matches_oracle(gpu, t, rows, cols, B):
    rng = np.random.default_rng(9100 + rows + cols + B + t)
    gen = gguf.random_q4k if t == gguf.GGML_Q4_K else gguf.random_q6k
    W = gen(rng, rows * cols // 256).reshape(-1)
    X = rng.standard_normal((B, cols)).astype(np.float32)
    y = run_bgemv(gpu, packed(gpu, W, t, rows, cols), t, X, rows)
    ref = oracle_rows(W, t, X, rows)
    assert np.isfinite(y).all()
    worst = max(rel_l2(y[n], ref[n]) for n in range(B))
    assert worst < GEMV_TOL and worst < 1e-4, worst


def test_batched_gemv_is_deterministic_and_matches_single_vector(gpu):
    """Two calls give identical bytes; each vector agrees with the
    single-vector GEMV (16-bit input grids per 256 vs per 32 values)."""
    import torch
    rng = np.random.default_rng(5)
    rows, cols, B = 4096, 4096, 16
    W = gguf.random_q4k(rng, rows * cols // 256).reshape(-1)
    X = rng.standard_normal((B, cols)).astype(np.float32)
    Wd = packed(gpu, W, gguf.GGML_Q4_K, rows, cols)
    y1 = run_bgemv(gpu, Wd, gguf.GGML_Q4_K, X, rows)
    y2 = run_bgemv(gpu, Wd, gguf.GGML_Q4_K, X, rows)
    np.testing.assert_array_equal(y1, y2)
    for n in (0, 7, 15):
        xd = dev(X[n].copy())
        y = torch.empty(rows, dtype=torch.float32, device="cuda")
        assert gpu.af_gemv_f32(y.data_ptr(), Wd.data_ptr(), gguf.GGML_Q4_K, xd.data_ptr(), rows, cols, None) == 0
        assert rel_l2(y.cpu().numpy(), y1[n]) < 1e-4


def test_batched_gemv_activation_range_and_zeros(gpu):
    """Per-token scales: vectors of very different magnitude and an
    all-zero vector keep their own accuracy."""
    rng = np.random.default_rng(12)
    rows, cols = 512, 1024
    W = gguf.random_q4k(rng, rows * cols // 256).reshape(-1)
    X = rng.standard_normal((6, cols)).astype(np.float32)
    X *= np.array([1e-20, 1e-3, 1.0, 1e3, 1e20, 0.0], np.float32)[:, None]
    y = run_bgemv(gpu, packed(gpu, W, gguf.GGML_Q4_K, rows, cols), gguf.GGML_Q4_K, X, rows)
    ref = oracle_rows(W, gguf.GGML_Q4_K, X, rows)
    for n in range(5):
        assert rel_l2(y[n], ref[n]) < 1e-4, n
    assert (y[5] == 0).all()


def test_batched_gemv_rejects_bad_arguments(gpu):
    assert gpu.af_gemv_batched_f32(None, None, gguf.GGML_Q4_K, None, 16, 256, 33, None) != 0
    assert b"n_vec" in gpu.af_last_error()
    assert gpu.af_gemv_batched_f32(None, None, gguf.GGML_Q4_K, None, 16, 300, 4, None) != 0
