"""Prefill dequant-GEMM (tcgen05 / TMEM) through the C ABI against the C
oracle: every token's row of Y must equal the reference-order F32 GEMV of
that token (oracle/af_oracle.c, pinned to gemv_q4k_avx2_range /
gemv_q6k_avx2_range).

Tolerance: 2e-3 relative L2 (the GEMV bar), and 1e-3 as a tighter check: the
GEMM rounds the dequantised weights and the (power-of-two scaled) activations
to f16, ≈2e-4 relative rms together."""
import ctypes

import numpy as np
import pytest

from helpers import GEMV_TOL, dev, rel_l2
from llm_core_b200 import gguf
from oracle import COracle

pytestmark = pytest.mark.gpu


def run_prefill(lib, W, t, X, rows):
    import torch
    T, cols = X.shape
    src = dev(W)
    Wd = torch.empty(lib.af_weight_bytes(t, rows, cols), dtype=torch.uint8, device="cuda")
    assert lib.af_weight_pack(Wd.data_ptr(), src.data_ptr(), t, rows, cols, None) == 0
    xd = dev(np.ascontiguousarray(X, dtype=np.float32))
    y = torch.full((T, rows), float("nan"), dtype=torch.float32, device="cuda")
    assert lib.af_prefill_gemm_f32(y.data_ptr(), Wd.data_ptr(), t, xd.data_ptr(), rows, cols, T, None) == 0
    torch.cuda.synchronize()
    code = ctypes.c_int()
    lib.af_device_error(ctypes.byref(code), 1)
    assert code.value == 0
    return y.cpu().numpy()


def oracle_rows(W, t, X, rows):
    """Y = X · Wᵀ with W dequantised by the oracle's row dequantiser (f64 sums)."""
    D = COracle().dequant_rows(W, t, rows, X.shape[1]).astype(np.float64)
    return (X.astype(np.float64) @ D.T).astype(np.float32)


@pytest.mark.parametrize("t", [gguf.GGML_Q4_K, gguf.GGML_Q6_K])
@pytest.mark.parametrize("rows,cols,T", [(128, 256, 128), (256, 2048, 64), (300, 768, 130), (37, 512, 1),
                                         (1024, 4096, 200), (4096, 512, 1200),
                                         # the batched-GEMV sizes of the sweep: 4 and 16 vectors
                                         (2048, 4096, 4), (4096, 2048, 16)])
def test_prefill_gemm_matches_oracle(gpu, t, rows, cols, T):
    """(4096, 512, 1200) is a grid of 320 CTAs: the two-CTAs-per-SM variant;
    the others run one CTA per SM with four stages."""
    rng = np.random.default_rng(7000 + rows + cols + T + t)
    gen = gguf.random_q4k if t == gguf.GGML_Q4_K else gguf.random_q6k
    W = gen(rng, rows * cols // 256).reshape(-1)
    X = rng.standard_normal((T, cols)).astype(np.float32)
    y = run_prefill(gpu, W, t, X, rows)
    ref = oracle_rows(W, t, X, rows)
    assert np.isfinite(y).all()
    err = rel_l2(y, ref)
    assert err < GEMV_TOL and err < 1e-3, err
    # every token on its own, so a slip in one tile cannot hide in the total
    worst = max(rel_l2(y[n], ref[n]) for n in range(T))
    assert worst < 2 * GEMV_TOL, worst


def test_prefill_gemm_activation_range(gpu):
    """Per-token scales: tokens of very different magnitude (1e-6 .. 1e6, f16
    alone would underflow or overflow) keep the same relative accuracy."""
    rng = np.random.default_rng(11)
    rows, cols = 256, 1024
    W = gguf.random_q4k(rng, rows * cols // 256).reshape(-1)
    X = rng.standard_normal((6, cols)).astype(np.float32)
    X *= np.array([1e-6, 1e-3, 1.0, 1e3, 1e5, 1e6], np.float32)[:, None]
    y = run_prefill(gpu, W, gguf.GGML_Q4_K, X, rows)
    ref = oracle_rows(W, gguf.GGML_Q4_K, X, rows)
    for n in range(X.shape[0]):
        assert rel_l2(y[n], ref[n]) < 1e-3, n


def test_prefill_gemm_zero_input(gpu):
    rng = np.random.default_rng(3)
    W = gguf.random_q4k(rng, 64 * 8).reshape(-1)
    y = run_prefill(gpu, W, gguf.GGML_Q4_K, np.zeros((5, 2048), np.float32), 64)
    assert np.all(y == 0)


def test_prefill_gemm_rejects_bad_shapes(gpu):
    assert gpu.af_prefill_gemm_f32(None, None, gguf.GGML_Q4_K, None, 16, 100, 4, None) != 0
    assert gpu.af_prefill_gemm_f32(None, None, 99, None, 16, 256, 4, None) != 0
