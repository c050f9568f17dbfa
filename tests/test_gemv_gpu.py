"""GEMV parity on the B200 through the C ABI (af_gemv_f32) against the
reference's F32-activation x86 kernels (fixtures) and the C oracle.

Tolerance: 2e-3 relative L2 per GEMV (north star); the design's 16-bit split of
x gives ~1e-5, so the tests also assert a much tighter 1e-4 to catch layout
slips that would still hide under 2e-3."""
import glob
import os

import numpy as np
import pytest

from helpers import GEMV_TOL, dev, rel_l2
from llm_core_b200 import gguf
from oracle import COracle

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
TIGHT = 1e-4


def to_device_layout(lib, W: np.ndarray, t: int, rows: int, cols: int):
    import torch
    src = dev(W)
    dst = torch.empty(lib.af_weight_bytes(t, rows, cols), dtype=torch.uint8, device="cuda")
    assert lib.af_weight_pack(dst.data_ptr(), src.data_ptr(), t, rows, cols, None) == 0
    return dst


def run_gemv(lib, W, t, x, rows):
    import torch
    cols = x.size
    Wd = to_device_layout(lib, W, t, rows, cols)
    xd = dev(x.astype(np.float32))
    y = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    assert lib.af_gemv_f32(y.data_ptr(), Wd.data_ptr(), t, xd.data_ptr(), rows, cols, None) == 0
    torch.cuda.synchronize()
    code = (__import__("ctypes").c_int)()
    lib.af_device_error(__import__("ctypes").byref(code), 1)
    assert code.value == 0
    return y.cpu().numpy()


@pytest.mark.parametrize("fx", sorted(glob.glob(os.path.join(GOLD, "gemv_*.npz"))), ids=os.path.basename)
def test_gemv_matches_reference_fixture(gpu, fx):
    z = np.load(fx)
    y = run_gemv(gpu, z["W"], int(z["ggml_type"]), z["x"], int(z["rows"]))
    err = rel_l2(y, z["y"])
    assert err < GEMV_TOL and err < TIGHT, err


# TinyLlama layer shapes, seeded Q4_K blocks, x ~ N(0,1)
CONFIG0 = [(2048, 2048), (256, 2048), (5632, 2048), (2048, 5632)]


@pytest.mark.parametrize("t", [gguf.GGML_Q4_K, gguf.GGML_Q6_K])
@pytest.mark.parametrize("rows,cols", CONFIG0 + [(1, 256), (37, 768), (300, 11008), (4096, 4096), (11008, 4096)])
def test_gemv_matches_oracle(gpu, t, rows, cols):
    rng = np.random.default_rng(1000 + rows + cols + t)
    gen = gguf.random_q4k if t == gguf.GGML_Q4_K else gguf.random_q6k
    W = gen(rng, rows * cols // 256).reshape(-1)
    x = rng.standard_normal(cols).astype(np.float32)
    y = run_gemv(gpu, W, t, x, rows)
    ref = COracle().gemv(W, t, x, rows)
    err = rel_l2(y, ref)
    assert err < GEMV_TOL and err < TIGHT, err


def test_gemv_edge_inputs(gpu):
    rng = np.random.default_rng(5)
    W = gguf.random_q4k(rng, 64 * 8).reshape(-1)
    orc = COracle()
    for x in (np.zeros(2048, np.float32),                      # all-zero input
              np.full(2048, 3.0, np.float32),                  # constant input
              (rng.standard_normal(2048) * 1e4).astype(np.float32),
              np.where(rng.random(2048) < 0.9, 0, rng.standard_normal(2048)).astype(np.float32)):
        y = run_gemv(gpu, W, gguf.GGML_Q4_K, x, 64)
        ref = orc.gemv(W, gguf.GGML_Q4_K, x, 64)
        if np.linalg.norm(ref) == 0:
            assert np.all(y == 0)
        else:
            assert rel_l2(y, ref) < TIGHT


@pytest.mark.parametrize("t", [gguf.GGML_Q4_K, gguf.GGML_Q6_K])
def test_weight_pack_round_trip(gpu, t):
    """The packed layout is a bit-preserving permutation of the GGUF bytes
    (Q4_K: a byte permutation; Q6_K: nibbles and 2-bit fields regrouped)."""
    import torch
    rng = np.random.default_rng(9)
    gen = gguf.random_q4k if t == gguf.GGML_Q4_K else gguf.random_q6k
    for rows, cols in ((3, 256), (17, 2048), (40, 11008)):
        W = gen(rng, rows * cols // 256).reshape(-1)
        packed = to_device_layout(gpu, W, t, rows, cols)
        assert packed.numel() == gpu.af_weight_bytes(t, rows, cols)
        back = torch.zeros(W.size, dtype=torch.uint8, device="cuda")
        assert gpu.af_weight_unpack(back.data_ptr(), packed.data_ptr(), t, rows, cols, None) == 0
        torch.cuda.synchronize()
        assert np.array_equal(back.cpu().numpy(), W)
        # same set bits, plus zero padding
        p = packed.cpu().numpy()
        assert int(np.unpackbits(p).sum()) == int(np.unpackbits(W).sum())
        if t == gguf.GGML_Q4_K:
            assert np.count_nonzero(p) == np.count_nonzero(W)


def test_reference_op_set(gpu):
    """RMSNorm / SiLU / Mul / RoPE — the reference CUDA backend's v1 ops."""
    import torch
    # tests/test_backend_cuda.cpp:36-76: x = 1..8, w = 1 + 0.1 i, WithinRel 1e-5
    x = np.arange(1, 9, dtype=np.float32)
    w = (1 + 0.1 * np.arange(8)).astype(np.float32)
    xd, wd = dev(x), dev(w)
    y = torch.zeros(8, device="cuda")
    assert gpu.af_rms_norm_f32(y.data_ptr(), xd.data_ptr(), wd.data_ptr(), 8, 1e-5, None) == 0
    inv = 1.0 / np.sqrt(np.float32((x * x).sum() / 8) + np.float32(1e-5))
    np.testing.assert_allclose(y.cpu().numpy(), x * inv * w, rtol=1e-5)
    rng = np.random.default_rng(2)
    a = rng.standard_normal(1000).astype(np.float32)
    b = rng.standard_normal(1000).astype(np.float32)
    ad, bd = dev(a), dev(b)
    o = torch.zeros(1000, device="cuda")
    assert gpu.af_silu_f32(o.data_ptr(), ad.data_ptr(), 1000, None) == 0
    np.testing.assert_allclose(o.cpu().numpy(), a / (1 + np.exp(-a)), rtol=1e-5, atol=1e-6)
    assert gpu.af_mul_f32(o.data_ptr(), ad.data_ptr(), bd.data_ptr(), 1000, None) == 0
    np.testing.assert_allclose(o.cpu().numpy(), a * b, rtol=1e-6)
    q = rng.standard_normal(4 * 64).astype(np.float32)
    qd = dev(q)
    assert gpu.af_rope_f32(qd.data_ptr(), 4, 64, 17, 10000.0, None) == 0
    c, s = COracle().rope_tables(64, 10000.0, 18)
    qh = q.reshape(4, 64)
    exp = np.concatenate([qh[:, :32] * c[17] - qh[:, 32:] * s[17], qh[:, :32] * s[17] + qh[:, 32:] * c[17]], 1)
    np.testing.assert_allclose(qd.cpu().numpy().reshape(4, 64), exp, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("rows,cols", [(2048, 2048), (1000, 4096), (37, 512)])
def test_q4km_gemv_on_raw_gguf_rows(gpu, rows, cols):
    """af_q4km_gemv_f32 takes the reference backend's arguments — raw GGUF
    Q4_K_M rows and row_bytes (cuda_kernels.hpp:13-19) — and matches the
    oracle's F32 GEMV; a row_bytes that is not the GGUF row size is refused."""
    import torch
    rng = np.random.default_rng(rows + cols)
    W = gguf.random_q4k(rng, rows * cols // 256).reshape(-1)
    x = rng.standard_normal(cols).astype(np.float32)
    wd, xd = dev(W), dev(x)
    y = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    rb = cols // 256 * 144
    assert gpu.af_q4km_gemv_f32(y.data_ptr(), wd.data_ptr(), xd.data_ptr(), rows, cols, rb, None) == 0
    got = y.cpu().numpy()
    want = COracle().gemv(W, gguf.GGML_Q4_K, x, rows)
    assert rel_l2(got, want) < GEMV_TOL and rel_l2(got, want) < 1e-4
    assert gpu.af_q4km_gemv_f32(y.data_ptr(), wd.data_ptr(), xd.data_ptr(), rows, cols, rb + 16, None) != 0
    assert b"row_bytes" in gpu.af_last_error()
