"""The fused GEMV variants and the decode-attention kernel in isolation, through
the C ABI, against numpy / C-oracle restatements of the reference's math."""
import ctypes as C

import numpy as np
import pytest

from helpers import dev, rel_l2
from llm_core_b200 import _lib, gguf
from oracle import COracle

pytestmark = pytest.mark.gpu
TIGHT = 1e-4


def mat(lib, rng, t, rows, cols):
    import torch
    gen = gguf.random_q4k if t == gguf.GGML_Q4_K else gguf.random_q6k
    W = gen(rng, rows * cols // 256).reshape(-1)
    src = dev(W)
    d = torch.empty(lib.af_weight_bytes(t, rows, cols), dtype=torch.uint8, device="cuda")
    assert lib.af_weight_pack(d.data_ptr(), src.data_ptr(), t, rows, cols, None) == 0
    return W, d


def rms(x, w, eps):
    x = x.astype(np.float32)
    return w * (x * (np.float32(1) / np.sqrt(np.float32((x * x).sum() / x.size) + np.float32(eps))))


def run(lib, a):
    import torch
    assert lib.af_gemv_fused(C.byref(a), None) == 0, lib.af_last_error()
    torch.cuda.synchronize()
    code = C.c_int()
    lib.af_device_error(C.byref(code), 1)
    assert code.value == 0


@pytest.mark.parametrize("E,kv", [(256, 128), (2048, 256), (4096, 4096)])
def test_norm_qkv_bias(gpu, E, kv):
    import torch
    rng = np.random.default_rng(E)
    orc = COracle()
    segs = [(gguf.GGML_Q4_K, E), (gguf.GGML_Q4_K, kv), (gguf.GGML_Q6_K, kv)]
    x = rng.standard_normal(E).astype(np.float32) * 3
    nw = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
    a = _lib.GemvFusedArgs()
    keep, exp, outs = [], [], []
    xn = rms(x, nw, 1e-5)
    for s, (t, rows) in enumerate(segs):
        W, Wd = mat(gpu, rng, t, rows, E)
        b = rng.normal(0, 0.02, rows).astype(np.float32)
        bd = dev(b)
        y = torch.zeros(rows, device="cuda")
        keep += [Wd, bd, y]
        a.w[s], a.type[s], a.rows[s], a.y[s], a.bias[s] = Wd.data_ptr(), t, rows, y.data_ptr(), bd.data_ptr()
        exp.append(orc.gemv(W, t, xn, rows) + b)
        outs.append(y)
    xd, nwd = dev(x), dev(nw)
    a.nseg, a.cols, a.x, a.norm_w, a.eps, a.epi = 3, E, xd.data_ptr(), nwd.data_ptr(), 1e-5, _lib.EPI_STORE
    run(gpu, a)
    for y, e in zip(outs, exp):
        assert rel_l2(y.cpu().numpy(), e) < TIGHT


@pytest.mark.parametrize("E,F", [(256, 512), (2048, 5632), (4096, 11008)])
def test_norm_gateup_swiglu(gpu, E, F):
    import torch
    rng = np.random.default_rng(F)
    orc = COracle()
    x = rng.standard_normal(E).astype(np.float32)
    nw = np.ones(E, np.float32)
    Wg, Wgd = mat(gpu, rng, gguf.GGML_Q4_K, F, E)
    Wu, Wud = mat(gpu, rng, gguf.GGML_Q4_K, F, E)
    h = torch.zeros(F, device="cuda")
    xd, nwd = dev(x), dev(nw)
    a = _lib.GemvFusedArgs()
    a.w[0], a.type[0], a.rows[0], a.y[0] = Wgd.data_ptr(), 12, F, h.data_ptr()
    a.w[1], a.type[1], a.rows[1] = Wud.data_ptr(), 12, F
    a.nseg, a.cols, a.x, a.norm_w, a.eps, a.epi = 2, E, xd.data_ptr(), nwd.data_ptr(), 1e-5, _lib.EPI_SWIGLU
    run(gpu, a)
    xn = rms(x, nw, 1e-5)
    g, u = orc.gemv(Wg, 12, xn, F), orc.gemv(Wu, 12, xn, F)
    assert rel_l2(h.cpu().numpy(), g / (1 + np.exp(-g)) * u) < TIGHT


@pytest.mark.parametrize("t", [gguf.GGML_Q4_K, gguf.GGML_Q6_K])
@pytest.mark.parametrize("E,K", [(256, 512), (4096, 11008), (2048, 2048)])
def test_residual_epilogue(gpu, t, E, K):
    rng = np.random.default_rng(E + K + t)
    orc = COracle()
    W, Wd = mat(gpu, rng, t, E, K)
    x = rng.standard_normal(K).astype(np.float32)
    r0 = rng.standard_normal(E).astype(np.float32) * 10
    xd, rd = dev(x), dev(r0)
    a = _lib.GemvFusedArgs()
    a.w[0], a.type[0], a.rows[0] = Wd.data_ptr(), t, E
    a.nseg, a.cols, a.x, a.epi, a.resid = 1, K, xd.data_ptr(), _lib.EPI_RESID, rd.data_ptr()
    run(gpu, a)
    exp = r0 + orc.gemv(W, t, x, E)
    assert rel_l2(rd.cpu().numpy(), exp) < TIGHT
    run(gpu, a)  # applied exactly once per call
    exp2 = exp + orc.gemv(W, t, x, E)
    assert rel_l2(rd.cpu().numpy(), exp2) < TIGHT


@pytest.mark.parametrize("V,E,t", [(512, 256, 14), (32000, 4096, 14), (1000, 512, 12)])
def test_norm_lmhead_argmax(gpu, V, E, t):
    import torch
    rng = np.random.default_rng(V)
    orc = COracle()
    W, Wd = mat(gpu, rng, t, V, E)
    x = rng.standard_normal(E).astype(np.float32)
    nw = np.ones(E, np.float32)
    xd, nwd = dev(x), dev(nw)
    y = torch.zeros(V, device="cuda")
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    a = _lib.GemvFusedArgs()
    a.w[0], a.type[0], a.rows[0], a.y[0] = Wd.data_ptr(), t, V, y.data_ptr()
    a.nseg, a.cols, a.x, a.norm_w, a.eps, a.epi = 1, E, xd.data_ptr(), nwd.data_ptr(), 1e-5, _lib.EPI_ARGMAX
    a.argmax, a.argmax_base = key.data_ptr(), 7
    run(gpu, a)
    exp = orc.gemv(W, t, rms(x, nw, 1e-5), V)
    got = y.cpu().numpy()
    assert rel_l2(got, exp) < TIGHT
    k = int(key.cpu().numpy()[0]) & 0xFFFFFFFFFFFFFFFF
    idx = 0xFFFFFFFF - (k & 0xFFFFFFFF)
    assert idx == 7 + int(np.argmax(got))


def test_residual_add_store(gpu):
    """x_add / x_store: input = x + x_add, stored once, then normalised."""
    import torch
    rng = np.random.default_rng(3)
    orc = COracle()
    E, R = 2048, 300
    W, Wd = mat(gpu, rng, 12, R, E)
    x = rng.standard_normal(E).astype(np.float32)
    xa = rng.standard_normal(E).astype(np.float32)
    nw = np.ones(E, np.float32)
    xd, xad, nwd = dev(x), dev(xa), dev(nw)
    st = torch.zeros(E, device="cuda")
    y = torch.zeros(R, device="cuda")
    a = _lib.GemvFusedArgs()
    a.w[0], a.type[0], a.rows[0], a.y[0] = Wd.data_ptr(), 12, R, y.data_ptr()
    a.nseg, a.cols, a.x, a.x_add, a.x_store = 1, E, xd.data_ptr(), xad.data_ptr(), st.data_ptr()
    a.norm_w, a.eps, a.epi = nwd.data_ptr(), 1e-5, _lib.EPI_STORE
    run(gpu, a)
    assert np.array_equal(st.cpu().numpy(), x + xa)
    assert rel_l2(y.cpu().numpy(), orc.gemv(W, 12, rms(x + xa, nw, 1e-5), R)) < TIGHT


def np_attention(q, kc, vc, pos, H, KVH, hd):
    G = H // KVH
    out = np.zeros(H * hd, np.float32)
    for h in range(H):
        kvh = h // G
        qh = q[h * hd:(h + 1) * hd].astype(np.float64)
        K = kc[:pos + 1, kvh * hd:(kvh + 1) * hd].astype(np.float64)
        V = vc[:pos + 1, kvh * hd:(kvh + 1) * hd].astype(np.float64)
        s = K @ qh / np.sqrt(hd)
        p = np.exp(s - s.max())
        out[h * hd:(h + 1) * hd] = (p / p.sum()) @ V
    return out


def rope(x, nh, hd, c, s):
    x = x.reshape(nh, hd).copy()
    h = hd // 2
    x0, x1 = x[:, :h].copy(), x[:, h:].copy()
    x[:, :h] = x0 * c - x1 * s
    x[:, h:] = x0 * s + x1 * c
    return x.reshape(-1)


@pytest.mark.parametrize("H,KVH,hd,pos,nsplit,qk", [
    (4, 2, 64, 0, 64, 0), (32, 4, 64, 300, 37, 0), (32, 32, 128, 200, 10, 0), (16, 2, 128, 4000, 64, 0),
    (16, 2, 128, 31, 1, 0), (8, 8, 128, 5, 3, 0),
    # GQA ratio 8 (the step kernel's widest group), and per-head Q/K RMSNorm
    # before RoPE (qwen3, 1) and after it (hunyuan, 2) with real norm weights
    (64, 8, 128, 700, 16, 0), (16, 2, 128, 130, 4, 1), (32, 4, 64, 77, 8, 2), (16, 2, 128, 2047, 32, 2),
])
def test_attention_decode(gpu, H, KVH, hd, pos, nsplit, qk):
    """af_attention_decode_f32 against the oracle's restatement of the
    reference attention block (oracle/af_oracle.c afo_attention_decode,
    src/models/llama_model.cpp:1236-1272)."""
    import torch
    rng = np.random.default_rng(pos + H + qk)
    n_ctx = 4096
    kvd = KVH * hd
    orc = COracle()
    c, s = orc.rope_tables(hd, 10000.0, n_ctx)
    kc = np.zeros((n_ctx, kvd), np.float32)
    vc = np.zeros((n_ctx, kvd), np.float32)
    kc[:pos] = rng.standard_normal((pos, kvd))
    vc[:pos] = rng.standard_normal((pos, kvd))
    q = rng.standard_normal(H * hd).astype(np.float32)
    k = rng.standard_normal(kvd).astype(np.float32)
    v = rng.standard_normal(kvd).astype(np.float32)
    qn = rng.uniform(0.5, 1.5, hd).astype(np.float32) if qk else None
    kn = rng.uniform(0.5, 1.5, hd).astype(np.float32) if qk else None
    d = {n: dev(a) for n, a in dict(q=q, k=k, v=v, kc=kc, vc=vc, c=c, s=s).items()}
    dqn, dkn = (dev(qn), dev(kn)) if qk else (None, None)
    posd = torch.tensor([pos], dtype=torch.int32, device="cuda")
    out = torch.zeros(H * hd, device="cuda")
    part = torch.zeros(H * nsplit * (hd + 2), device="cuda")
    cnt = torch.zeros(KVH, dtype=torch.int32, device="cuda")
    for _ in range(2):  # the counters must come back to zero
        assert gpu.af_attention_decode_f32(out.data_ptr(), d["q"].data_ptr(), d["k"].data_ptr(), d["v"].data_ptr(),
                                           d["kc"].data_ptr(), d["vc"].data_ptr(), d["c"].data_ptr(),
                                           d["s"].data_ptr(), dqn.data_ptr() if qk else None,
                                           dkn.data_ptr() if qk else None, posd.data_ptr(), H, KVH, hd, n_ctx, qk,
                                           1e-5, nsplit, part.data_ptr(), cnt.data_ptr(), None) == 0
        torch.cuda.synchronize()
        assert int(cnt.abs().sum()) == 0
    kc_o, vc_o = kc.copy(), vc.copy()
    exp = orc.attention_decode(q, k, v, kc_o, vc_o, c[pos], s[pos], qn, kn, pos, H, KVH, qk, 1e-5)
    np.testing.assert_allclose(d["kc"].cpu().numpy()[pos], kc_o[pos], atol=1e-5)
    assert np.array_equal(d["vc"].cpu().numpy()[pos], v)
    assert rel_l2(out.cpu().numpy(), exp) < 1e-5
    # the in-file double-precision restatement agrees for the plain case
    if qk == 0:
        qr = rope(q, H, hd, c[pos], s[pos])
        assert rel_l2(exp, np_attention(qr, kc_o, vc_o, pos, H, KVH, hd)) < 1e-5
