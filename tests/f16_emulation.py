"""Numpy emulation of the batched prompt pass's rounding (test helper).

The batched pass (af_engine_prefill_batched) rounds both operands of every
linear layer to f16 (the tcgen05 prefill GEMM); the per-token path keeps them
at f32 / 16-bit-quantised precision.  This module runs the reference forward
(llama_forward_batch, src/models/llama_model.cpp:1339-1462: RMSNorm, q/k/v +
bias, half-split RoPE, causal GQA softmax attention, SwiGLU, residuals) in
float64 on the oracle's dequantised weights twice — exact, and with f16
operands in the linear layers — and returns per-layer relative deviations of
the K and V cache rows, i.e. what that rounding alone predicts.
"""
from __future__ import annotations

import numpy as np

from llm_core_b200 import gguf
from oracle import COracle


def _rel(a, b) -> float:
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def kv_rounding_deviation(path: str, tokens, n_layers: int) -> list[tuple[float, float]]:
    orc = COracle()
    r = gguf.GGUFReader(path)
    cfg = gguf.ModelConfig.from_gguf(r)
    E, H, KV = cfg.n_embd, cfg.n_head, cfg.n_kv_head
    hd = E // H
    G = H // KV

    def mat(name):
        ti = r.get(name)
        return orc.dequant_rows(np.ascontiguousarray(r.data(name)), ti.ggml_type, ti.dims[1], ti.dims[0])

    def vec(name):
        return None if r.get(name) is None else np.array(r.data(name)).view(np.float32).astype(np.float64)

    T = len(tokens)
    inv = 1.0 / (cfg.theta ** (np.arange(0, hd, 2) / hd))
    ang = np.arange(T)[:, None] * inv[None, :]
    cos, sin = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]

    def rope(x):
        a, b = x[..., :hd // 2], x[..., hd // 2:]
        return np.concatenate([a * cos - b * sin, a * sin + b * cos], -1)

    def norm(x, w):
        return w * (x / np.sqrt((x * x).mean(-1, keepdims=True) + cfg.eps))

    def f16(a):
        return a.astype(np.float16).astype(np.float64)

    emb = mat("token_embd.weight")
    out = {}
    for mode in ("exact", "f16"):
        lin = (lambda X, W: X @ W.T) if mode == "exact" else (lambda X, W: f16(X) @ f16(W).T)
        x = emb[list(tokens)].astype(np.float64)
        rows = []
        for layer in range(min(n_layers, cfg.n_layer)):
            pre = f"blk.{layer}."
            xn = norm(x, vec(pre + "attn_norm.weight"))
            q, k, v = (lin(xn, mat(pre + f"attn_{m}.weight")) for m in "qkv")
            bq, bk, bv = (vec(pre + f"attn_{m}.bias") for m in "qkv")
            q, k, v = (t if b is None else t + b for t, b in ((q, bq), (k, bk), (v, bv)))
            q, k, v = rope(q.reshape(T, H, hd)), rope(k.reshape(T, KV, hd)), v.reshape(T, KV, hd)
            rows.append((k.reshape(T, -1), v.reshape(T, -1)))
            att = np.zeros((T, H, hd))
            mask = np.triu(np.full((T, T), -np.inf), 1)
            for h in range(H):
                s = q[:, h] @ k[:, h // G].T / np.sqrt(hd) + mask
                s = np.exp(s - s.max(-1, keepdims=True))
                att[:, h] = (s / s.sum(-1, keepdims=True)) @ v[:, h // G]
            x = x + lin(att.reshape(T, -1), mat(pre + "attn_output.weight"))
            xn = norm(x, vec(pre + "ffn_norm.weight"))
            g, u = lin(xn, mat(pre + "ffn_gate.weight")), lin(xn, mat(pre + "ffn_up.weight"))
            x = x + lin(g / (1 + np.exp(-g)) * u, mat(pre + "ffn_down.weight"))
        out[mode] = rows
    return [(_rel(fk, ek), _rel(fv, ev)) for (ek, ev), (fk, fv) in zip(out["exact"], out["f16"])]
