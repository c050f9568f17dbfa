"""Host-side mirror of the reference generation API on the B200 engine.

``LlamaCudaModel`` is the decode path behind ``llama_cuda_generate``
(include/axonforge/models/llama_cuda.hpp:25-28): it loads a GGUF (weights
byte-for-byte to the device), and ``generate`` follows llama_generate's
decode-loop semantics (src/models/llama_model.cpp:1562-1624), greedy or
sampled (repetition penalty, temperature / top-k / top-p on the device).  All compute is
in libaf_b200.so; this module only moves arguments across the C ABI.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Callable

import numpy as np

from . import _lib
from ._lib import ModelConfig, Sampling, check

SAMPLER_SEED = 42  # std::mt19937 rng(42) (src/models/llama_model.cpp:1560)


def mt19937_uniform(n: int, seed: int = SAMPLER_SEED) -> np.ndarray:
    """The reference sampler's uniform draws: std::uniform_real_distribution<float>(0, 1)
    over std::mt19937(seed), computed by the library's host C++ code."""
    out = np.zeros(max(n, 1), np.float32)
    check(_lib.load().af_mt19937_uniform(seed, n, out.ctypes.data_as(C.POINTER(C.c_float))), "af_mt19937_uniform")
    return out[:n]


def sampling_of(cfg: "LlamaConfig") -> Sampling:
    return Sampling(cfg.temperature, cfg.top_k, cfg.top_p, cfg.rep_penalty, cfg.rep_penalty_last_n)


@dataclass
class LlamaConfig:
    """LlamaConfig (include/axonforge/models/llama.hpp:17-36), same defaults:
    temperature 1 with top-k 40 samples; temperature <= 0 is greedy.  The
    sampler draws from std::mt19937(42) as the reference does."""
    max_new_tokens: int = 200
    temperature: float = 1.0
    top_k: int = 40
    verbose: bool = False
    n_threads: int = 0
    max_context_len: int = 4096
    top_p: float = 1.0
    rep_penalty: float = 1.0
    rep_penalty_last_n: int = 64
    on_token: Callable[[int], None] | None = field(default=None, repr=False)


def nccl_unique_id() -> bytes:
    lib = _lib.load()
    buf = C.create_string_buffer(128)
    check(lib.af_nccl_unique_id(buf), "af_nccl_unique_id")
    return buf.raw


def block_split(n: int, r: int, t: int) -> tuple[int, int]:
    """[lo, hi) of n items for rank r of t, the remainder to the low ranks —
    the engine's split of FFN super-blocks and vocabulary rows."""
    base, rem = divmod(n, t)
    lo = r * base + min(r, rem)
    return lo, lo + base + (1 if r < rem else 0)


@dataclass
class TpShard:
    """What tensor-parallel rank `rank` of `size` holds (af_engine_create's
    geometry): query / kv heads [h0, h1) / [kv0, kv1) (column-parallel QKV,
    row-parallel attn_output over the same heads), FFN values [f0, f1)
    (column-parallel gate/up, row-parallel down over whole 256-value
    super-blocks) and vocabulary rows [v0, v1) of the LM head."""
    h0: int
    h1: int
    kv0: int
    kv1: int
    f0: int
    f1: int
    v0: int
    v1: int


def tp_shard(cfg: ModelConfig, rank: int, size: int) -> TpShard:
    """Shard of one rank; raises ValueError for shapes the engine rejects."""
    if size < 1 or not 0 <= rank < size:
        raise ValueError("bad tp rank/size")
    if size > 1 and (cfg.n_kv_head % size or (cfg.n_embd // size) % 256):
        raise ValueError("tensor parallel needs n_kv_head and n_embd/256 divisible by tp_size")
    hl, kvl = cfg.n_head // size, cfg.n_kv_head // size
    f0, f1 = block_split(cfg.ffn // 256, rank, size)
    v0, v1 = block_split(cfg.vocab, rank, size)
    return TpShard(rank * hl, (rank + 1) * hl, rank * kvl, (rank + 1) * kvl, f0 * 256, f1 * 256, v0, v1)


def read_config(path: str, max_context_len: int = 4096) -> ModelConfig:
    lib = _lib.load()
    cfg = ModelConfig()
    check(lib.af_gguf_read_config(path.encode(), max_context_len, C.byref(cfg)), "af_gguf_read_config")
    return cfg


class LlamaCudaModel:
    """A GGUF model resident on one GPU (or one tensor-parallel rank)."""

    def __init__(self, path: str | None = None, *, config: ModelConfig | None = None, device: int = 0,
                 tp_rank: int = 0, tp_size: int = 1, nccl_id: bytes | None = None,
                 max_context_len: int = 4096, tensors=None, q8_activations: bool = False):
        self.lib = _lib.load()
        if config is None:
            if path is None:
                raise ValueError("need a GGUF path or a config")
            config = read_config(path, max_context_len)
        self.cfg = config
        h = C.c_void_p()
        idbuf = C.create_string_buffer(nccl_id, 128) if nccl_id else None
        check(self.lib.af_engine_create(C.byref(config), device, tp_rank, tp_size, idbuf, C.byref(h)),
              "af_engine_create")
        self.h = h
        self.tp_size = tp_size
        if tensors is not None:
            for name, ggml_type, dims, data in tensors:
                self.load_tensor(name, ggml_type, dims, data)
        elif path is not None:
            check(self.lib.af_engine_load_gguf(self.h, path.encode()), "af_engine_load_gguf")
        if q8_activations:
            check(self.lib.af_engine_set_q8_activations(self.h, 1), "af_engine_set_q8_activations")
        check(self.lib.af_engine_finalize(self.h), "af_engine_finalize")

    def load_tensor(self, name: str, ggml_type: int, dims, data: np.ndarray):
        d = (C.c_int64 * len(dims))(*dims)
        a = np.ascontiguousarray(data)
        check(self.lib.af_engine_load_tensor(self.h, name.encode(), ggml_type, d, len(dims),
                                             a.ctypes.data_as(C.c_void_p), a.nbytes), f"load {name}")

    # ------------------------------------------------------------ stepping
    def step(self, token: int, pos: int, want_logits: bool = True):
        lg = np.zeros(self.cfg.vocab, np.float32) if want_logits else None
        nxt = C.c_int32()
        check(self.lib.af_engine_step(self.h, token, pos,
                                      lg.ctypes.data_as(C.POINTER(C.c_float)) if want_logits else None,
                                      C.byref(nxt)), "af_engine_step")
        return nxt.value, lg

    def prefill(self, tokens, pos0: int = 0, want_logits: bool = True, batched: bool = False):
        """Feed a prompt; batched=True runs it as one batched pass on the
        tensor cores (af_engine_prefill_batched) instead of token by token."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        lg = np.zeros(self.cfg.vocab, np.float32) if want_logits else None
        nxt = C.c_int32()
        fn = self.lib.af_engine_prefill_batched if batched else self.lib.af_engine_prefill
        check(fn(self.h, t.ctypes.data_as(C.POINTER(C.c_int32)), t.size, pos0,
                 lg.ctypes.data_as(C.POINTER(C.c_float)) if want_logits else None,
                 C.byref(nxt)), "af_engine_prefill")
        return nxt.value, lg

    def decode_greedy(self, first_token: int, pos0: int, n_steps: int) -> np.ndarray:
        out = np.zeros(max(n_steps, 1), np.int32)
        check(self.lib.af_engine_decode_greedy(self.h, first_token, pos0, n_steps,
                                               out.ctypes.data_as(C.POINTER(C.c_int32))),
              "af_engine_decode_greedy")
        return out[:n_steps]

    def sample(self, cfg: LlamaConfig, window, r: float) -> int:
        """One sampling step from the last logits (af_engine_sample)."""
        w = np.ascontiguousarray(window, dtype=np.int32)
        nxt = C.c_int32()
        s = sampling_of(cfg)
        check(self.lib.af_engine_sample(self.h, C.byref(s), w.ctypes.data_as(C.POINTER(C.c_int32)), w.size,
                                        float(r), C.byref(nxt)), "af_engine_sample")
        return nxt.value

    def generate(self, prompt_ids, cfg: LlamaConfig | None = None) -> list[int]:
        cfg = cfg or LlamaConfig()
        p = np.ascontiguousarray(prompt_ids, dtype=np.int32)
        if p.size == 0:
            raise ValueError("llama_generate: empty prompt")
        out = np.zeros(max(cfg.max_new_tokens, 1), np.int32)
        n = C.c_int()
        if cfg.temperature <= 0 and cfg.rep_penalty == 1.0:
            # greedy: the device-fed decode loop
            check(self.lib.af_engine_generate(self.h, p.ctypes.data_as(C.POINTER(C.c_int32)), p.size,
                                              cfg.max_new_tokens, out.ctypes.data_as(C.POINTER(C.c_int32)),
                                              C.byref(n)), "af_engine_generate")
        else:
            draws = mt19937_uniform(cfg.max_new_tokens + 1) if cfg.temperature > 0 else np.zeros(1, np.float32)
            s = sampling_of(cfg)
            check(self.lib.af_engine_generate_sampled(self.h, p.ctypes.data_as(C.POINTER(C.c_int32)), p.size,
                                                      cfg.max_new_tokens, C.byref(s),
                                                      draws.ctypes.data_as(C.POINTER(C.c_float)), draws.size,
                                                      out.ctypes.data_as(C.POINTER(C.c_int32)), C.byref(n)),
                  "af_engine_generate_sampled")
        ids = out[:n.value].tolist()
        if cfg.on_token:
            for t in ids:
                cfg.on_token(t)
        return ids

    def hidden(self) -> np.ndarray:
        h = np.zeros(self.cfg.n_embd, np.float32)
        check(self.lib.af_engine_hidden(self.h, h.ctypes.data_as(C.POINTER(C.c_float))), "af_engine_hidden")
        return h

    def kv(self, layer: int, which_v: bool, n_pos: int) -> np.ndarray:
        kvd = self.cfg.n_kv_head // self.tp_size * (self.cfg.n_embd // self.cfg.n_head)
        out = np.zeros((n_pos, kvd), np.float32)
        check(self.lib.af_engine_kv(self.h, layer, int(which_v), n_pos, out.ctypes.data_as(C.POINTER(C.c_float))),
              "af_engine_kv")
        return out

    PROF_KINDS = ("embed", "gemv_qkv", "attention", "gemv_o", "gemv_gateup", "gemv_down", "gemv_lmhead",
                  "finalize", "nccl")

    def profile(self, token: int, pos0: int, n_steps: int) -> dict:
        """Per-launch-kind device ms / algorithmic bytes / launches over n_steps
        eager (event-bracketed) decode steps."""
        n = len(self.PROF_KINDS)
        ms = (C.c_double * n)()
        by = (C.c_double * n)()
        ct = (C.c_int * n)()
        check(self.lib.af_engine_profile(self.h, token, pos0, n_steps, ms, by, ct), "af_engine_profile")
        return {k: {"ms": ms[i], "bytes": by[i], "launches": ct[i]} for i, k in enumerate(self.PROF_KINDS)}

    @property
    def stream(self) -> int:
        return self.lib.af_engine_stream(self.h) or 0

    @property
    def kernels_per_step(self) -> int:
        return self.lib.af_engine_kernels_per_step(self.h)

    @property
    def weight_bytes(self) -> int:
        return self.lib.af_engine_weight_bytes(self.h)

    def close(self):
        if getattr(self, "h", None):
            self.lib.af_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def llama_cuda_generate(model: LlamaCudaModel, prompt_ids, cfg: LlamaConfig | None = None) -> list[int]:
    """llama_cuda_generate (include/axonforge/models/llama_cuda.hpp:25-28) on the B200 path."""
    return model.generate(prompt_ids, cfg)
