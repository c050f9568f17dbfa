"""Test-infrastructure bindings for the CPU oracles (never the product path).

Two checkers live here:

* ``COracle`` — ``oracle/liboracle.so``, the C restatement in ``af_oracle.c``.
* ``RefLib``  — ``oracle/_ref/libaxref.so``, the reference's own CPU code
  compiled in place by ``oracle/ref.mk`` (present only where it was built).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm import this package.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(_HERE, "liboracle.so")
REF_SO = os.path.join(_HERE, "_ref", "libaxref.so")

_fp = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)


def _f(a: np.ndarray):
    return a.ctypes.data_as(_fp)


def _b(a: np.ndarray):
    return a.ctypes.data_as(_u8p)


def build_oracle() -> str:
    """Compile liboracle.so (gcc) if it is missing or stale."""
    src = os.path.join(_HERE, "af_oracle.c")
    if not os.path.exists(ORACLE_SO) or os.path.getmtime(ORACLE_SO) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE, "liboracle.so"])
    return ORACLE_SO


def build_ref(ref_root: str | None = None) -> str | None:
    """Compile oracle/_ref/libaxref.so from the reference sources when they are
    present (only in the build container): AXONFORGE_SRC, else a `reference`
    directory beside the repository; returns the path or None."""
    if ref_root is None:
        ref_root = os.environ.get("AXONFORGE_SRC") or os.path.join(os.path.dirname(os.path.dirname(_HERE)), "reference")
    if os.path.isdir(os.path.join(ref_root, "src")):
        repo = os.path.dirname(_HERE)
        subprocess.check_call(["make", "-s", "-j8", "-f", os.path.join("oracle", "ref.mk"),
                               f"REF={ref_root}"], cwd=repo)
    return REF_SO if os.path.exists(REF_SO) else None


class _Layer(C.Structure):
    _fields_ = [(n, _fp) for n in ("attn_norm", "ffn_norm", "bq", "bk", "bv", "q_norm", "k_norm")] + \
               [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd")] + \
               [(n, C.c_int) for n in ("tq", "tk", "tv", "to", "tg", "tu", "td")]


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layer", "n_embd", "n_head", "n_kv_head", "ffn", "vocab", "n_ctx")] + \
               [("eps", C.c_float), ("theta", C.c_float), ("qk_norm_order", C.c_int)]


class COracle:
    """The C restatement: kernels and a whole-model forward over a GGUF."""

    def __init__(self, threads: int | None = None):
        self.lib = C.CDLL(build_oracle())
        L = self.lib
        L.afo_q4k_dot_row.restype = C.c_float
        L.afo_q6k_dot_row.restype = C.c_float
        L.afo_f16_to_f32.restype = C.c_float
        L.afo_create.restype = C.c_void_p
        L.afo_create.argtypes = [C.POINTER(_Cfg)]
        L.afo_set_global.argtypes = [C.c_void_p, C.c_void_p, C.c_int, _fp, C.c_void_p, C.c_int]
        L.afo_set_layer.argtypes = [C.c_void_p, C.c_int, C.POINTER(_Layer)]
        L.afo_forward_token.argtypes = [C.c_void_p, C.c_int, C.c_int, _fp]
        L.afo_destroy.argtypes = [C.c_void_p]
        L.afo_hidden.argtypes = [C.c_void_p, _fp]
        L.afo_kv.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, _fp]
        L.afo_attention_decode.argtypes = [_fp] * 10 + [C.c_int] * 5 + [C.c_float, _fp]
        L.afo_set_threads(int(threads or min(os.cpu_count() or 1, 32)))
        self._model = None

    # -- kernels
    def gemv(self, W: np.ndarray, ggml_type: int, x: np.ndarray, rows: int) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(rows, np.float32)
        self.lib.afo_gemv(_f(y), W.ctypes.data_as(C.c_void_p), ggml_type, _f(x), rows, x.size)
        return y

    def quantize_q8(self, x: np.ndarray):
        """(d[k/32], q[k] int8): the Q8_0 blocks of x."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        d = np.zeros(x.size // 32, np.float32)
        q = np.zeros(x.size, np.int8)
        self.lib.afo_quantize_q8(_f(d), q.ctypes.data_as(C.c_void_p), _f(x), x.size)
        return d, q

    def sample(self, logits: np.ndarray, window, rep_penalty: float, top_k: int, top_p: float,
               temperature: float, r: float) -> int:
        """Penalty + sample() on a copy of `logits` with the uniform draw r."""
        lg = np.array(logits, dtype=np.float32)
        w = np.ascontiguousarray(window, dtype=np.int32)
        return self.lib.afo_sample(_f(lg), lg.size, w.ctypes.data_as(C.c_void_p), w.size, C.c_float(rep_penalty),
                                   top_k, C.c_float(top_p), C.c_float(temperature), C.c_float(r))

    def gemv_q8(self, W: np.ndarray, ggml_type: int, x: np.ndarray, rows: int) -> np.ndarray:
        """The production (Q8_0-input) GEMV."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(rows, np.float32)
        self.lib.afo_gemv_q8(_f(y), W.ctypes.data_as(C.c_void_p), ggml_type, _f(x), rows, x.size)
        return y

    def dequant_rows(self, W: np.ndarray, ggml_type: int, rows: int, cols: int) -> np.ndarray:
        from llm_core_b200.gguf import row_bytes
        out = np.zeros((rows, cols), np.float32)
        rb = row_bytes(ggml_type, cols)
        fn = self.lib.afo_q4k_row_to_f32 if ggml_type == 12 else self.lib.afo_q6k_row_to_f32
        Wc = np.ascontiguousarray(W)
        for r in range(rows):
            fn(_f(out[r]), C.c_void_p(Wc.ctypes.data + r * rb), cols)
        return out

    def rope_tables(self, head_dim: int, theta: float, n_pos: int):
        c = np.zeros((n_pos, head_dim // 2), np.float32)
        s = np.zeros_like(c)
        self.lib.afo_rope_tables(_f(c), _f(s), head_dim, C.c_float(theta), n_pos)
        return c, s

    def attention_decode(self, q, k, v, kc, vc, cos_row, sin_row, q_norm, k_norm, pos: int, H: int, KVH: int,
                         qk_norm_order: int, eps: float):
        """One token's attention (af_oracle.c afo_attention_decode, restating
        llama_model.cpp:1236-1272): returns the output [H*hd]; kc / vc (float32
        [n_ctx][KVH*hd], modified in place) receive the new row at pos."""
        hd = q.size // H
        q = np.array(q, np.float32)
        k = np.array(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        ao = np.zeros(H * hd, np.float32)
        att = np.zeros(pos + 1, np.float32)
        qn = np.ascontiguousarray(q_norm, np.float32) if q_norm is not None else None
        kn = np.ascontiguousarray(k_norm, np.float32) if k_norm is not None else None
        self.lib.afo_attention_decode(_f(ao), _f(q), _f(k), _f(v), _f(kc), _f(vc),
                                      _f(np.ascontiguousarray(cos_row, np.float32)),
                                      _f(np.ascontiguousarray(sin_row, np.float32)),
                                      _f(qn) if qn is not None else _fp(), _f(kn) if kn is not None else _fp(),
                                      pos, H, KVH, hd, qk_norm_order, C.c_float(eps), _f(att))
        return ao

    # -- model
    def open_model(self, reader, n_ctx: int | None = None):
        from llm_core_b200.gguf import ModelConfig
        cfg = ModelConfig.from_gguf(reader)
        nc = min(cfg.ctx, n_ctx or 4096)
        c = _Cfg(cfg.n_layer, cfg.n_embd, cfg.n_head, cfg.n_kv_head, cfg.ffn, cfg.vocab, nc,
                 cfg.eps, cfg.theta, cfg.qk_norm_order)
        self.close_model()
        h = self.lib.afo_create(C.byref(c))
        keep = []

        def ptr(name):
            ti = reader.get(name)
            if ti is None:
                return None, 0
            a = reader.data(name)
            keep.append(a)
            return a.ctypes.data, ti.ggml_type

        def fptr(name):
            p, _ = ptr(name)
            return C.cast(p, _fp) if p else _fp()

        emb, te = ptr("token_embd.weight")
        out, to = ptr("output.weight")
        self.lib.afo_set_global(h, emb, te, fptr("output_norm.weight"), out, to)
        for l in range(cfg.n_layer):
            p = f"blk.{l}."
            lw = _Layer()
            for fld, nm in (("attn_norm", "attn_norm.weight"), ("ffn_norm", "ffn_norm.weight"),
                            ("bq", "attn_q.bias"), ("bk", "attn_k.bias"), ("bv", "attn_v.bias"),
                            ("q_norm", "attn_q_norm.weight"), ("k_norm", "attn_k_norm.weight")):
                setattr(lw, fld, fptr(p + nm))
            for fld, tf, nm in (("wq", "tq", "attn_q"), ("wk", "tk", "attn_k"), ("wv", "tv", "attn_v"),
                                ("wo", "to", "attn_output"), ("wg", "tg", "ffn_gate"),
                                ("wu", "tu", "ffn_up"), ("wd", "td", "ffn_down")):
                a, t = ptr(p + nm + ".weight")
                setattr(lw, fld, a)
                setattr(lw, tf, t)
            self.lib.afo_set_layer(h, l, C.byref(lw))
        self._model, self._keep, self.cfg, self.n_ctx = h, keep, cfg, nc
        return cfg

    def forward_token(self, token: int, pos: int) -> np.ndarray:
        lg = np.zeros(self.cfg.vocab, np.float32)
        rc = self.lib.afo_forward_token(self._model, token, pos, _f(lg))
        if rc != 0:
            raise ValueError("oracle forward: token/pos out of range")
        return lg

    def hidden(self) -> np.ndarray:
        h = np.zeros(self.cfg.n_embd, np.float32)
        self.lib.afo_hidden(self._model, _f(h))
        return h

    def kv(self, layer: int, which_v: bool, n_pos: int) -> np.ndarray:
        kvd = self.cfg.n_kv_head * self.cfg.head_dim
        out = np.zeros((n_pos, kvd), np.float32)
        self.lib.afo_kv(self._model, layer, int(which_v), n_pos, _f(out))
        return out

    def generate_greedy(self, prompt, max_new: int, bos: int = 1):
        """BOS prepend + per-token prefill + argmax decode (llama_model.cpp:1562-1624)."""
        ids = list(prompt)
        if not ids or ids[0] != bos:
            ids = [bos] + ids
        for p, t in enumerate(ids):
            lg = self.forward_token(t, p)
        out, logits = [], []
        pos = len(ids)
        for _ in range(max_new):
            if pos >= self.n_ctx:
                break
            nxt = int(np.argmax(lg))
            out.append(nxt)
            logits.append(lg)
            lg = self.forward_token(nxt, pos)
            pos += 1
        return out, np.array(logits)

    def close_model(self):
        if self._model:
            self.lib.afo_destroy(self._model)
            self._model = None

    def __del__(self):
        try:
            self.close_model()
        except Exception:
            pass


class RefLib:
    """The reference's own CPU path (oracle/_ref/libaxref.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = L = C.CDLL(path)
        L.axref_open.restype = C.c_void_p
        L.axref_open.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int]
        L.axref_last_error.restype = C.c_char_p
        for fn in ("axref_close", "axref_vocab", "axref_n_ctx", "axref_bos", "axref_n_past"):
            getattr(L, fn).argtypes = [C.c_void_p]
        L.axref_forward_token.argtypes = [C.c_void_p, C.c_int, C.c_int, _fp]
        L.axref_forward_batch.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_int, _fp]
        L.axref_generate_greedy.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_int,
                                            C.POINTER(C.c_int32), _fp]
        L.axref_time_decode.restype = C.c_double
        L.axref_time_decode.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.axref_set_n_past.argtypes = [C.c_void_p, C.c_int]
        L.axref_hidden.argtypes = [C.c_void_p, _fp]
        _ip = C.POINTER(C.c_int32)
        L.axref_sample.argtypes = [_fp, C.c_int, _ip, C.c_int, C.c_float, C.c_int, C.c_float, C.c_float, C.c_uint32]
        L.axref_generate_sampled.argtypes = [C.c_void_p, _ip, C.c_int, C.c_int, C.c_float, C.c_int, C.c_float,
                                             C.c_float, C.c_int, _ip]
        L.axref_uniform.argtypes = [C.c_uint32, C.c_int, _fp]
        self.h = None

    @staticmethod
    def available(path: str = REF_SO) -> bool:
        return os.path.exists(path)

    def gemv_f32(self, W: np.ndarray, ggml_type: int, x: np.ndarray, rows: int, scalar=False):
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(rows, np.float32)
        name = {12: "axref_gemv_q4k_f32", 14: "axref_gemv_q6k_f32"}[ggml_type] + ("_scalar" if scalar else "")
        getattr(self.lib, name)(_f(y), _b(W), _f(x), rows, x.size)
        return y

    def quantize_q8(self, x: np.ndarray):
        """The reference's own Q8_0 quantiser: (d[k/32], q[k] int8)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        d = np.zeros(x.size // 32, np.float32)
        q = np.zeros(x.size, np.int8)
        self.lib.axref_quantize_q8(_f(x), x.size, _f(d), q.ctypes.data_as(C.c_void_p))
        return d, q

    def gemv_q8(self, W: np.ndarray, ggml_type: int, x: np.ndarray, rows: int, threads: int = 1):
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(rows, np.float32)
        self.lib.axref_gemv_q8_production(_f(y), _b(W), ggml_type, _f(x), rows, x.size, threads)
        return y

    def open(self, path: str, threads: int = 1, f32_mode: bool = True, max_ctx: int = 4096):
        self.close()
        self.h = self.lib.axref_open(path.encode(), threads, int(f32_mode), max_ctx)
        if not self.h:
            raise RuntimeError(self.lib.axref_last_error().decode())
        self.vocab = self.lib.axref_vocab(self.h)
        self.n_ctx = self.lib.axref_n_ctx(self.h)
        return self

    def forward_token(self, token: int, pos: int) -> np.ndarray:
        lg = np.zeros(self.vocab, np.float32)
        if self.lib.axref_forward_token(self.h, token, pos, _f(lg)) != 0:
            raise RuntimeError(self.lib.axref_last_error().decode())
        return lg

    def forward_batch(self, tokens, pos0: int) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        lg = np.zeros(self.vocab, np.float32)
        if self.lib.axref_forward_batch(self.h, t.ctypes.data_as(C.POINTER(C.c_int32)), t.size, pos0, _f(lg)) != 0:
            raise RuntimeError(self.lib.axref_last_error().decode())
        return lg

    def hidden(self, n_embd: int) -> np.ndarray:
        h = np.zeros(n_embd, np.float32)
        self.lib.axref_hidden(self.h, _f(h))
        return h

    def generate_greedy(self, prompt, max_new: int, want_logits: bool = False):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max_new, np.int32)
        lg = np.zeros((max_new, self.vocab), np.float32) if want_logits else None
        n = self.lib.axref_generate_greedy(self.h, p.ctypes.data_as(C.POINTER(C.c_int32)), p.size, max_new,
                                           out.ctypes.data_as(C.POINTER(C.c_int32)),
                                           _f(lg) if want_logits else _fp())
        if n < 0:
            raise RuntimeError(self.lib.axref_last_error().decode())
        return out[:n].tolist(), (lg[:n] if want_logits else None)

    def sample(self, logits: np.ndarray, window, rep_penalty: float, top_k: int, top_p: float,
               temperature: float, seed: int) -> int:
        """The reference's penalty + sample() on a copy of `logits`, rng mt19937(seed)."""
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        w = np.ascontiguousarray(window, dtype=np.int32)
        return self.lib.axref_sample(_f(lg), lg.size, w.ctypes.data_as(C.POINTER(C.c_int32)), w.size, rep_penalty,
                                     top_k, top_p, temperature, seed)

    def generate_sampled(self, prompt, max_new: int, temperature: float, top_k: int, top_p: float,
                         rep_penalty: float, rep_last_n: int):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        n = self.lib.axref_generate_sampled(self.h, p.ctypes.data_as(C.POINTER(C.c_int32)), p.size, max_new,
                                            temperature, top_k, top_p, rep_penalty, rep_last_n,
                                            out.ctypes.data_as(C.POINTER(C.c_int32)))
        if n < 0:
            raise RuntimeError(self.lib.axref_last_error().decode())
        return out[:n].tolist()

    def uniform(self, seed: int, n: int) -> np.ndarray:
        out = np.zeros(n, np.float32)
        self.lib.axref_uniform(seed, n, _f(out))
        return out

    def time_decode(self, first_token: int, steps: int) -> float:
        return self.lib.axref_time_decode(self.h, first_token, steps)

    def set_n_past(self, n: int):
        self.lib.axref_set_n_past(self.h, n)

    def close(self):
        if self.h:
            self.lib.axref_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


REF_B200_SO = os.path.join(_HERE, "_ref", "libaxref_b200.so")


class RefB200:
    """The UNMODIFIED reference engine with the B200 path bound in through its
    own plugin API (oracle/_ref/libaxref_b200.so, built by oracle/ref.mk from
    the reference sources, integration/ and oracle/integ_harness.cpp).  Test
    infrastructure: it shows the drop-in working from the reference's side."""

    def __init__(self, path: str = REF_B200_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = L = C.CDLL(path)
        _ip = C.POINTER(C.c_int32)
        L.axintg_last_error.restype = C.c_char_p
        L.axintg_has_backend.argtypes = [C.c_char_p]
        L.axintg_generate.argtypes = [C.c_char_p, C.c_char_p, _ip, C.c_int, C.c_int, C.c_float, C.c_int, C.c_float,
                                      C.c_float, C.c_int, _ip, _ip]
        L.axintg_matmul.argtypes = [C.c_char_p, C.c_int, C.c_void_p, C.c_int, C.c_int, _fp, C.c_int, _fp]
        L.axintg_rms_norm.argtypes = [C.c_char_p, _fp, _fp, C.c_int, C.c_float, _fp]

    @staticmethod
    def available(path: str = REF_B200_SO) -> bool:
        return os.path.exists(path)

    def has_backend(self, name: str) -> bool:
        return bool(self.lib.axintg_has_backend(name.encode()))

    def _err(self):
        return RuntimeError(self.lib.axintg_last_error().decode(errors="replace"))

    def generate(self, model_path: str, prompt, max_new: int, backend: str = "cuda", temperature: float = 1.0,
                 top_k: int = 40, top_p: float = 1.0, rep_penalty: float = 1.0, rep_last_n: int = 64):
        """llama_generate(Engine::from_gguf(path, {backend}), prompt, cfg); returns
        (ids, ids seen by cfg.on_token)."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        streamed = np.full(max(max_new, 1), -1, np.int32)
        n = self.lib.axintg_generate(model_path.encode(), backend.encode(), p.ctypes.data_as(C.POINTER(C.c_int32)),
                                     p.size, max_new, temperature, top_k, top_p, rep_penalty, rep_last_n,
                                     out.ctypes.data_as(C.POINTER(C.c_int32)),
                                     streamed.ctypes.data_as(C.POINTER(C.c_int32)))
        if n < 0:
            raise self._err()
        return out[:n].tolist(), streamed[:n].tolist()

    def matmul(self, W: np.ndarray, ggml_type: int, x: np.ndarray, rows: int, backend: str = "cuda"):
        """MATMUL through get_kernel(MATMUL, {type, F32})->execute on raw GGUF
        blocks; x is [cols] or [T][cols]."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0] if x.ndim == 2 else 1
        cols = x.shape[-1]
        y = np.zeros((T, rows) if x.ndim == 2 else rows, np.float32)
        if self.lib.axintg_matmul(backend.encode(), ggml_type, _b(W), rows, cols, _f(x), T, _f(y)) != 0:
            raise self._err()
        return y

    def rms_norm(self, x: np.ndarray, w: np.ndarray, eps: float, backend: str = "cuda"):
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        y = np.zeros_like(x)
        if self.lib.axintg_rms_norm(backend.encode(), _f(x), _f(w), x.size, eps, _f(y)) != 0:
            raise self._err()
        return y
