"""GGUF v3 reading and seeded random-init model writing.

The reader mirrors the reference loader's parse (src/loader/gguf_loader.cpp:84-163):
magic ``GGUF``, u32 version (2 or 3), i64 tensor / KV counts, typed KV pairs,
tensor infos ``(name, n_dims, i64 dims[n], i32 ggml_type, u64 offset)`` and a data
blob aligned to ``general.alignment`` (default 32).  Tensor byte sizes use the
exact block sizes of ``gguf_tensor_nbytes`` (include/axonforge/dtype.hpp:136-155),
not ``numel * element_size`` (the reference's ``Tensor::nbytes`` bug).

The writer produces the random-init Q4_K_M checkpoints the benchmark configs
name (the benchmark workloads): Q4_K everywhere except Q6_K for ``attn_v``, the
even-indexed ``ffn_down`` layers and ``output`` (or the tied ``token_embd``).
Bit fields are seeded and uniform: 4-bit quants 0-15, 6-bit scales/mins 0-63,
``d``/``dmin`` uniform in [1e-4, 1e-3] rounded to f16; Q6_K int8 scales 0-63.
The tensor-name table is the one ``build_weights`` resolves
(src/models/llama_model.cpp:973-1004).
"""
from __future__ import annotations

import hashlib
import os
import struct
from dataclasses import dataclass, field

import numpy as np

GGML_F32 = 0
GGML_F16 = 1
GGML_Q4_K = 12
GGML_Q6_K = 14

QK_K = 256
BLOCK_BYTES = {GGML_Q4_K: 144, GGML_Q6_K: 210}

# GGUF KV value type tags (dtype.hpp:94-109).
_T_U8, _T_I8, _T_U16, _T_I16, _T_U32, _T_I32, _T_F32, _T_BOOL, _T_STR, _T_ARR, _T_U64, _T_I64, _T_F64 = range(13)
_POD = {_T_U8: "<B", _T_I8: "<b", _T_U16: "<H", _T_I16: "<h", _T_U32: "<I", _T_I32: "<i",
        _T_F32: "<f", _T_BOOL: "<b", _T_U64: "<Q", _T_I64: "<q", _T_F64: "<d"}


def tensor_nbytes(ggml_type: int, numel: int) -> int:
    """Exact byte count (gguf_tensor_nbytes, dtype.hpp:136-155)."""
    if ggml_type == GGML_F32:
        return numel * 4
    if ggml_type == GGML_F16:
        return numel * 2
    if ggml_type in BLOCK_BYTES:
        return (numel + QK_K - 1) // QK_K * BLOCK_BYTES[ggml_type]
    raise ValueError(f"unsupported ggml type {ggml_type}")


def row_bytes(ggml_type: int, cols: int) -> int:
    return tensor_nbytes(ggml_type, cols)


# --------------------------------------------------------------------------- reader

@dataclass
class TensorInfo:
    name: str
    dims: tuple  # GGML order: dims[0] is the innermost (columns)
    ggml_type: int
    offset: int
    nbytes: int

    @property
    def rows(self) -> int:
        r = 1
        for d in self.dims[1:]:
            r *= d
        return r

    @property
    def cols(self) -> int:
        return self.dims[0]


class GGUFReader:
    """mmap-backed GGUF parser (gguf_loader.cpp:84-163)."""

    def __init__(self, path: str):
        self.path = path
        self._mm = np.memmap(path, dtype=np.uint8, mode="r")
        self._pos = 0
        self.kv: dict = {}
        self.tensors: dict[str, TensorInfo] = {}
        self.order: list[str] = []
        self._parse()

    def _take(self, n: int) -> bytes:
        if self._pos + n > self._mm.size:
            raise ValueError("GGUF: unexpected end of file (truncated)")
        b = bytes(self._mm[self._pos:self._pos + n])
        self._pos += n
        return b

    def _pod(self, fmt: str):
        return struct.unpack(fmt, self._take(struct.calcsize(fmt)))[0]

    def _str(self) -> str:
        n = self._pod("<Q")
        return self._take(n).decode("utf-8", errors="replace")

    def _value(self, tag: int):
        if tag == _T_STR:
            return self._str()
        if tag == _T_ARR:
            et = self._pod("<i")
            cnt = self._pod("<Q")
            if et == _T_STR:
                return [self._str() for _ in range(cnt)]
            if et not in _POD:
                raise ValueError("GGUF: nested ARRAY or unknown type in array")
            sz = struct.calcsize(_POD[et])
            raw = self._take(sz * cnt)
            return list(np.frombuffer(raw, dtype=np.dtype(_POD[et])))
        if tag not in _POD:
            raise ValueError(f"GGUF: unknown KV type {tag}")
        return self._pod(_POD[tag])

    def _parse(self):
        if self._take(4) != b"GGUF":
            raise ValueError("GGUF: invalid magic (not a GGUF file)")
        ver = self._pod("<I")
        if ver < 2 or ver > 3:
            raise ValueError(f"GGUF: unsupported version {ver} (supported: 2, 3)")
        n_t = self._pod("<q")
        n_kv = self._pod("<q")
        if n_t < 0 or n_kv < 0:
            raise ValueError("GGUF: negative tensor/kv counts")
        for _ in range(n_kv):
            k = self._str()
            tag = self._pod("<i")
            self.kv[k] = self._value(tag)
        align = int(self.kv.get("general.alignment", 32))
        infos = []
        for _ in range(n_t):
            name = self._str()
            nd = self._pod("<I")
            if nd > 4:
                raise ValueError(f"GGUF: tensor '{name}' has more than 4 dimensions")
            dims = tuple(self._pod("<q") for _ in range(nd))
            t = self._pod("<i")
            off = self._pod("<Q")
            numel = int(np.prod(dims)) if dims else 1
            infos.append(TensorInfo(name, dims, t, off, tensor_nbytes(t, numel)))
        base = (self._pos + align - 1) // align * align
        for ti in infos:
            ti.offset += base
            if ti.offset + ti.nbytes > self._mm.size:
                raise ValueError(f"GGUF: tensor '{ti.name}' extends past end of file")
            self.tensors[ti.name] = ti
            self.order.append(ti.name)

    def data(self, name: str) -> np.ndarray:
        ti = self.tensors[name]
        return self._mm[ti.offset:ti.offset + ti.nbytes]

    def get(self, name: str):
        return self.tensors.get(name)


# --------------------------------------------------------------------------- config

@dataclass
class ModelConfig:
    """Hyper-parameters as Engine::from_gguf reads them (src/engine.cpp:85-118)."""
    arch: str
    n_layer: int
    n_embd: int
    n_head: int
    n_kv_head: int
    ffn: int
    vocab: int
    ctx: int = 4096
    eps: float = 1e-5
    theta: float = 10000.0
    qkv_bias: bool = False
    tied: bool = False
    name: str = ""
    qk_norm: bool = False  # per-head attn_q_norm / attn_k_norm weights (qwen3, hunyuan-dense)

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    @property
    def qk_norm_order(self) -> int:
        # QkNormOrder at llama_model.cpp:1520-1522.
        return 2 if self.arch == "hunyuan-dense" else (1 if self.arch == "qwen3" else 0)

    @classmethod
    def from_gguf(cls, r: GGUFReader) -> "ModelConfig":
        arch = r.kv.get("general.architecture", "unknown")
        g = lambda k, d: r.kv.get(f"{arch}.{k}", d)
        n_head = int(g("attention.head_count", 0))
        toks = r.kv.get("tokenizer.ggml.tokens", [])
        return cls(
            arch=arch,
            n_layer=int(g("block_count", 0)),
            n_embd=int(g("embedding_length", 0)),
            n_head=n_head,
            n_kv_head=int(g("attention.head_count_kv", n_head)),
            ffn=int(g("feed_forward_length", 0)),
            vocab=len(toks),
            ctx=int(g("context_length", 4096)),
            eps=float(g("attention.layer_norm_rms_epsilon", 1e-5)),
            theta=float(g("rope.freq_base", 10000.0)),
            qkv_bias="blk.0.attn_q.bias" in r.tensors,
            tied="output.weight" not in r.tensors,
            qk_norm="blk.0.attn_q_norm.weight" in r.tensors,
        )


PRESETS = {
    # TinyLlama-1.1B Q4_K_M workload.
    "tinyllama": ModelConfig("llama", 22, 2048, 32, 4, 5632, 32000, 2048, 1e-5, 1e4, name="tinyllama-1.1b"),
    # Qwen2.5-3B Q4_K_M workload (q/k/v bias, tied Q6_K vocab).
    "qwen2.5-3b": ModelConfig("qwen2", 36, 2048, 16, 2, 11008, 151936, 32768, 1e-6, 1e6,
                              qkv_bias=True, tied=True, name="qwen2.5-3b"),
    # Llama-2-7B Q4_K_M workload (the headline bs=1 decode).
    "llama2-7b": ModelConfig("llama", 32, 4096, 32, 32, 11008, 32000, 4096, 1e-5, 1e4, name="llama-2-7b"),
    # Small shapes for CPU tests (same code paths; K multiples of 256).
    "tiny": ModelConfig("llama", 2, 256, 4, 2, 512, 512, 256, 1e-5, 1e4, name="tiny-llama"),
    "tiny-qwen": ModelConfig("qwen2", 2, 512, 4, 2, 768, 1000, 512, 1e-6, 1e6,
                             qkv_bias=True, tied=True, name="tiny-qwen2"),
    "small": ModelConfig("llama", 4, 1024, 8, 4, 2816, 4000, 1024, 1e-5, 1e4, name="small-llama"),
    # splits over 8 tensor-parallel ranks (8 kv heads, n_embd = 8 super-blocks;
    # ffn_down's 22 super-blocks split unevenly)
    "tp8": ModelConfig("llama", 3, 2048, 16, 8, 5632, 4000, 1024, 1e-5, 1e4, name="tp8-llama"),
    # Per-head Q/K RMSNorm before RoPE (qwen3) and after it (hunyuan-dense),
    # QkNormOrder at src/models/llama_model.cpp:1520-1522.
    "tiny-qwen3": ModelConfig("qwen3", 2, 512, 4, 2, 768, 1000, 512, 1e-6, 1e6, qk_norm=True, name="tiny-qwen3"),
    "tiny-hunyuan": ModelConfig("hunyuan-dense", 2, 512, 8, 2, 768, 1000, 512, 1e-5, 1e4, qk_norm=True,
                                name="tiny-hunyuan"),
}


# --------------------------------------------------------------------------- random blocks

def _f16_uniform(rng: np.random.Generator, n: int, lo=1e-4, hi=1e-3) -> np.ndarray:
    return rng.uniform(lo, hi, size=n).astype(np.float16).view(np.uint8).reshape(n, 2)


def random_q4k(rng: np.random.Generator, nblocks: int) -> np.ndarray:
    """Q4_K super-blocks (144 B): random qs and packed 6-bit scales/mins
    (uniform bytes give uniform 0-15 nibbles and 0-63 six-bit fields), d/dmin
    f16 uniform in [1e-4, 1e-3]."""
    b = np.frombuffer(rng.bytes(nblocks * 144), dtype=np.uint8).reshape(nblocks, 144).copy()
    b[:, 0:2] = _f16_uniform(rng, nblocks)
    b[:, 2:4] = _f16_uniform(rng, nblocks)
    return b


def random_q6k(rng: np.random.Generator, nblocks: int) -> np.ndarray:
    """Q6_K super-blocks (210 B): random ql/qh, int8 scales uniform 0-63, d f16."""
    b = np.frombuffer(rng.bytes(nblocks * 210), dtype=np.uint8).reshape(nblocks, 210).copy()
    b[:, 192:208] &= 63
    b[:, 208:210] = _f16_uniform(rng, nblocks)
    return b


def _seed_for(seed: int, name: str) -> int:
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little")


def model_tensor_table(cfg: ModelConfig):
    """(name, ggml_type, dims) for every tensor of the model, in write order."""
    E, F, V = cfg.n_embd, cfg.ffn, cfg.vocab
    KV = cfg.n_kv_head * cfg.head_dim
    t = []
    t.append(("token_embd.weight", GGML_Q6_K if cfg.tied else GGML_Q4_K, (E, V)))
    for l in range(cfg.n_layer):
        p = f"blk.{l}."
        t.append((p + "attn_norm.weight", GGML_F32, (E,)))
        t.append((p + "attn_q.weight", GGML_Q4_K, (E, E)))
        t.append((p + "attn_k.weight", GGML_Q4_K, (E, KV)))
        t.append((p + "attn_v.weight", GGML_Q6_K, (E, KV)))
        if cfg.qkv_bias:
            t.append((p + "attn_q.bias", GGML_F32, (E,)))
            t.append((p + "attn_k.bias", GGML_F32, (KV,)))
            t.append((p + "attn_v.bias", GGML_F32, (KV,)))
        if cfg.qk_norm:
            t.append((p + "attn_q_norm.weight", GGML_F32, (cfg.head_dim,)))
            t.append((p + "attn_k_norm.weight", GGML_F32, (cfg.head_dim,)))
        t.append((p + "attn_output.weight", GGML_Q4_K, (E, E)))
        t.append((p + "ffn_norm.weight", GGML_F32, (E,)))
        t.append((p + "ffn_gate.weight", GGML_Q4_K, (E, F)))
        t.append((p + "ffn_up.weight", GGML_Q4_K, (E, F)))
        # "half of the ffn_down layers" in Q6_K: the even-indexed ones.
        t.append((p + "ffn_down.weight", GGML_Q6_K if l % 2 == 0 else GGML_Q4_K, (F, E)))
    t.append(("output_norm.weight", GGML_F32, (E,)))
    if not cfg.tied:
        t.append(("output.weight", GGML_Q6_K, (E, V)))
    return t


def random_tensor(name: str, ggml_type: int, dims, seed: int) -> np.ndarray:
    rng = np.random.default_rng(_seed_for(seed, name))
    numel = int(np.prod(dims))
    if ggml_type == GGML_Q4_K:
        return random_q4k(rng, numel // QK_K).reshape(-1)
    if ggml_type == GGML_Q6_K:
        return random_q6k(rng, numel // QK_K).reshape(-1)
    if name.endswith(".bias"):
        return rng.normal(0.0, 0.02, size=numel).astype(np.float32).view(np.uint8)
    if name.endswith(("attn_q_norm.weight", "attn_k_norm.weight")):
        # per-head norm weights away from 1 so that applying them (or not) shows
        return rng.uniform(0.5, 1.5, size=numel).astype(np.float32).view(np.uint8)
    return np.ones(numel, dtype=np.float32).view(np.uint8)  # norm weights


# --------------------------------------------------------------------------- writer

def _w_str(f, s: str):
    b = s.encode("utf-8")
    f.write(struct.pack("<Q", len(b)))
    f.write(b)


def _w_kv(f, key: str, val):
    _w_str(f, key)
    if isinstance(val, str):
        f.write(struct.pack("<i", _T_STR)); _w_str(f, val)
    elif isinstance(val, list):
        f.write(struct.pack("<i", _T_ARR))
        if val and isinstance(val[0], str):
            f.write(struct.pack("<iQ", _T_STR, len(val)))
            for s in val:
                _w_str(f, s)
        else:
            f.write(struct.pack("<iQ", _T_I32, len(val)))
            f.write(np.asarray(val, dtype=np.int32).tobytes())
    elif isinstance(val, float):
        f.write(struct.pack("<if", _T_F32, val))
    elif isinstance(val, tuple) and val[0] == "i32":
        f.write(struct.pack("<ii", _T_I32, val[1]))
    elif isinstance(val, tuple) and val[0] == "u32":
        f.write(struct.pack("<iI", _T_U32, val[1]))
    elif isinstance(val, int):
        f.write(struct.pack("<iQ", _T_U64, val))
    else:
        raise TypeError(f"unsupported KV value for {key}")


def write_gguf(path: str, kv: dict, tensors, align: int = 32):
    """tensors: iterable of (name, ggml_type, dims, producer) where producer()
    returns the tensor's bytes as a uint8 array of exactly tensor_nbytes."""
    tensors = list(tensors)
    kv = dict(kv)
    kv["general.alignment"] = ("u32", align)
    offs, off = [], 0
    for name, t, dims, _ in tensors:
        offs.append(off)
        off += tensor_nbytes(t, int(np.prod(dims)))
        off = (off + align - 1) // align * align
    with open(path, "wb") as f:
        f.write(b"GGUF")
        f.write(struct.pack("<Iqq", 3, len(tensors), len(kv)))
        for k, v in kv.items():
            _w_kv(f, k, v)
        for (name, t, dims, _), o in zip(tensors, offs):
            _w_str(f, name)
            f.write(struct.pack("<I", len(dims)))
            for d in dims:
                f.write(struct.pack("<q", d))
            f.write(struct.pack("<iQ", t, o))
        pos = f.tell()
        base = (pos + align - 1) // align * align
        f.write(b"\0" * (base - pos))
        for (name, t, dims, prod), o in zip(tensors, offs):
            cur = f.tell() - base
            if cur < o:
                f.write(b"\0" * (o - cur))
            data = prod()
            assert data.nbytes == tensor_nbytes(t, int(np.prod(dims))), name
            f.write(data.tobytes())


def model_kv(cfg: ModelConfig) -> dict:
    a = cfg.arch
    return {
        "general.architecture": a,
        "general.name": cfg.name or a,
        f"{a}.block_count": ("u32", cfg.n_layer),
        f"{a}.embedding_length": ("u32", cfg.n_embd),
        f"{a}.feed_forward_length": ("u32", cfg.ffn),
        f"{a}.attention.head_count": ("u32", cfg.n_head),
        f"{a}.attention.head_count_kv": ("u32", cfg.n_kv_head),
        f"{a}.context_length": ("u32", cfg.ctx),
        f"{a}.attention.layer_norm_rms_epsilon": float(cfg.eps),
        f"{a}.rope.freq_base": float(cfg.theta),
        "tokenizer.ggml.model": "llama",
        "tokenizer.ggml.tokens": [f"<t{i}>" for i in range(cfg.vocab)],
        "tokenizer.ggml.bos_token_id": ("i32", 1),
        # An id that can never be sampled, so random decoding never stops early.
        "tokenizer.ggml.eos_token_id": ("i32", -1),
    }


def write_random_model(path: str, cfg: ModelConfig | str, seed: int = 0) -> ModelConfig:
    """Write a seeded random-init Q4_K_M GGUF for `cfg` (a ModelConfig or a
    PRESETS key).  Deterministic in (cfg, seed)."""
    if isinstance(cfg, str):
        cfg = PRESETS[cfg]
    table = model_tensor_table(cfg)
    tensors = [(n, t, d, (lambda n=n, t=t, d=d: random_tensor(n, t, d, seed))) for n, t, d in table]
    tmp = path + ".tmp"
    write_gguf(tmp, model_kv(cfg), tensors)
    os.replace(tmp, path)
    return cfg


def model_weight_bytes(cfg: ModelConfig) -> int:
    """Per-token weight bytes a decode step streams: every matrix once
    (the embedding row read is negligible and excluded)."""
    total = 0
    for name, t, dims in model_tensor_table(cfg):
        if name == "token_embd.weight" and not cfg.tied:
            continue
        if t == GGML_F32:
            continue
        total += tensor_nbytes(t, int(np.prod(dims)))
    return total
