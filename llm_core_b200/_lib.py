"""ctypes binding of libaf_b200.so (the C ABI declared in include/af_b200.h).

The library is built in-tree (llm_core_b200/libaf_b200.so, see build.py).  There
is no fallback: if it is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.environ.get("AF_LIB_PATH") or os.path.join(HERE, "libaf_b200.so")
HEADER = os.path.join(ROOT, "include", "af_b200.h")

_lib = None


class AfError(RuntimeError):
    pass


class ModelConfig(C.Structure):
    """af_model_config (include/af_b200.h)."""
    _fields_ = [(n, C.c_int) for n in ("n_layer", "n_embd", "n_head", "n_kv_head", "ffn", "vocab", "n_ctx")] + \
               [("eps", C.c_float), ("theta", C.c_float), ("qk_norm_order", C.c_int),
                ("bos_id", C.c_int), ("eos_id", C.c_int)]


class Sampling(C.Structure):
    """af_sampling (include/af_b200.h)."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float), ("rep_penalty", C.c_float),
                ("rep_last_n", C.c_int)]


class GemvFusedArgs(C.Structure):
    """af_gemv_fused_args (include/af_b200.h)."""
    _fields_ = [("w", C.c_void_p * 3), ("type", C.c_int * 3), ("rows", C.c_int * 3), ("y", C.c_void_p * 3),
                ("bias", C.c_void_p * 3), ("nseg", C.c_int), ("cols", C.c_int), ("x", C.c_void_p),
                ("x_add", C.c_void_p), ("x_store", C.c_void_p), ("norm_w", C.c_void_p), ("eps", C.c_float),
                ("epi", C.c_int), ("resid", C.c_void_p), ("argmax", C.c_void_p), ("argmax_base", C.c_int)]


EPI_STORE, EPI_SWIGLU, EPI_RESID, EPI_ARGMAX = 0, 1, 2, 3


def header_symbols() -> list[str]:
    """Every function the public header declares."""
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(af_\w+)\s*\(", txt, re.M)))


def load() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise AfError(f"{LIB_PATH} is missing: build it with `python -m llm_core_b200.build`")
    # Load NCCL's soname from the same place torch does when torch is around,
    # so a process never maps two NCCL copies.
    try:
        import torch  # noqa: F401
    except Exception:
        pass
    lib = C.CDLL(LIB_PATH)
    vp, i, f, sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t
    fp, ip = C.POINTER(C.c_float), C.POINTER(C.c_int32)
    sig = {
        "af_last_error": (C.c_char_p, []),
        "af_device_error": (i, [C.POINTER(C.c_int), i]),
        "af_row_stride": (sz, [i, i]),
        "af_weight_bytes": (sz, [i, i, i]),
        "af_weight_pack": (i, [vp, vp, i, i, i, vp]),
        "af_weight_unpack": (i, [vp, vp, i, i, i, vp]),
        "af_gemv_f32": (i, [vp, vp, i, vp, i, i, vp]),
        "af_gemv_q8_f32": (i, [vp, vp, i, vp, i, i, vp]),
        "af_q4km_gemv_f32": (i, [vp, vp, vp, i, i, C.c_size_t, vp]),
        "af_prefill_gemm_f32": (i, [vp, vp, i, vp, i, i, i, vp]),
        "af_gemv_batched_f32": (i, [vp, vp, i, vp, i, i, i, vp]),
        "af_rms_norm_f32": (i, [vp, vp, vp, i, f, vp]),
        "af_gemv_fused": (i, [C.POINTER(GemvFusedArgs), vp]),
        "af_attention_decode_f32": (i, [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i, i, i, i, i, f, i, vp, vp,
                                        vp]),
        "af_attention_decode_f32_noalloc": (i, [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i, i, i, i, i, f, i,
                                                vp]),
        "af_silu_f32": (i, [vp, vp, i, vp]),
        "af_mul_f32": (i, [vp, vp, vp, i, vp]),
        "af_rope_f32": (i, [vp, i, i, i, f, vp]),
        "af_nccl_unique_id": (i, [vp]),
        "af_engine_create": (i, [C.POINTER(ModelConfig), i, i, i, vp, C.POINTER(vp)]),
        "af_engine_destroy": (i, [vp]),
        "af_engine_load_tensor": (i, [vp, C.c_char_p, i, C.POINTER(C.c_int64), i, vp, sz]),
        "af_gguf_read_config": (i, [C.c_char_p, i, C.POINTER(ModelConfig)]),
        "af_engine_load_gguf": (i, [vp, C.c_char_p]),
        "af_engine_finalize": (i, [vp]),
        "af_engine_set_q8_activations": (i, [vp, i]),
        "af_engine_step": (i, [vp, C.c_int32, C.c_int32, fp, ip]),
        "af_engine_prefill": (i, [vp, ip, i, C.c_int32, fp, ip]),
        "af_engine_prefill_batched": (i, [vp, ip, i, C.c_int32, fp, ip]),
        "af_engine_decode_greedy": (i, [vp, C.c_int32, C.c_int32, i, ip]),
        "af_engine_generate": (i, [vp, ip, i, i, ip, C.POINTER(C.c_int)]),
        "af_sample_f32": (i, [vp, i, vp, i, C.POINTER(Sampling), f, vp, vp]),
        "af_mt19937_uniform": (i, [C.c_uint32, i, fp]),
        "af_engine_sample": (i, [vp, C.POINTER(Sampling), ip, i, f, ip]),
        "af_engine_generate_sampled": (i, [vp, ip, i, i, C.POINTER(Sampling), fp, i, ip, C.POINTER(C.c_int)]),
        "af_engine_hidden": (i, [vp, fp]),
        "af_engine_kv": (i, [vp, i, i, i, fp]),
        "af_engine_profile": (i, [vp, C.c_int32, C.c_int32, i, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                  C.POINTER(C.c_int)]),
        "af_engine_stream": (vp, [vp]),
        "af_engine_kernels_per_step": (i, [vp]),
        "af_engine_weight_bytes": (sz, [vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str = ""):
    """Raise AfError for a non-zero cudaError_t, with the library's message."""
    if rc != 0:
        msg = load().af_last_error().decode(errors="replace")
        raise AfError(f"{what}: cudaError {rc}" + (f" ({msg})" if msg else ""))
