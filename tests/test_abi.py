"""The C-ABI library loads and exports every symbol include/af_b200.h declares;
host-side argument checks work without a GPU."""
import ctypes as C
import subprocess

import numpy as np
import pytest

from llm_core_b200 import _lib


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    syms = _lib.header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(lib, s), s
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.strip()}
    missing = [s for s in syms if s not in exported]
    assert not missing, missing


def test_row_stride():
    lib = _lib.load()
    assert lib.af_row_stride(12, 4096) == 16 * 144
    assert lib.af_row_stride(14, 4096) == 16 * 210                   # units are whole GGUF blocks
    assert lib.af_row_stride(14, 11008) == 43 * 210
    assert lib.af_row_stride(12, 100) == 0                           # not a multiple of 256
    assert lib.af_weight_bytes(12, 17, 4096) == 32 * 16 * 144          # whole 16-row tiles
    assert lib.af_weight_bytes(14, 16, 11008) == 16 * 43 * 210
    assert lib.af_weight_bytes(3, 16, 4096) == 0


def test_gemv_rejects_bad_arguments_without_touching_a_device():
    lib = _lib.load()
    assert lib.af_gemv_f32(None, None, 12, None, 4, 100, None) != 0   # cols % 256
    assert b"256" in lib.af_last_error()
    assert lib.af_gemv_f32(None, None, 3, None, 4, 256, None) != 0    # unsupported type


def test_other_gemv_entries_reject_bad_arguments_without_touching_a_device():
    lib = _lib.load()
    # the reference backend's raw-GGUF entry: row_bytes must be the dense Q4_K row
    assert lib.af_q4km_gemv_f32(None, None, None, 4, 256, 150, None) != 0
    assert b"row_bytes" in lib.af_last_error()
    assert lib.af_q4km_gemv_f32(None, None, None, 4, 100, 144, None) != 0          # cols % 256
    assert lib.af_q4km_gemv_f32(None, C.c_void_p(8), None, 4, 256, 144, None) != 0  # misaligned weights
    assert b"aligned" in lib.af_last_error()
    assert lib.af_q4km_gemv_f32(None, None, None, 0, 256, 144, None) == 0           # nothing to do
    # Q8_0-input GEMV
    assert lib.af_gemv_q8_f32(None, None, 3, None, 4, 256, None) != 0               # unsupported type
    assert lib.af_gemv_q8_f32(None, None, 12, None, 4, 12288 + 256, None) != 0      # K above the limit
    assert lib.af_gemv_q8_f32(None, None, 14, None, 0, 256, None) == 0
    # batched GEMV: 1..32 vectors
    assert lib.af_gemv_batched_f32(None, None, 12, None, 4, 256, 0, None) != 0
    assert lib.af_gemv_batched_f32(None, None, 12, None, 4, 256, 33, None) != 0
    assert b"n_vec" in lib.af_last_error()
    assert lib.af_gemv_batched_f32(None, None, 12, None, 4, 200, 4, None) != 0      # cols % 256
    assert lib.af_gemv_batched_f32(None, None, 12, None, 0, 256, 4, None) == 0


def test_prefill_gemm_rejects_bad_arguments_without_touching_a_device():
    lib = _lib.load()
    assert lib.af_prefill_gemm_f32(None, None, 12, None, 16, 100, 4, None) != 0   # cols % 256
    assert b"256" in lib.af_last_error()
    assert lib.af_prefill_gemm_f32(None, None, 3, None, 16, 256, 4, None) != 0    # unsupported type
    assert lib.af_prefill_gemm_f32(None, None, 12, None, 16, 256, -1, None) != 0  # negative token count
    assert lib.af_prefill_gemm_f32(None, C.c_void_p(8), 12, None, 16, 256, 4, None) != 0  # misaligned weights
    assert b"aligned" in lib.af_last_error()
    assert lib.af_prefill_gemm_f32(None, None, 12, None, 0, 256, 4, None) == 0    # nothing to do


def test_gguf_config_reader(tmp_path):
    from llm_core_b200 import gguf
    from llm_core_b200.engine import read_config
    p = str(tmp_path / "q.gguf")
    gguf.write_random_model(p, "tiny-qwen", seed=3)
    c = read_config(p, 4096)
    assert (c.n_layer, c.n_embd, c.n_head, c.n_kv_head, c.ffn, c.vocab, c.n_ctx) == (2, 512, 4, 2, 768, 1000, 512)
    assert abs(c.eps - 1e-6) < 1e-12 and c.theta == 1e6 and c.bos_id == 1 and c.eos_id == -1
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + b"\0" * 64)
    with pytest.raises(_lib.AfError, match="magic"):
        read_config(str(bad))


def test_sampler_draws_are_the_reference_stream():
    """af_mt19937_uniform is the reference sampler's rng stream
    (std::mt19937(42) + uniform_real_distribution<float>, llama_model.cpp:1560,
    1494-1495): known answer for the first draws, and the compiled reference
    when it is built."""
    from llm_core_b200.engine import mt19937_uniform
    from oracle import RefLib
    d = mt19937_uniform(4, 42)
    # first output of std::mt19937(42) is 1608637542; / 2^32 rounded to float
    assert d[0] == np.float32(np.float32(1608637542) / np.float32(4294967296.0))
    assert np.all((d >= 0) & (d < 1))
    if RefLib.available():
        np.testing.assert_array_equal(mt19937_uniform(1000, 7), RefLib().uniform(7, 1000))


def test_sampler_rejects_bad_arguments_without_touching_a_device():
    import ctypes as C
    s = _lib.Sampling(1.0, 40, 0.95, 1.0, 0)
    assert _lib.load().af_sample_f32(None, 100, None, 0, C.byref(s), 0.5, None, None) != 0


def test_engine_entries_reject_a_null_engine_without_touching_a_device():
    lib = _lib.load()
    i1 = (C.c_int32 * 1)()
    n = C.c_int(0)
    assert lib.af_engine_destroy(None) == 0
    assert lib.af_engine_load_gguf(None, b"x.gguf") != 0 and b"null" in lib.af_last_error()
    assert lib.af_engine_set_q8_activations(None, 1) != 0
    assert lib.af_engine_finalize(None) != 0
    for call in (lambda: lib.af_engine_step(None, 0, 0, None, i1),
                 lambda: lib.af_engine_prefill(None, i1, 1, 0, None, i1),
                 lambda: lib.af_engine_prefill_batched(None, i1, 1, 0, None, i1),
                 lambda: lib.af_engine_decode_greedy(None, 0, 0, 1, i1),
                 lambda: lib.af_engine_generate(None, i1, 1, 1, i1, C.byref(n)),
                 lambda: lib.af_engine_hidden(None, None),
                 lambda: lib.af_engine_kv(None, 0, 0, 1, None)):
        assert call() != 0
        assert b"not finalized" in lib.af_last_error()
