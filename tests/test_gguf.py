"""GGUF reader/writer (loader semantics of src/loader/gguf_loader.cpp:84-163)."""
import os
import struct

import numpy as np
import pytest

from llm_core_b200 import gguf


def test_weight_bytes_per_token_match_the_blueprint():
    # per-token weight bytes of the three decode configs
    assert gguf.model_weight_bytes(gguf.PRESETS["tinyllama"]) == 634_441_728
    assert gguf.model_weight_bytes(gguf.PRESETS["qwen2.5-3b"]) == 1_925_412_864
    assert gguf.model_weight_bytes(gguf.PRESETS["llama2-7b"]) == 4_074_676_224


def test_exact_block_sizes():
    # gguf_tensor_nbytes (dtype.hpp:136-155), not numel * element size
    assert gguf.tensor_nbytes(gguf.GGML_Q4_K, 4096 * 4096) == 4096 * 16 * 144
    assert gguf.tensor_nbytes(gguf.GGML_Q6_K, 4096 * 11008) == 4096 * 43 * 210
    assert gguf.tensor_nbytes(gguf.GGML_F32, 7) == 28


def test_round_trip(tmp_path):
    p = str(tmp_path / "m.gguf")
    cfg = gguf.write_random_model(p, "tiny", seed=7)
    r = gguf.GGUFReader(p)
    c2 = gguf.ModelConfig.from_gguf(r)
    assert (c2.n_layer, c2.n_embd, c2.n_head, c2.n_kv_head, c2.ffn, c2.vocab) == \
        (cfg.n_layer, cfg.n_embd, cfg.n_head, cfg.n_kv_head, cfg.ffn, cfg.vocab)
    assert r.kv["tokenizer.ggml.eos_token_id"] == -1
    for name, t, dims in gguf.model_tensor_table(cfg):
        ti = r.tensors[name]
        assert ti.ggml_type == t and ti.dims == tuple(dims)
        assert ti.offset % 32 == 0
        assert np.array_equal(r.data(name), gguf.random_tensor(name, t, dims, 7))
    # bit-field distributions of the random blocks
    q = r.data("blk.0.attn_q.weight").reshape(-1, 144)
    d = q[:, 0:2].copy().view(np.float16).astype(np.float32)
    assert d.min() >= 1e-4 * 0.999 and d.max() <= 1e-3 * 1.001
    q6 = r.data("blk.0.attn_v.weight").reshape(-1, 210)
    assert q6[:, 192:208].max() <= 63


def test_errors(tmp_path):
    p = str(tmp_path / "m.gguf")
    gguf.write_random_model(p, "tiny", seed=1)
    raw = open(p, "rb").read()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"XXXX" + raw[4:])
    with pytest.raises(ValueError, match="magic"):
        gguf.GGUFReader(str(bad))
    bad.write_bytes(raw[:4] + struct.pack("<I", 7) + raw[8:])
    with pytest.raises(ValueError, match="version"):
        gguf.GGUFReader(str(bad))
    bad.write_bytes(raw[:200])
    with pytest.raises(ValueError, match="truncated|past end"):
        gguf.GGUFReader(str(bad))
    bad.write_bytes(raw[: len(raw) - 1000])
    with pytest.raises(ValueError, match="past end"):
        gguf.GGUFReader(str(bad))
