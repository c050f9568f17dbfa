"""The CPU oracle (oracle/af_oracle.c) pinned against the reference's own code.

Golden fixtures in tests/golden/ come from the reference compiled in place
(tests/golden/make_golden.py).  Where oracle/_ref/libaxref.so exists, the
oracle is also checked against it directly.
"""
import glob
import hashlib
import os

import numpy as np
import pytest

from helpers import model_path, rel_l2
from llm_core_b200 import gguf
from oracle import COracle, RefLib

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def orc():
    return COracle()


@pytest.mark.parametrize("fx", sorted(glob.glob(os.path.join(GOLD, "gemv_*.npz"))), ids=os.path.basename)
def test_oracle_gemv_matches_reference_fixture(orc, fx):
    z = np.load(fx)
    y = orc.gemv(z["W"], int(z["ggml_type"]), z["x"], int(z["rows"]))
    # same fp32 math, different summation order than the AVX2 kernel
    assert rel_l2(y, z["y"]) < 1e-5
    # the reference's production (Q8_0-activation) path is 4e-3..9e-3 away:
    # it cannot be the parity target for a 2e-3 bound
    assert rel_l2(z["y_q8"], z["y"]) > 2e-3


def test_rms_norm_known_answer(orc):
    # tests/test_backend_x86.cpp:84-116 of the reference: x = 1..8, w = 1
    import ctypes as C
    x = np.arange(1, 9, dtype=np.float32)
    w = np.ones(8, np.float32)
    y = np.zeros(8, np.float32)
    fp = C.POINTER(C.c_float)
    orc.lib.afo_rms_norm(y.ctypes.data_as(fp), x.ctypes.data_as(fp), w.ctypes.data_as(fp), 8, C.c_float(1e-5))
    rms = np.sqrt(np.float32(204.0 / 8.0) + np.float32(1e-5))
    np.testing.assert_allclose(y, x / rms, rtol=1e-4)


def test_dequant_matches_dot(orc):
    rng = np.random.default_rng(3)
    for t, gen in ((gguf.GGML_Q4_K, gguf.random_q4k), (gguf.GGML_Q6_K, gguf.random_q6k)):
        W = gen(rng, 4 * 3).reshape(-1)  # 4 rows x 768 cols
        x = rng.standard_normal(768).astype(np.float32)
        deq = orc.dequant_rows(W, t, 4, 768)
        assert rel_l2(deq @ x, orc.gemv(W, t, x, 4)) < 1e-5


@pytest.mark.parametrize("fx", ["model_tiny", "model_tiny_qwen"])
def test_oracle_forward_matches_reference_fixture(orc, fx):
    z = np.load(os.path.join(GOLD, fx + ".npz"))
    path = model_path(str(z["preset"]), int(z["seed"]))
    h = hashlib.sha256(open(path, "rb").read()).hexdigest()
    assert h == str(z["sha256"]), "seeded GGUF writer no longer reproduces the fixture's bytes"
    orc.open_model(gguf.GGUFReader(path))
    for p, tok in enumerate(z["tokens"]):
        lg = orc.forward_token(int(tok), p)
        assert rel_l2(lg, z["logits"][p]) < 1e-5
        assert int(np.argmax(lg)) == int(np.argmax(z["logits"][p]))


@pytest.mark.parametrize("fx", ["model_tiny", "model_tiny_qwen"])
def test_oracle_greedy_matches_reference_fixture(orc, fx):
    z = np.load(os.path.join(GOLD, fx + ".npz"))
    path = model_path(str(z["preset"]), int(z["seed"]))
    orc.open_model(gguf.GGUFReader(path))
    gen, _ = orc.generate_greedy(z["prompt"].tolist(), len(z["greedy"]))
    assert gen == z["greedy"].tolist()


@pytest.mark.skipif(not RefLib.available(), reason="oracle/_ref not built here")
def test_oracle_against_compiled_reference(orc):
    ref = RefLib()
    rng = np.random.default_rng(99)
    for t, gen in ((gguf.GGML_Q4_K, gguf.random_q4k), (gguf.GGML_Q6_K, gguf.random_q6k)):
        for rows, cols in ((96, 2048), (33, 5632), (8, 11008)):
            W = gen(rng, rows * cols // 256).reshape(-1)
            x = rng.standard_normal(cols).astype(np.float32)
            assert rel_l2(orc.gemv(W, t, x, rows), ref.gemv_f32(W, t, x, rows)) < 1e-5
            assert rel_l2(ref.gemv_f32(W, t, x, rows, scalar=True), ref.gemv_f32(W, t, x, rows)) < 1e-5
    path = model_path("tiny-qwen", 5)
    orc.open_model(gguf.GGUFReader(path))
    ref.open(path, threads=2)
    for p, tok in enumerate([1, 3, 900, 42]):
        assert rel_l2(orc.forward_token(tok, p), ref.forward_token(tok, p)) < 1e-5


@pytest.mark.skipif(not RefLib.available(), reason="oracle/_ref not built here")
@pytest.mark.parametrize("preset,seed", [("tiny", 1), ("tiny-qwen", 4), ("small", 5)])
def test_reference_prompt_paths(preset, seed):
    """The reference's own prompt paths on the prompts the batched-prefill GPU
    test uses: in F32 mode llama_forward_batch equals the per-token forward
    exactly; its shipped Q8_0 batched prefill (gemm_q4k_q8_avx2_range) differs
    from the F32 per-token forward by about 2.5e-3 .. 1.1e-2 in the last logits
    (bounded here by 2e-2) — the scale against which the B200 batched pass's
    f16 GEMM (≤ 5e-3) sits."""
    from helpers import model_path
    from llm_core_b200.engine import read_config
    path = model_path(preset, seed)
    cfg = read_config(path)
    rng = np.random.default_rng(100 + seed)
    prompt = [1] + rng.integers(0, cfg.vocab, 40).tolist()

    def run(f32, batched):
        r = RefLib()
        r.open(path, threads=4, f32_mode=f32)
        if batched:
            lg = r.forward_batch(prompt, 0)
        else:
            for i, t in enumerate(prompt):
                lg = r.forward_token(t, i)
        r.close()
        return lg

    tok = run(True, False)
    assert np.array_equal(run(True, True), tok)
    dev = float(np.linalg.norm(run(False, True) - tok) / np.linalg.norm(tok))
    assert dev < 2e-2, dev
