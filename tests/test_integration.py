"""The drop-in from the reference's side: the UNMODIFIED reference engine
(Engine::from_gguf, llama_generate, BackendRegistry / IBackend / IKernel)
with the B200 path bound in through its plugin API (integration/, linked into
oracle/_ref/libaxref_b200.so by oracle/ref.mk).

CPU: the "cuda" backend registers beside the reference's "cpu_x86" one and
declines to initialise without a device, as the reference's does.
GPU: llama_generate(engine{backend="cuda"}) reaches llama_cuda_generate and
returns the reference's F32-activation tokens (greedy and sampled); the
backend's MATMUL kernel takes raw GGUF blocks; RMS_NORM meets the
reference's own known answer (tests/test_backend_cuda.cpp:36-76)."""
import numpy as np
import pytest

from helpers import GEMV_TOL, model_path, rel_l2
from llm_core_b200 import gguf
from oracle import RefB200, RefLib

needs_ref = pytest.mark.skipif(not RefB200.available(), reason="reference sources were not built here")


@needs_ref
def test_cuda_backend_registers_beside_the_reference_backends():
    r = RefB200()
    assert r.has_backend("cuda")
    assert r.has_backend("cpu_x86")


def _device_present() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@needs_ref
@pytest.mark.skipif(_device_present(), reason="a device is present")
def test_cuda_backend_declines_without_a_device():
    with pytest.raises(RuntimeError, match="initialise"):
        RefB200().rms_norm(np.ones(8, np.float32), np.ones(8, np.float32), 1e-5)


@pytest.mark.gpu
@needs_ref
@pytest.mark.parametrize("preset,kw", [
    ("tiny", dict(temperature=0.0)),
    ("tiny-qwen", dict(temperature=0.0)),
    ("tiny", dict(temperature=0.8, top_k=40, top_p=0.95, rep_penalty=1.1, rep_last_n=64)),
    ("tiny", dict(temperature=1.0, top_k=40, top_p=1.0)),  # the reference's LlamaConfig defaults
])
def test_reference_llama_generate_on_the_cuda_backend(gpu, preset, kw):
    path = model_path(preset, 21)
    prompt = [3, 141, 59, 26, 5, 35]
    max_new = 40
    ids, streamed = RefB200().generate(path, prompt, max_new, backend="cuda", **kw)
    ref = RefLib().open(path, threads=4, f32_mode=True)
    if kw.get("temperature", 1.0) > 0 or kw.get("rep_penalty", 1.0) != 1.0:
        want = ref.generate_sampled(prompt, max_new, kw.get("temperature", 1.0), kw.get("top_k", 40),
                                    kw.get("top_p", 1.0), kw.get("rep_penalty", 1.0), kw.get("rep_last_n", 64))
    else:
        want, _ = ref.generate_greedy(prompt, max_new)
    ref.close()
    assert ids == want
    assert streamed == ids  # on_token saw every emitted id, in order


@pytest.mark.gpu
@needs_ref
@pytest.mark.parametrize("ggml_type,rows,cols,T", [
    (gguf.GGML_Q4_K, 2048, 2048, 1),
    (gguf.GGML_Q4_K, 5632, 2048, 1),
    (gguf.GGML_Q6_K, 256, 2048, 1),
    (gguf.GGML_Q4_K, 1000, 4096, 1),   # rows not a multiple of the 16-row tile
    (gguf.GGML_Q4_K, 2048, 2048, 5),   # [T][K] activation: the tensor-core GEMM
])
def test_backend_matmul_kernel_on_raw_gguf_blocks(gpu, ggml_type, rows, cols, T):
    rng = np.random.default_rng(rows + cols + T)
    gen = gguf.random_q4k if ggml_type == gguf.GGML_Q4_K else gguf.random_q6k
    W = gen(rng, rows * cols // 256).reshape(-1)
    x = rng.standard_normal((T, cols) if T > 1 else cols).astype(np.float32)
    y = RefB200().matmul(W, ggml_type, x, rows)
    ref = RefLib()
    if T == 1:
        assert rel_l2(y, ref.gemv_f32(W, ggml_type, x, rows)) < GEMV_TOL
    else:
        for t in range(T):
            assert rel_l2(y[t], ref.gemv_f32(W, ggml_type, x[t], rows)) < GEMV_TOL


@pytest.mark.gpu
@needs_ref
def test_backend_rms_norm_known_answer(gpu):
    """x = [1..8], w = 1: y = x / sqrt(mean(x^2) + eps) (the reference's CUDA
    backend test, tests/test_backend_cuda.cpp:36-76)."""
    x = np.arange(1, 9, dtype=np.float32)
    y = RefB200().rms_norm(x, np.ones(8, np.float32), 1e-5)
    want = x / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-5)
    np.testing.assert_allclose(y, want, rtol=1e-5)
