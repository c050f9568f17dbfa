"""CPU check of the batched prompt pass's error model (no GPU): a float64
emulation of the forward with f16 operands in the linear layers predicts the
K/V deviation the GPU test allows.  The random-init llama preset stays near
the f16 rounding itself; the qwen2 preset's near-hard attention amplifies it
about tenfold by layer 1, which is why deeper-layer rows are bounded by the
prediction rather than by a fixed tolerance."""
import numpy as np

from f16_emulation import kv_rounding_deviation
from helpers import model_path
from llm_core_b200.engine import read_config


def _prompt(path, seed):
    cfg = read_config(path)
    rng = np.random.default_rng(100 + seed)
    return [1] + rng.integers(0, cfg.vocab, 40).tolist()


def test_llama_preset_rounding_stays_small():
    path = model_path("tiny", 1)
    dev = kv_rounding_deviation(path, _prompt(path, 1)[:-1], 2)
    assert all(k < 1e-3 and v < 1e-3 for k, v in dev), dev


def test_qwen_preset_amplifies_rounding():
    path = model_path("tiny-qwen", 4)
    dev = kv_rounding_deviation(path, _prompt(path, 4)[:-1], 2)
    assert dev[0][1] < 1e-3 and dev[1][1] > 5 * dev[0][1], dev
