"""Tensor parallelism: host-side shard plumbing on CPU (gloo, world size 2),
TP=2/4/8 parity against the reference and the single-GPU engine (skipped
with fewer GPUs), and NCCL init failure detection."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from helpers import LOGITS_TOL, model_path, rel_l2

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, q):
    import torch.distributed as dist
    from llm_core_b200 import gguf
    from llm_core_b200.engine import tp_shard
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    from llm_core_b200._lib import ModelConfig
    p = gguf.PRESETS["llama2-7b"]
    c = ModelConfig()
    c.n_layer, c.n_embd, c.n_head, c.n_kv_head, c.ffn, c.vocab = p.n_layer, p.n_embd, p.n_head, p.n_kv_head, p.ffn, p.vocab
    shard = tp_shard(c, rank, world)
    # the NCCL id travels as an opaque byte string from rank 0
    obj = [bytes(range(128)) if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    allsh = [None] * world
    dist.all_gather_object(allsh, shard)
    q.put((rank, obj[0], allsh))
    dist.destroy_process_group()


def test_tp_shards_cover_the_model_over_gloo():
    """Two gloo ranks compute their shards and exchange them: heads, kv heads,
    FFN super-blocks and vocabulary rows are covered exactly once."""
    import torch.multiprocessing as mp
    from llm_core_b200 import gguf
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg = gguf.PRESETS["llama2-7b"]
    for rank, nid, shards in res:
        assert nid == bytes(range(128))
        shards = sorted(shards, key=lambda s: s.h0)
        assert shards[0].h0 == 0 and shards[-1].h1 == cfg.n_head
        assert shards[0].f0 == 0 and shards[-1].f1 == cfg.ffn
        assert shards[0].v0 == 0 and shards[-1].v1 == cfg.vocab
        for a, b in zip(shards, shards[1:]):
            assert a.h1 == b.h0 and a.kv1 == b.kv0 and a.f1 == b.f0 and a.v1 == b.v0
        # ffn_down K = 11008 = 43 super-blocks splits 22 / 21
        assert [(s.f1 - s.f0) // 256 for s in shards] == [22, 21]


def test_tp_shard_rejects_unsupported_shapes():
    from llm_core_b200._lib import ModelConfig
    from llm_core_b200.engine import tp_shard
    c = ModelConfig()
    c.n_layer, c.n_embd, c.n_head, c.n_kv_head, c.ffn, c.vocab = 2, 256, 4, 2, 512, 512
    with pytest.raises(ValueError):
        tp_shard(c, 0, 2)  # n_embd / 2 = 128 is not a whole super-block
    assert tp_shard(c, 0, 1).h1 == 4


def run_tp(world: int, path: str, xred: bool = True):
    """Launch tests/tp_worker.py on `world` ranks; rank 0's outputs."""
    out = os.path.join(os.environ.get("TMPDIR", "/tmp"), f"af_tp{world}_{int(xred)}_{os.getpid()}.npz")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", str(world), "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), os.path.join(ROOT, "tests", "tp_worker.py"), path, out]
    env = dict(os.environ, AF_TP_XRED="1" if xred else "0")
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return np.load(out)


@pytest.mark.gpu
@pytest.mark.parametrize("world,xred", [(2, True), (2, False), (4, True), (8, True), (8, False)])
def test_tp_matches_reference(world, xred):
    """TP=2/4/8 (torchrun, NCCL; partial sums over peer memory, reduced by a
    reduction phase or by every consuming CTA) against the reference's
    F32-activation forward: prefill logits within the logits bar and every
    greedy token equal to the reference's (>= 99 %)."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle import RefLib
    if not RefLib.available():
        pytest.skip("reference library not built")
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import tp_worker
    path = model_path("tp8", 5)
    z = run_tp(world, path, xred)
    ref = RefLib().open(path, threads=8, f32_mode=True)
    want, want_lg = ref.generate_greedy(tp_worker.PROMPT, tp_worker.STEPS + 1, want_logits=True)
    ref.close()
    assert rel_l2(z["logits"], want_lg[0]) < LOGITS_TOL
    got = [int(z["first"])] + [int(v) for v in z["ids"]]
    n = min(len(got), len(want))  # the reference stops at EOS
    agree = np.mean(np.array(got[:n]) == np.array(want[:n]))
    assert n > 8 and agree >= 0.99, (agree, got[:n], want[:n])


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_tp_matches_single_gpu(world):
    """TP=2 / TP=4 prefill logits and greedy continuation equal the
    single-GPU engine's on the same GGUF."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from llm_core_b200.engine import LlamaCudaModel
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import tp_worker
    path = model_path("small", 5)
    z = run_tp(world, path)
    m = LlamaCudaModel(path)
    nxt, lg = m.prefill(tp_worker.PROMPT, 0)
    ids = m.decode_greedy(nxt, len(tp_worker.PROMPT), tp_worker.STEPS)
    m.close()
    assert rel_l2(z["logits"], lg) < LOGITS_TOL
    assert int(z["first"]) == nxt
    agree = np.mean(z["ids"] == ids)
    assert agree >= 0.99, agree


@pytest.mark.gpu
def test_rank_that_never_joins_ends_nccl_init_with_an_error(gpu, tmp_path):
    """Failure detection on the host: rank 0 of a 2-rank engine whose peer
    never calls af_engine_create gets an error from af_engine_create once
    AF_NCCL_INIT_TIMEOUT_S passes (non-blocking init, then ncclCommAbort),
    instead of hanging.  Nothing runs on the GPU but NCCL's setup."""
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "from llm_core_b200 import gguf\n"
        "from llm_core_b200.engine import LlamaCudaModel, nccl_unique_id, read_config\n"
        "from llm_core_b200._lib import AfError\n"
        "import time\n"
        "t = time.time()\n"
        "try:\n"
        "    LlamaCudaModel(config=read_config(%r), tp_rank=0, tp_size=2, nccl_id=nccl_unique_id())\n"
        "    print('JOINED')\n"
        "except AfError as e:\n"
        "    print('ERR', round(time.time() - t, 1), e)\n"
    ) % (ROOT, model_path("small", 3))
    env = dict(os.environ, AF_NCCL_INIT_TIMEOUT_S="4", NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120, env=env)
    assert "ERR" in r.stdout, r.stdout + r.stderr
    assert "did not join" in r.stdout


def test_tp_shards_of_the_eight_way_preset():
    """The preset the TP parity runs use splits over 2, 4 and 8 ranks with
    every head, kv head, FFN super-block and vocabulary row owned exactly
    once (ffn_down's 22 super-blocks unevenly at 4 and 8)."""
    from llm_core_b200 import gguf
    from llm_core_b200._lib import ModelConfig
    from llm_core_b200.engine import tp_shard
    p = gguf.PRESETS["tp8"]
    c = ModelConfig()
    c.n_layer, c.n_embd, c.n_head, c.n_kv_head, c.ffn, c.vocab = p.n_layer, p.n_embd, p.n_head, p.n_kv_head, p.ffn, p.vocab
    for world in (2, 4, 8):
        sh = [tp_shard(c, r, world) for r in range(world)]
        assert sh[0].h0 == 0 and sh[-1].h1 == p.n_head
        assert sh[0].kv0 == 0 and sh[-1].kv1 == p.n_kv_head
        assert sh[0].f0 == 0 and sh[-1].f1 == p.ffn
        assert sh[0].v0 == 0 and sh[-1].v1 == p.vocab
        for a, b in zip(sh, sh[1:]):
            assert a.h1 == b.h0 and a.kv1 == b.kv0 and a.f1 == b.f0 and a.v1 == b.v0
        blocks = [(s.f1 - s.f0) // 256 for s in sh]
        assert sum(blocks) == p.ffn // 256 and max(blocks) - min(blocks) <= 1
