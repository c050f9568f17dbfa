"""Tensor-parallel rank of the TP parity test (launched by torch.distributed.run).

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port P tests/tp_worker.py MODEL.gguf OUT.npz

Each rank loads its shard of the GGUF, the ranks exchange the NCCL id over
torch.distributed, and rank 0 writes the prefill logits and a greedy
continuation for the test to compare with a single-GPU engine.
"""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from llm_core_b200.engine import LlamaCudaModel, nccl_unique_id  # noqa: E402

PROMPT = [1, 17, 999, 4, 250, 3000, 12, 7]
STEPS = 48


def main(path: str, out: str) -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    m = LlamaCudaModel(path, device=local, tp_rank=rank, tp_size=world, nccl_id=obj[0])
    nxt, lg = m.prefill(PROMPT, 0)
    ids = m.decode_greedy(nxt, len(PROMPT), STEPS)
    if rank == 0:
        np.savez(out, logits=lg, first=np.int32(nxt), ids=ids)
    dist.barrier()
    m.close()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1], sys.argv[2]))
