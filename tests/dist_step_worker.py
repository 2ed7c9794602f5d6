"""Worker for tests/test_dist_gpu.py: one rank of a data-parallel step.

Launched by torch.distributed.run; every rank builds the same tiny model,
takes its half of a fixed global batch, runs one AdamW step with the bucketed
NCCL gradient all-reduce, and rank 0 writes the resulting parameters and loss.
"""
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from tinytrain_b200 import trainer as trn  # noqa: E402

CFG = dict(vocab=1000, dim=128, layers=2, heads=4, ffn=256, max_seq=64)
B, T, GLOBAL = 2, 64, 4


def main(out):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    rng = np.random.default_rng(0)
    w = (rng.standard_normal(2_000_000) * 0.05).astype(np.float32)
    idx = rng.integers(0, CFG["vocab"], GLOBAL * T)
    tgt = rng.integers(0, CFG["vocab"], GLOBAL * T)
    tr = trn.Trainer(CFG, seed=1, host_init=False)
    shapes_n = tr.n_params
    params = w[:shapes_n].copy()
    tr.set_params(params)
    tr.set_optimizer(lr=1e-2, clip=1.0)
    uid = trn.dist_unique_id() if rank == 0 else b"\0" * 128
    obj = [uid]
    dist.broadcast_object_list(obj, src=0)
    tr.dist_init(rank, world, obj[0], bucket_bytes=256 << 10)  # several buckets
    per = GLOBAL // world
    sl = slice(rank * per * T, (rank + 1) * per * T)
    n_micro = per // B
    loss, gn = tr.step(idx[sl], tgt[sl], B, T, n_micro, 1e-2)
    if rank == 0:
        np.savez(out, params=tr.get_params(), loss=np.float32(loss), gn=np.float32(gn))
    tr.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
