"""Worker for tests/test_failure_gpu.py: a data-parallel job whose rank 1
leaves between steps.

Launched by torch.distributed.run on 2 GPUs with NCCL_NVLS_ENABLE=0. Both
ranks run one distributed step of a small model (NCCL gradient all-reduce).
Then rank 1 closes its trainer and exits, with no kernel or collective in
flight. Rank 0, with a 5 s collective deadline, starts a second step: its
all-reduce has no peer, so the watchdog aborts the communicator and the step
fails. Rank 0 writes the error message, the time the failing step took, and
whether a fresh single-GPU step still runs on the same device afterwards.
"""
import json
import os
import sys
import time
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from tinytrain_b200 import _ttk, trainer as trn  # noqa: E402

CFG = dict(vocab=1000, dim=128, layers=2, heads=4, ffn=256, max_seq=64)
B, T = 2, 64


def main(out):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    rng = np.random.default_rng(rank)
    idx = rng.integers(0, CFG["vocab"], B * T)
    tgt = rng.integers(0, CFG["vocab"], B * T)
    tr = trn.Trainer(CFG, seed=1, host_init=False)
    tr.init_normal(0.02, seed=1)
    tr.set_optimizer(lr=1e-3, clip=1.0)
    uid = trn.dist_unique_id() if rank == 0 else b"\0" * 128
    obj = [uid]
    dist.broadcast_object_list(obj, src=0)
    tr.dist_init(rank, world, obj[0], bucket_bytes=256 << 10)
    tr.set_collective_timeout(5.0)
    tr.step(idx, tgt, B, T, 1, 1e-3)  # returns after its collectives completed
    dist.barrier()
    if rank != 0:
        tr.close()  # leaves between steps: nothing of this rank is in flight
        return
    time.sleep(1.0)
    t0 = time.time()
    err = None
    try:
        tr.step(idx, tgt, B, T, 1, 1e-3)
    except trn.TrainerError as e:
        err = str(e)
    took = time.time() - t0
    refused = None
    try:
        tr.step(idx, tgt, B, T, 1, 1e-3)
    except trn.TrainerError as e:
        refused = str(e)
    tr.close()
    # The device is still usable: a fresh single-GPU step runs.
    tr2 = trn.Trainer(CFG, seed=1, host_init=False)
    tr2.init_normal(0.02, seed=2)
    tr2.set_optimizer(lr=1e-3, clip=1.0)
    loss, _ = tr2.step(idx, tgt, B, T, 1, 1e-3)
    tr2.close()
    with open(out, "w") as f:
        json.dump({"error": err, "took": took, "refused": refused, "loss_after": loss,
                   "status": _ttk.device_status()}, f)


if __name__ == "__main__":
    main(sys.argv[1])
