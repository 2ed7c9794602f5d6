"""Host-side logic of the data-parallel path on CPU ranks (gloo, world size
2): the bucket plan is identical on every rank; reducing the per-rank
gradient arenas bucket by bucket in plan order gives the sum over ranks;
the step loss is the mean over ranks; the step time is the max over ranks;
and a rank that never joins a collective makes the other rank's collective
fail with an error after a short timeout instead of hanging."""
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    from tinytrain_b200.trainer import plan_buckets
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=30))
    sizes = [1000, 64, 4096, 4096, 64, 3000, 3000, 64]
    offs, ids, buckets = plan_buckets(sizes, 8 * 1024)
    plans = [None] * world
    dist.all_gather_object(plans, (offs.tolist(), ids.tolist(), buckets))
    same = all(p == plans[0] for p in plans)
    arena = torch.zeros(int(buckets[-1][0] + buckets[-1][1]), dtype=torch.float32)
    rng = np.random.default_rng(100 + rank)
    grads = [rng.standard_normal(n).astype(np.float32) for n in sizes]
    for i, g in enumerate(grads):
        arena[offs[i]:offs[i] + sizes[i]] = torch.from_numpy(g)
    for bo, bc in buckets:  # backward order
        view = arena[bo:bo + bc]
        dist.all_reduce(view)
    loss = torch.tensor([float(rank + 1)])
    dist.all_reduce(loss)
    step_ms = torch.tensor([10.0 + rank], dtype=torch.float64)
    dist.all_reduce(step_ms, op=dist.ReduceOp.MAX)
    out = {i: arena[offs[i]:offs[i] + sizes[i]].numpy().copy() for i in range(len(sizes))}
    q.put((rank, same, out, loss.item() / world, step_ms.item()))
    dist.barrier()
    dist.destroy_process_group()


def test_bucketed_allreduce_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    sizes = [1000, 64, 4096, 4096, 64, 3000, 3000, 64]
    per_rank = []
    for r in range(2):
        rng = np.random.default_rng(100 + r)
        per_rank.append([rng.standard_normal(n).astype(np.float32) for n in sizes])
    for rank, same, out, loss, ms in res:
        assert same
        assert abs(loss - 1.5) < 1e-6
        assert ms == 11.0
        for i in range(len(sizes)):
            np.testing.assert_allclose(out[i], per_rank[0][i] + per_rank[1][i], rtol=1e-6)


def _silent_worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=3))
    t = torch.ones(4)
    if rank == 0:
        try:
            dist.all_reduce(t)  # rank 1 never joins this collective
            q.put("completed")
        except Exception as e:
            q.put("error: " + type(e).__name__)
    else:
        q.put("left")
    q.close()
    q.join_thread()  # flush before leaving without teardown
    os._exit(0)


def test_missing_rank_fails_with_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_silent_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert got[1] == "left"
    assert got[0].startswith("error")
