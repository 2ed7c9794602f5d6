"""Training steps replayed from a CUDA graph (tt_trainer_step_graph) against
the same steps run eagerly (tt_trainer_step_device): the same kernels in the
same order, so parameters, losses and the optimizer's step count must agree
exactly, including across learning-rate changes (the AdamW kernel in the
graph reads lr and the bias correction from the device) and across a switch
of id buffers (the graph is dropped and recorded again)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# Sized so the projections and the LM head run on the tensor-core GEMM and
# head dim 64 takes the tcgen05 attention (as the smoke model).
CFG = dict(vocab=512, dim=256, layers=2, heads=4, ffn=512, max_seq=128)
B, T, NM = 4, 128, 2
LRS = [1e-3, 2e-3, 3e-3, 2.5e-3, 1.5e-3, 1e-3, 5e-4, 2e-4]


def _trainer():
    from tinytrain_b200 import trainer as TR
    t = TR.Trainer(CFG, seed=11)
    t.set_optimizer(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, clip=0.0)
    return t


def _batches(n):
    rng = np.random.default_rng(21)
    return [(torch.from_numpy(rng.integers(0, CFG["vocab"], B * T * NM)).cuda(),
             torch.from_numpy(rng.integers(0, CFG["vocab"], B * T * NM)).cuda())
            for _ in range(n)]


def test_graph_steps_equal_eager_steps(cuda):
    batches = _batches(len(LRS))
    eager, graph = _trainer(), _trainer()
    # the graph replays read the ids from two fixed buffers; each step's ids
    # are copied into them first (stream-ordered)
    bi = torch.empty_like(batches[0][0])
    bt = torch.empty_like(batches[0][1])
    other_i, other_t = torch.empty_like(bi), torch.empty_like(bt)
    for step, (lr, (ids, tgt)) in enumerate(zip(LRS, batches)):
        eager.step_device(ids.data_ptr(), tgt.data_ptr(), B, T, NM, lr)
        # steps 5 and 6 use other buffers: the graph is dropped, step 5 runs
        # eagerly, step 6 records again
        di, dt = (other_i, other_t) if step in (5, 6) else (bi, bt)
        # the trainer runs on its own stream: the previous step must be done
        # with the buffers before torch's copy overwrites them
        torch.cuda.synchronize()
        di.copy_(ids)
        dt.copy_(tgt)
        graph.step_graph(di.data_ptr(), dt.data_ptr(), B, T, NM, lr)
        torch.cuda.synchronize()
        le, lg = eager.last_loss(), graph.last_loss()
        # the loss is a sum of atomically added row losses: its last bits
        # may depend on the order
        assert abs(le - lg) <= 1e-6 * abs(le), (step, le, lg)
        assert np.array_equal(eager.get_params(), graph.get_params()), step
    from tinytrain_b200 import _ttk
    assert _ttk.device_status() == 0
    eager.close()
    graph.close()


def test_graph_then_eager_step(cuda):
    """An eager step after graph replays sees the replays' weights (the cached
    weight splits are refreshed) and gives the same result as eager steps
    throughout."""
    batches = _batches(4)
    a, b = _trainer(), _trainer()
    bi = torch.empty_like(batches[0][0])
    bt = torch.empty_like(batches[0][1])
    for step, (ids, tgt) in enumerate(batches):
        a.step_device(ids.data_ptr(), tgt.data_ptr(), B, T, NM, LRS[step])
        if step < 3:
            torch.cuda.synchronize()  # the buffers are free again (see above)
            bi.copy_(ids)
            bt.copy_(tgt)
            b.step_graph(bi.data_ptr(), bt.data_ptr(), B, T, NM, LRS[step])
        else:
            b.step_device(ids.data_ptr(), tgt.data_ptr(), B, T, NM, LRS[step])
    torch.cuda.synchronize()
    assert np.array_equal(a.get_params(), b.get_params())
    a.close()
    b.close()


def test_graph_dropped_when_params_written(cuda):
    """Parameters written from the host between replays (set_params) drop the
    recorded step: the next call runs eagerly, which uploads the new values,
    and the results stay equal to eager steps."""
    batches = _batches(6)
    a, b = _trainer(), _trainer()
    bi = torch.empty_like(batches[0][0])
    bt = torch.empty_like(batches[0][1])
    fresh = (np.random.default_rng(5).standard_normal(a.get_params().size) * 0.02).astype(
        np.float32)
    for step, (ids, tgt) in enumerate(batches):
        if step == 3:
            torch.cuda.synchronize()
            a.set_params(fresh)
            b.set_params(fresh)
        a.step_device(ids.data_ptr(), tgt.data_ptr(), B, T, NM, LRS[step])
        torch.cuda.synchronize()
        bi.copy_(ids)
        bt.copy_(tgt)
        b.step_graph(bi.data_ptr(), bt.data_ptr(), B, T, NM, LRS[step])
    torch.cuda.synchronize()
    assert np.array_equal(a.get_params(), b.get_params())
    a.close()
    b.close()
