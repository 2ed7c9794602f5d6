"""The host-side block cache over the device pool (ttk_set_block_cache): with
it on, training steps hand freed blocks back out instead of returning them to
the pool, which changes buffer addresses but no arithmetic. Steps with the
cache on must equal steps with it off bit for bit, including graph-replayed
steps (allocations inside a stream capture bypass the cache), and turning it
off returns the cached blocks to the pool."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CFG = dict(vocab=512, dim=256, layers=2, heads=4, ffn=512, max_seq=128)
B, T, NM = 4, 128, 2
LRS = [1e-3, 2e-3, 3e-3, 2e-3, 1e-3]


def _pool_used():
    from tinytrain_b200 import _ttk
    r, u = C.c_size_t(0), C.c_size_t(0)
    _ttk.call("ttk_pool_stats", C.byref(r), C.byref(u))
    return u.value


def _run(cache, graph):
    from tinytrain_b200 import _ttk
    from tinytrain_b200 import trainer as TR
    rng = np.random.default_rng(31)
    batches = [(torch.from_numpy(rng.integers(0, CFG["vocab"], B * T * NM)).cuda(),
                torch.from_numpy(rng.integers(0, CFG["vocab"], B * T * NM)).cuda())
               for _ in range(len(LRS))]
    _ttk.call("ttk_set_block_cache", 1 if cache else 0)
    try:
        t = TR.Trainer(CFG, seed=13)
        t.set_optimizer(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, clip=1.0)
        bi, bt = torch.empty_like(batches[0][0]), torch.empty_like(batches[0][1])
        losses = []
        for lr, (ids, tgt) in zip(LRS, batches):
            torch.cuda.synchronize()
            bi.copy_(ids)
            bt.copy_(tgt)
            if graph:
                t.step_graph(bi.data_ptr(), bt.data_ptr(), B, T, NM, lr)
            else:
                t.step_device(bi.data_ptr(), bt.data_ptr(), B, T, NM, lr)
            torch.cuda.synchronize()
            losses.append(t.last_loss())
        params = t.get_params()
        t.close()
        return params, losses
    finally:
        _ttk.call("ttk_set_block_cache", 0)


@pytest.mark.parametrize("graph", [False, True])
def test_block_cache_same_results(cuda, graph):
    p0, l0 = _run(False, graph)
    p1, l1 = _run(True, graph)
    assert np.array_equal(p0, p1)
    # losses are sums of atomically added row losses (order may vary)
    assert np.allclose(l0, l1, rtol=1e-6, atol=0)
    from tinytrain_b200 import _ttk
    assert _ttk.device_status() == 0


def test_block_cache_reuses_and_releases(cuda):
    from tinytrain_b200 import _ttk
    s = torch.cuda.current_stream().cuda_stream
    _ttk.call("ttk_set_block_cache", 1)
    try:
        p = C.c_void_p()
        _ttk.call("ttk_malloc", C.byref(p), 3 << 20, s)
        first = p.value
        _ttk.call("ttk_free", p, s)
        held = _pool_used()
        _ttk.call("ttk_malloc", C.byref(p), 3 << 20, s)
        assert p.value == first  # the same block, handed back out on the same stream
        _ttk.call("ttk_free", p, s)
        assert _pool_used() == held  # cached, not returned to the pool
    finally:
        _ttk.call("ttk_set_block_cache", 0)  # returns the cached blocks to the pool
    torch.cuda.synchronize()
    assert _pool_used() <= held - (3 << 20)
