"""Training-loop rows beyond the step itself, on the device: the dropout mask
stream (bit-exact with the reference's), the token-stream data feed (the same
step as host ids), and checkpoint / resume (weights loadable by the
reference, optimizer state restored so a run continues exactly)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CFG = dict(vocab=1000, dim=128, layers=2, heads=2, ffn=256, max_seq=64)


@pytest.mark.parametrize("n,p,seed", [(1, 0.5, 0), (33, 0.1, 7), (4097, 0.3, 12345),
                                      (1_000_003, 0.1, 99), (5_000_000, 0.9, (1 << 63) + 5)])
def test_dropout_mask_bitexact(cuda, n, p, seed):
    from oracle import refbind as rb
    from tinytrain_b200 import _ttk
    m = torch.empty(n, device=cuda)
    _ttk.call("ttk_dropout_mask", m.data_ptr(), n, p, seed,
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(m.cpu().numpy(), rb.dropout_mask(n, p, seed))


def _trainer(seed, clip=0.0):
    from tinytrain_b200 import trainer as TR
    t = TR.Trainer(CFG, seed=seed)
    t.set_optimizer(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, clip=clip)
    return t


def test_step_tokens_equals_host_ids(cuda):
    """Windows gathered on the device from the resident token stream give the
    same step as the same windows uploaded as host ids."""
    from tinytrain_b200 import trainer as TR
    rng = np.random.default_rng(5)
    tok = rng.integers(0, CFG["vocab"], 5000).astype(np.int32)
    ts = TR.TokenStream(host=tok)
    assert len(ts) == tok.size
    a, b = _trainer(3), _trainer(3)
    samp = TR.WindowSampler(7 + 999)
    B, T, nm = 2, 64, 2
    for step in range(3):
        starts = samp.draw(tok.size, T, B * nm)
        la, _ = a.step_tokens(ts, starts, B, T, nm, lr=TR.lr_at(1e-3, step, 2, 10))
        idx = np.stack([tok[s:s + T] for s in starts]).astype(np.int64).ravel()
        tgt = np.stack([tok[s + 1:s + T + 1] for s in starts]).astype(np.int64).ravel()
        lb, _ = b.step(idx, tgt, B, T, nm, lr=TR.lr_at(1e-3, step, 2, 10))
        assert abs(la - lb) <= 1e-6 * abs(lb)
    assert np.array_equal(a.get_params(), b.get_params())
    with pytest.raises(TR.TrainerError):
        a.step_tokens(ts, np.array([tok.size - T], np.int64), 1, T, 1)


def test_checkpoint_resume_continues_exactly(cuda, tmp_path):
    from oracle import refbind as rb
    rng = np.random.default_rng(6)
    B, T = 2, 64
    batches = [(rng.integers(0, CFG["vocab"], B * T), rng.integers(0, CFG["vocab"], B * T))
               for _ in range(5)]
    a = _trainer(3)
    for i, t_ in batches[:3]:
        a.step(i, t_, B, T)
    ck = str(tmp_path / "ck")
    a.save(ck)
    saved = a.get_params()
    la = [a.step(i, t_, B, T)[0] for i, t_ in batches[3:]]
    b = _trainer(11)  # different initial weights: everything must come from the checkpoint
    b.load(ck)
    assert np.array_equal(b.get_params(), saved)
    lb = [b.step(i, t_, B, T)[0] for i, t_ in batches[3:]]
    assert np.allclose(la, lb, rtol=1e-6, atol=0)
    assert np.array_equal(a.get_params(), b.get_params())
    # the weights file is the reference's format: its load_checkpoint reads it
    c = rb.cfg(vocab=CFG["vocab"], dim=CFG["dim"], layers=CFG["layers"], heads=CFG["heads"],
               ffn=CFG["ffn"], max_seq=CFG["max_seq"])
    assert np.array_equal(rb.load_checkpoint(c, ck), saved)


def test_step_submit_result_equals_step(cuda):
    """The pipelined halves (tt_trainer_step_submit / tt_trainer_step_result,
    two steps in flight) give every step's loss and gradient norm and the
    final weights of tt_trainer_step on the same ids, bit for bit; a third
    submit before a result is refused."""
    from tinytrain_b200 import trainer as TR
    rng = np.random.default_rng(9)
    B, T, n_micro, steps = 2, 64, 2, 4
    ids = [(rng.integers(0, CFG["vocab"], B * T * n_micro),
            rng.integers(0, CFG["vocab"], B * T * n_micro)) for _ in range(steps)]
    a, b = _trainer(3, clip=1.0), _trainer(3, clip=1.0)
    ref = [a.step(i, t, B, T, n_micro, 1e-3) for i, t in ids]
    got = []
    for k, (i, t) in enumerate(ids):
        b.step_submit(i, t, B, T, n_micro, 1e-3)
        if k == 1:  # two in flight now
            with pytest.raises(TR.TrainerError, match="two steps are in flight"):
                b.step_submit(i, t, B, T, n_micro, 1e-3)
        if k > 0:
            got.append(b.step_result())
    got.append(b.step_result())
    assert got == ref
    assert np.array_equal(a.get_params(), b.get_params())
    with pytest.raises(TR.TrainerError, match="no step in flight"):
        b.step_result()
    a.close()
    b.close()
