"""Kernel parity at the sizes the benchmarks run.

- Cross-entropy over the 1B micro-batch's logits, 32768 x 32000 (1.05e9
  elements, 4.2 GB: byte offsets past 2^31): the mean loss over every row
  and the gradient rows of three 1024-row blocks (first, middle, last)
  against the restatement of ops.cpp:840-930 (oracle/restate.py).
- RMSNorm forward/backward at the 1B micro-batch (32768 x 2048) and SwiGLU
  forward/backward at its feed-forward width (32768 x 5632), rows sampled,
  dw over all rows.
- The causal attention micro-bench: batch 8, heads 12, head dim 64, seq 128,
  512, 1024, 2048, RoPE theta 10000, inputs N(0, 1), forward and backward.
  Heads are independent, so the restated reference (model.cpp:127-141 and
  its backward) runs on six sampled (batch, head) pairs for seq >= 1024 and
  on all 96 below.
Tolerance: max |ours - ref| / max |ref| <= 1e-4.
"""
import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4


def n(x):
    torch.cuda.synchronize()
    return x.detach().cpu().numpy()


def test_cross_entropy_llama1b_microbatch(cuda):
    from oracle import restate as rs
    from tinytrain_b200 import _ttk, kernels as K
    N, V, blk = 32768, 32000, 1024
    g = torch.Generator(device=cuda).manual_seed(77)
    L = torch.randn(N, V, device=cuda, generator=g) * 3
    tg = torch.randint(0, V, (N,), device=cuda, generator=g, dtype=torch.int64)
    loss, dL = K.cross_entropy(L, tg)
    loss = float(n(loss)[0])
    tgh = n(tg)
    total = 0.0
    checked = 0
    for r0 in range(0, N, blk):
        Lh = n(L[r0:r0 + blk])
        lb, db = rs.cross_entropy(Lh, tgh[r0:r0 + blk])
        total += float(lb) * blk
        if r0 in (0, N // 2, N - blk):
            # restate scales by 1/blk; the whole-batch gradient is 1/N
            ref = db.astype(np.float64) * (blk / N)
            assert rel_err(n(dL[r0:r0 + blk]), ref) < TOL, r0
            checked += 1
    assert checked == 3
    ref_loss = total / N
    assert abs(loss - ref_loss) <= TOL * abs(ref_loss), (loss, ref_loss)
    assert _ttk.device_status() == 0


def test_rmsnorm_llama1b_microbatch(cuda):
    from oracle import restate as rs
    from tinytrain_b200 import _ttk, kernels as K
    R, D = 32768, 2048
    g = torch.Generator(device=cuda).manual_seed(78)
    x = torch.randn(R, D, device=cuda, generator=g)
    w = torch.rand(D, device=cuda, generator=g) + 0.5
    dy = torch.randn(R, D, device=cuda, generator=g)
    y, rstd = K.rmsnorm_fwd(x, w, 1e-5)
    dx, dw = K.rmsnorm_bwd(x, w, rstd, dy)
    wh = n(w)
    dw_ref = np.zeros(D, np.float64)
    for r0 in range(0, R, 4096):
        xh, gh = n(x[r0:r0 + 4096]), n(dy[r0:r0 + 4096])
        yr, r = rs.rmsnorm(xh, wh, 1e-5)
        dxr, dwr = rs.rmsnorm_bwd(xh, wh, r, gh)
        dw_ref += dwr.astype(np.float64)
        if r0 in (0, R - 4096):
            assert rel_err(n(y[r0:r0 + 4096]), yr) < TOL
            assert rel_err(n(dx[r0:r0 + 4096]), dxr) < TOL
    assert rel_err(n(dw), dw_ref) < TOL
    assert _ttk.device_status() == 0


def test_swiglu_llama1b_microbatch(cuda):
    from oracle import restate as rs
    from tinytrain_b200 import _ttk, kernels as K
    R, F = 32768, 5632
    g = torch.Generator(device=cuda).manual_seed(79)
    a = torch.randn(R, F, device=cuda, generator=g) * 3
    b = torch.randn(R, F, device=cuda, generator=g)
    dy = torch.randn(R, F, device=cuda, generator=g)
    y = K.swiglu_fwd(a, b)
    da, db = K.swiglu_bwd(a, b, dy)
    for r0 in (0, R // 2, R - 1024):
        sl = slice(r0, r0 + 1024)
        ah, bh, gh = n(a[sl]), n(b[sl]), n(dy[sl])
        assert rel_err(n(y[sl]), rs.swiglu(ah, bh)) < TOL
        dar, dbr = rs.swiglu_bwd(ah, bh, gh)
        assert rel_err(n(da[sl]), dar) < TOL
        assert rel_err(n(db[sl]), dbr) < TOL
    assert _ttk.device_status() == 0


@pytest.mark.parametrize("S", [128, 512, 1024, 2048])
def test_attention_microbench_config(cuda, S):
    from oracle import restate as rs
    from tinytrain_b200 import _ttk, kernels as K
    B, H, hd = 8, 12, 64
    g = torch.Generator(device=cuda).manual_seed(S)
    q, k, v, do = (torch.randn(B, S, H, hd, device=cuda, generator=g) for _ in range(4))
    cs, sn = K.rope_tables(S, hd, 10000.0, cuda)
    o, lse = K.attention_fwd(q, k, v, cs, sn)
    dq, dk, dv = K.attention_bwd(q, k, v, cs, sn, o, lse, do)
    if S >= 1024:
        rng = np.random.default_rng(S)
        pairs = [(0, 0), (B - 1, H - 1)] + [(int(rng.integers(B)), int(rng.integers(H)))
                                            for _ in range(4)]
    else:
        pairs = [(b, h) for b in range(B) for h in range(H)]
    qh, kh, vh, doh = n(q), n(k), n(v), n(do)
    oh, dqh, dkh, dvh = n(o), n(dq), n(dk), n(dv)
    for b, h in pairs:
        sel = (slice(b, b + 1), slice(None), slice(h, h + 1), slice(None))
        orf, cache = rs.attention(qh[sel], kh[sel], vh[sel], 10000.0)
        dqr, dkr, dvr = rs.attention_bwd(doh[sel].reshape(1, S, hd), cache)
        assert rel_err(oh[sel].reshape(1, S, hd), orf) < TOL, (b, h)
        assert rel_err(dqh[sel], dqr) < TOL, (b, h)
        assert rel_err(dkh[sel], dkr) < TOL, (b, h)
        assert rel_err(dvh[sel], dvr) < TOL, (b, h)
    assert _ttk.device_status() == 0
