"""Parity of the bandwidth-bound kernels and the fused attention with the
reference (tests/golden/ops_small.npz, produced by the reference's own CPU
library) and, at benchmark sizes, with the numpy restatement of the same
algorithms (oracle/restate.py, itself pinned to the reference).

Tolerance: max|err| / max|ref| <= 1e-4 (forward and gradient); the embedding
gather and the deterministic scatter-add are compared bit for bit.
"""
import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4


def t(a, dev, dtype=None):
    x = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return x if dtype is None else x.to(dtype)


def n(x):
    torch.cuda.synchronize()
    return x.detach().cpu().numpy()


def status_ok():
    from tinytrain_b200 import _ttk
    return _ttk.device_status() == 0


@pytest.mark.parametrize("R,D", [(4096, 2048), (1000, 768), (333, 256)])
def test_rmsnorm_fwd_split_planes_bitexact(cuda, R, D):
    """ttk_rmsnorm_fwd_split: y equals ttk_rmsnorm_fwd's and the planes equal
    ttk_gemm_split(y), bit for bit."""
    from tinytrain_b200 import kernels as K
    g = torch.Generator(device=cuda).manual_seed(R + D)
    x = torch.randn(R, D, device=cuda, generator=g) * 3
    w = torch.rand(D, device=cuda, generator=g) + 0.5
    y0, r0 = K.rmsnorm_fwd(x, w, 1e-5)
    y1, r1, planes = K.rmsnorm_fwd_split(x, w, 1e-5)
    ref = K.gemm_split(y1)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1) and torch.equal(r0, r1)
    assert torch.equal(planes, ref)
    assert status_ok()


def test_rmsnorm_golden(cuda, golden_ops):
    from tinytrain_b200 import kernels as K
    g = golden_ops
    x, w, gy = t(g["rms_X"], cuda), t(g["rms_W"], cuda), t(g["rms_G"], cuda)
    y, rstd = K.rmsnorm_fwd(x, w, 1e-5)
    dx, dw = K.rmsnorm_bwd(x, w, rstd, gy)
    assert rel_err(n(y), g["rms_Y"]) < TOL
    assert rel_err(n(dx), g["rms_dX"]) < TOL
    assert rel_err(n(dw), g["rms_dW"]) < TOL
    assert status_ok()


@pytest.mark.parametrize("R,D", [(2048, 256), (16384, 2048), (1000, 768), (37, 20)])
def test_rmsnorm_sizes(cuda, R, D):
    from oracle import restate as rs
    from tinytrain_b200 import kernels as K
    rng = np.random.default_rng(R + D)
    x = rng.uniform(-1, 1, (R, D)).astype(np.float32)
    w = rng.uniform(-1, 1, D).astype(np.float32)
    gy = rng.uniform(-1, 1, (R, D)).astype(np.float32)
    y, rstd = K.rmsnorm_fwd(t(x, cuda), t(w, cuda), 1e-5)
    dx, dw = K.rmsnorm_bwd(t(x, cuda), t(w, cuda), rstd, t(gy, cuda))
    yr, rr = rs.rmsnorm(x, w, 1e-5)
    dxr, dwr = rs.rmsnorm_bwd(x, w, rr, gy)
    assert rel_err(n(y), yr) < TOL
    assert rel_err(n(dx), dxr) < TOL
    assert rel_err(n(dw), dwr) < TOL


@pytest.mark.parametrize("R,D", [(1000, 2048), (16384, 2048), (37, 256)])
def test_rmsnorm_bwd_accumulates(cuda, R, D):
    """dx += and dw += into existing gradients (the residual stream's
    gradient in a transformer block), row counts that leave the last sweep of
    the row-parallel kernel partly empty."""
    from oracle import restate as rs
    from tinytrain_b200 import kernels as K
    rng = np.random.default_rng(7 * R + D)
    x = rng.uniform(-1, 1, (R, D)).astype(np.float32)
    w = rng.uniform(-1, 1, D).astype(np.float32)
    gy = rng.uniform(-1, 1, (R, D)).astype(np.float32)
    dx0 = rng.uniform(-1, 1, (R, D)).astype(np.float32)
    dw0 = rng.uniform(-1, 1, D).astype(np.float32)
    _, rstd = K.rmsnorm_fwd(t(x, cuda), t(w, cuda), 1e-5)
    dx, dw = t(dx0, cuda), t(dw0, cuda)
    K.rmsnorm_bwd(t(x, cuda), t(w, cuda), rstd, t(gy, cuda), dx=dx, dw=dw, accumulate=True)
    _, rr = rs.rmsnorm(x, w, 1e-5)
    dxr, dwr = rs.rmsnorm_bwd(x, w, rr, gy)
    assert rel_err(n(dx), dxr + dx0) < TOL
    assert rel_err(n(dw), dwr + dw0) < TOL


@pytest.mark.parametrize("shape,bshape,offset", [
    ((4096,), (4096,), 0), ((1027,), (1027,), 0), ((8, 2048, 64), (8, 2048, 64), 0),
    ((3, 1, 5), (3, 1, 5), 0), ((4096,), (4096,), 1), ((6, 33), (33,), 0), ((6, 33), (6, 1), 0)])
def test_binary_paths_bitexact(cuda, shape, bshape, offset):
    """Elementwise add/sub/mul/div on the vector path (same-shape contiguous,
    16-byte aligned) and on the strided path (broadcast, or an operand one
    element off alignment) equal numpy's IEEE results bit for bit."""
    from tinytrain_b200 import _ttk
    import ctypes as C
    rng = np.random.default_rng(len(shape) * 100 + offset)
    a = rng.uniform(-2, 2, shape).astype(np.float32)
    b = rng.uniform(0.5, 2, bshape).astype(np.float32)
    full = np.broadcast_shapes(shape, bshape)
    bb = np.broadcast_to(b, full)
    nd = len(full)
    ext = (C.c_int64 * nd)(*full)

    def strides(arr_shape):
        pad = (1,) * (nd - len(arr_shape)) + tuple(arr_shape)
        st, acc = [0] * nd, 1
        for d in range(nd - 1, -1, -1):
            st[d] = 0 if pad[d] == 1 and full[d] != 1 else acc
            acc *= pad[d]
        return (C.c_int64 * nd)(*st)

    abuf = torch.zeros(a.size + offset, dtype=torch.float32, device=cuda)
    abuf[offset:] = t(a.ravel(), cuda)
    da, db = abuf[offset:], t(b.ravel(), cuda)
    out = torch.empty(int(np.prod(full)), dtype=torch.float32, device=cuda)
    for op, f in enumerate([np.add, np.subtract, np.multiply, np.divide]):
        _ttk.call("ttk_binary", op, da.data_ptr(), strides(shape), db.data_ptr(), strides(bshape),
                  out.data_ptr(), ext, nd, torch.cuda.current_stream().cuda_stream)
        ref = f(np.broadcast_to(a, full), bb).astype(np.float32).ravel()
        assert np.array_equal(n(out).view(np.uint32), ref.view(np.uint32)), op


def test_swiglu_golden(cuda, golden_ops):
    from tinytrain_b200 import kernels as K
    g = golden_ops
    a, b, gy = t(g["swi_A"], cuda), t(g["swi_B"], cuda), t(g["swi_G"], cuda)
    y = K.swiglu_fwd(a, b)
    da, db = K.swiglu_bwd(a, b, gy)
    assert rel_err(n(y), g["swi_Y"]) < TOL
    assert rel_err(n(da), g["swi_dA"]) < TOL
    assert rel_err(n(db), g["swi_dB"]) < TOL
    # accumulate path
    da2, db2 = K.swiglu_bwd(a, b, gy, da=da.clone(), db=db.clone(), accumulate=True)
    assert rel_err(n(da2), 2 * g["swi_dA"]) < TOL


def test_cross_entropy_golden(cuda, golden_ops):
    from tinytrain_b200 import kernels as K
    g = golden_ops
    L = t(g["ce_L"], cuda)
    tg = t(g["ce_t"].astype(np.int64), cuda)
    loss, dL = K.cross_entropy(L, tg)
    assert abs(float(n(loss)[0]) - float(g["ce_loss"])) <= 1e-4 * abs(float(g["ce_loss"]))
    assert rel_err(n(dL), g["ce_dL"]) < TOL


@pytest.mark.parametrize("N,C", [(2048, 32000), (333, 32000), (64, 50000), (5, 7)])
def test_cross_entropy_sizes(cuda, N, C):
    from oracle import restate as rs
    from tinytrain_b200 import kernels as K
    rng = np.random.default_rng(N + C)
    L = (rng.standard_normal((N, C)) * 3).astype(np.float32)
    tg = rng.integers(0, C, N).astype(np.int64)
    loss, dL = K.cross_entropy(t(L, cuda), t(tg, cuda))
    lr_, dLr = rs.cross_entropy(L, tg)
    assert abs(float(n(loss)[0]) - float(lr_)) <= 1e-4 * abs(float(lr_))
    assert rel_err(n(dL), dLr) < TOL
    # in-place gradient (dlogits aliasing logits) gives the same values and loss
    Ld = t(L, cuda)
    loss_ip, _ = K.cross_entropy(Ld, t(tg, cuda), dlogits=Ld)
    assert rel_err(n(Ld), dLr) < TOL
    assert abs(float(n(loss_ip)[0]) - float(lr_)) <= 1e-4 * abs(float(lr_))
    assert status_ok()


def test_embedding_golden_bitexact(cuda, golden_ops):
    from tinytrain_b200 import kernels as K
    g = golden_ops
    W = t(g["emb_W"], cuda)
    idx = t(g["emb_idx"], cuda)
    out = K.embedding_fwd(W, idx)
    assert np.array_equal(n(out), g["emb_out"])
    dW = torch.zeros_like(W)
    K.embedding_bwd(t(g["emb_G"], cuda), idx, dW)
    assert np.array_equal(n(dW), g["emb_dW"])


@pytest.mark.parametrize("N,V,D", [(2048, 32000, 256), (16384, 32000, 2048), (3000, 7, 64),
                                   (32768, 32000, 512), (40000, 7, 64)])
def test_embedding_scatter_bitexact(cuda, N, V, D):
    """Sequential per-row order of ops.cpp:766-771 reproduced bit for bit,
    including heavy collisions (V = 7) and a non-zero starting gradient. Above
    16384 ids the sort runs in 8192-key shared-memory chunks with the passes
    across chunks in global memory (the 1B micro-batch has 32768)."""
    from oracle import restate as rs
    from tinytrain_b200 import kernels as K
    rng = np.random.default_rng(N + V)
    idx = rng.integers(0, V, N).astype(np.int64)
    g = rng.standard_normal((N, D)).astype(np.float32)
    base = rng.standard_normal((V, D)).astype(np.float32) if V < 100 else np.zeros((V, D), np.float32)
    ref = base.copy()
    for i, tk in enumerate(idx):
        ref[tk] += g[i]
    dW = t(base, cuda)
    K.embedding_bwd(t(g, cuda), t(idx, cuda), dW)
    assert np.array_equal(n(dW), ref)
    W = rng.standard_normal((V, D)).astype(np.float32)
    assert np.array_equal(n(K.embedding_fwd(t(W, cuda), t(idx, cuda))), rs.embedding(W, idx))


def test_embedding_bad_index_is_flagged(cuda):
    from tinytrain_b200 import _ttk, kernels as K
    W = torch.zeros(10, 8, device=cuda)
    idx = torch.tensor([1, 12, 3], dtype=torch.int64, device=cuda)
    K.embedding_fwd(W, idx)
    assert _ttk.device_status() & 2


def test_rope_golden(cuda, golden_ops):
    from tinytrain_b200 import kernels as K
    g = golden_ops
    x, cs, sn, gy = (t(g[k], cuda) for k in ("rope_X", "rope_cos", "rope_sin", "rope_G"))
    y = K.rope_fwd(x, cs, sn)
    dx = K.rope_bwd(gy, cs, sn)
    assert rel_err(n(y), g["rope_Y"]) < TOL
    assert rel_err(n(dx), g["rope_dX"]) < TOL


def test_softmax_golden(cuda, golden_ops):
    from tinytrain_b200 import kernels as K
    g = golden_ops
    x, gy = t(g["sm_X"], cuda), t(g["sm_G"], cuda)
    y = K.softmax_fwd(x)
    dx = K.softmax_bwd(y, gy)
    assert rel_err(n(y), g["sm_Y"]) < TOL
    assert rel_err(n(dx), g["sm_dX"]) < TOL


@pytest.fixture(params=[0, 2], ids=["tensorcore", "mma"])
def attn_impl(request, cuda):
    """Runs a test under each attention engine; restores the default."""
    from tinytrain_b200 import _ttk
    old = _ttk.call("ttk_attention_get_impl")
    _ttk.call("ttk_attention_set_impl", request.param)
    yield request.param
    _ttk.call("ttk_attention_set_impl", old)


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_attention_golden(cuda, golden_ops, tag, attn_impl):
    from tinytrain_b200 import kernels as K
    g = golden_ops
    q, k, v, go = (t(g[f"att_{tag}_{s}"], cuda) for s in ("q", "k", "v", "G"))
    B, T, H, hd = q.shape
    if hd not in (32, 64, 128):
        pytest.skip("head_dim outside the fused kernel's set")
    cs, sn = K.rope_tables(T, hd, 10000.0, cuda)
    o, lse = K.attention_fwd(q, k, v, cs, sn)
    dq, dk, dv = K.attention_bwd(q, k, v, cs, sn, o, lse, go.view(B, T, H, hd))
    assert rel_err(n(o).reshape(B, T, H * hd), g[f"att_{tag}_O"]) < TOL
    assert rel_err(n(dq), g[f"att_{tag}_dq"]) < TOL
    assert rel_err(n(dk), g[f"att_{tag}_dk"]) < TOL
    assert rel_err(n(dv), g[f"att_{tag}_dv"]) < TOL
    assert status_ok()


@pytest.mark.parametrize("B,T,H,hd", [(2, 128, 8, 32), (1, 200, 2, 64), (1, 512, 2, 128),
                                     (1, 70, 3, 32), (1, 333, 1, 128), (2, 1000, 2, 64),
                                     (1, 2048, 1, 128)])
def test_attention_sizes(cuda, B, T, H, hd, attn_impl):
    from oracle import restate as rs
    from tinytrain_b200 import kernels as K
    rng = np.random.default_rng(B * T * H + hd)
    q, k, v = (rng.standard_normal((B, T, H, hd)).astype(np.float32) for _ in range(3))
    go = rng.standard_normal((B, T, H, hd)).astype(np.float32)
    cs, sn = K.rope_tables(T, hd, 10000.0, cuda)
    o, lse = K.attention_fwd(t(q, cuda), t(k, cuda), t(v, cuda), cs, sn)
    dq, dk, dv = K.attention_bwd(t(q, cuda), t(k, cuda), t(v, cuda), cs, sn, o, lse, t(go, cuda))
    orf, cache = rs.attention(q, k, v, 10000.0)
    dqr, dkr, dvr = rs.attention_bwd(go.reshape(B, T, H * hd), cache)
    assert rel_err(n(o).reshape(B, T, H * hd), orf) < TOL
    assert rel_err(n(dq), dqr) < TOL
    assert rel_err(n(dk), dkr) < TOL
    assert rel_err(n(dv), dvr) < TOL


@pytest.mark.parametrize("B,T,H,hd", [(2, 300, 4, 64), (1, 256, 16, 128), (4, 128, 8, 32)])
def test_attention_fwd_split_planes_bitexact(cuda, B, T, H, hd, attn_impl):
    """ttk_attention_fwd_split: o and lse equal ttk_attention_fwd's, and the
    planes equal ttk_gemm_split of o as [B*T, H*hd], bit for bit."""
    from tinytrain_b200 import kernels as K
    g = torch.Generator(device=cuda).manual_seed(B * T + hd)
    q, k, v = (torch.randn(B, T, H, hd, device=cuda, generator=g) for _ in range(3))
    cs, sn = K.rope_tables(T, hd, 10000.0, cuda)
    o0, l0 = K.attention_fwd(q, k, v, cs, sn)
    o1, l1, planes = K.attention_fwd_split(q, k, v, cs, sn)
    ref = K.gemm_split(o1.view(B * T, H * hd))
    torch.cuda.synchronize()
    assert torch.equal(o0, o1) and torch.equal(l0, l1)
    assert torch.equal(planes, ref)
    assert status_ok()


@pytest.mark.parametrize("B,T,H,hd", [(2, 300, 4, 64), (1, 256, 16, 128), (4, 128, 8, 32)])
@pytest.mark.parametrize("accumulate", [False, True])
def test_attention_bwd_split_planes_bitexact(cuda, B, T, H, hd, accumulate, attn_impl):
    """ttk_attention_bwd_split: dq, dk, dv equal ttk_attention_bwd_ex's (with
    and without accumulation into existing gradients), and each plane set
    equals ttk_gemm_split of the stored gradient as [B*T, H*hd], bit for bit."""
    from tinytrain_b200 import kernels as K
    g = torch.Generator(device=cuda).manual_seed(B * T + hd + accumulate)
    q, k, v, do = (torch.randn(B, T, H, hd, device=cuda, generator=g) for _ in range(4))
    cs, sn = K.rope_tables(T, hd, 10000.0, cuda)
    o, lse, fw = K.attention_fwd(q, k, v, cs, sn, keep_ws=True)
    base = [torch.randn(B, T, H, hd, device=cuda, generator=g) for _ in range(3)]
    ref = K.attention_bwd(q, k, v, cs, sn, o, lse, do, out=[x.clone() for x in base],
                          accumulate=accumulate, fwd_ws=fw)
    *got, planes = K.attention_bwd_split(q, k, v, cs, sn, o, lse, do,
                                         out=[x.clone() for x in base], accumulate=accumulate,
                                         fwd_ws=fw)
    for a, b, p in zip(got, ref, planes):
        torch.cuda.synchronize()
        assert torch.equal(a, b)
        assert torch.equal(p, K.gemm_split(a.view(B * T, H * hd)))
    assert status_ok()


@pytest.mark.parametrize("hd", [64, 128])
def test_attention_bwd_accumulates(cuda, hd, attn_impl):
    """accumulate = 1 adds the gradients into dq, dk, dv (the autograd engine's
    += into existing grads, ops.cpp ensure_grad + accumulation)."""
    from tinytrain_b200 import kernels as K
    B, T, H = 1, 300, 2
    rng = np.random.default_rng(hd)
    q, k, v, go = (t(rng.standard_normal((B, T, H, hd)).astype(np.float32), cuda)
                   for _ in range(4))
    cs, sn = K.rope_tables(T, hd, 10000.0, cuda)
    o, lse = K.attention_fwd(q, k, v, cs, sn)
    dq, dk, dv = K.attention_bwd(q, k, v, cs, sn, o, lse, go)
    base = [torch.randn_like(x) for x in (dq, dk, dv)]
    acc = [x.clone() for x in base]
    K.attention_bwd(q, k, v, cs, sn, o, lse, go, out=acc, accumulate=True)
    for a, b0, g in zip(acc, base, (dq, dk, dv)):
        assert rel_err(n(a), n(b0) + n(g)) < 1e-6
    assert status_ok()


@pytest.mark.parametrize("hd", [64, 128, 32])
def test_attention_bwd_reuses_forward_planes(cuda, hd, attn_impl):
    """ttk_attention_bwd_ex with the forward's workspace (its q, k, v planes)
    gives the same gradients, bit for bit, as ttk_attention_bwd, which splits
    q, k, v again."""
    from tinytrain_b200 import kernels as K
    B, T, H = 2, 300, 2
    g = torch.Generator(device=cuda).manual_seed(hd)
    q, k, v, do = (torch.randn(B, T, H, hd, device=cuda, generator=g) for _ in range(4))
    cs, sn = K.rope_tables(T, hd, 10000.0, cuda)
    o, lse, fw = K.attention_fwd(q, k, v, cs, sn, keep_ws=True)
    ref = K.attention_bwd(q, k, v, cs, sn, o, lse, do)
    got = K.attention_bwd(q, k, v, cs, sn, o, lse, do, fwd_ws=fw)
    torch.cuda.synchronize()
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    assert status_ok()


def test_adamw_golden(cuda, golden_ops):
    """6 steps of the fused multi-tensor AdamW equal the reference's AdamW."""
    from tinytrain_b200 import kernels as K
    g = golden_ops
    p = t(g["adam_p"], cuda)
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    for s in range(g["adam_g"].shape[0]):
        gr = t(g["adam_g"][s], cuda)
        K.adamw([p], [gr], [m], [v], 1e-2, 0.9, 0.95, 1e-8, 0.1, s + 1)
    assert rel_err(n(p), g["adam_out"]) < 1e-6


def test_adamw_clip_multi(cuda):
    """Global-norm clipping folded into a multi-tensor AdamW step equals the
    restated clip followed by the reference update rule."""
    from oracle import restate as rs
    from tinytrain_b200 import kernels as K
    rng = np.random.default_rng(3)
    sizes = [1000, 4096, 3, 257, 65536]
    ps = [rng.standard_normal(s).astype(np.float32) for s in sizes]
    gs = [(rng.standard_normal(s) * 0.5).astype(np.float32) for s in sizes]
    dp = [t(x, cuda) for x in ps]
    dg = [t(x, cuda) for x in gs]
    dm = [torch.zeros_like(x) for x in dp]
    dv = [torch.zeros_like(x) for x in dp]
    acc = K.sumsq(dg)
    K.adamw(dp, dg, dm, dv, 3e-4, 0.9, 0.95, 1e-8, 0.1, 1, sumsq_acc=acc, max_norm=1.0)
    gsc = [x.copy() for x in gs]
    total = rs.clip_grad_norm(gsc, 1.0)
    assert abs(float(n(acc)[0]) ** 0.5 - total) <= 1e-9 * total
    for i in range(len(sizes)):
        p, m, v = ps[i].copy(), np.zeros_like(ps[i]), np.zeros_like(ps[i])
        rs.adamw_step(p, gsc[i], m, v, 1, 3e-4, 0.9, 0.95, 1e-8, 0.1)
        assert rel_err(n(dp[i]), p) < 1e-6
