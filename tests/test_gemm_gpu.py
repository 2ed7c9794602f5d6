"""Parity of the tcgen05 3xTF32 GEMM (ttk_gemm) with the reference's sgemm.

Small shapes: against fixtures the reference produced (tests/golden/
ops_small.npz: matmul forward, dA = G B^T, dB = A^T G; Linear through the
transpose; bmm). Sweep shapes (M, K, N) of the op-level benchmark: against an
fp64 product on the same seeded U(-1, 1) inputs, for forward, dX and dW.
Tolerance: max|err| / max|ref| <= 1e-4 (the per-op bound), the 3xTF32 path
typically lands near 1e-6.
"""
import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.fixture(autouse=True)
def tensor_cores_at_every_size(cuda):
    """These tests cover the tcgen05 kernel, its tile edges included: small
    problems, which ttk_gemm otherwise runs as exact fp32 SIMT, are sent to
    the tensor cores too (tests/test_gemm_fp32_gpu.py covers that path)."""
    from tinytrain_b200 import _ttk
    old = _ttk.call("ttk_gemm_get_fp32_max_macs")
    _ttk.call("ttk_gemm_set_fp32_max_macs", 0)
    yield
    _ttk.call("ttk_gemm_set_fp32_max_macs", old)


def t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("tag", ["a", "b", "c", "d"])
def test_matmul_golden(cuda, golden_ops, tag):
    from tinytrain_b200 import kernels as K
    g = golden_ops
    A, B, G = (t(g[f"mm_{tag}_{n}"], cuda) for n in "ABG")
    C = K.gemm(A, B)
    dA = K.gemm(G, B, transB=True)
    dB = K.gemm(A, G, transA=True)
    torch.cuda.synchronize()
    assert rel_err(C.cpu().numpy(), g[f"mm_{tag}_C"]) < TOL
    assert rel_err(dA.cpu().numpy(), g[f"mm_{tag}_dA"]) < TOL
    assert rel_err(dB.cpu().numpy(), g[f"mm_{tag}_dB"]) < TOL


def test_linear_golden(cuda, golden_ops):
    from tinytrain_b200 import kernels as K
    g = golden_ops
    X, W, G = t(g["lin_X"], cuda), t(g["lin_W"], cuda), t(g["lin_G"], cuda)
    Y = K.linear_fwd(X, W)
    dX, dW = K.linear_bwd(X, W, G)
    assert rel_err(Y.cpu().numpy(), g["lin_Y"]) < TOL
    assert rel_err(dX.cpu().numpy(), g["lin_dX"]) < TOL
    assert rel_err(dW.cpu().numpy(), g["lin_dW"]) < TOL


def test_bmm_golden(cuda, golden_ops):
    from tinytrain_b200 import kernels as K
    g = golden_ops
    A, B, G = t(g["bmm_A"], cuda), t(g["bmm_B"], cuda), t(g["bmm_G"], cuda)
    C = K.gemm(A, B)
    dA = K.gemm(G, B, transB=True)
    dB = K.gemm(A, G, transA=True)
    assert rel_err(C.cpu().numpy(), g["bmm_C"]) < TOL
    assert rel_err(dA.cpu().numpy(), g["bmm_dA"]) < TOL
    assert rel_err(dB.cpu().numpy(), g["bmm_dB"]) < TOL


def test_accumulate_beta(cuda):
    from tinytrain_b200 import kernels as K
    gen = torch.Generator(device=cuda).manual_seed(5)
    A = torch.rand(300, 200, device=cuda, generator=gen) * 2 - 1
    B = torch.rand(200, 260, device=cuda, generator=gen) * 2 - 1
    C0 = torch.rand(300, 260, device=cuda, generator=gen) * 2 - 1
    C = C0.clone()
    K.gemm(A, B, C_out=C, beta=1.0)
    ref = C0.double() + A.double() @ B.double()
    assert rel_err(C.cpu().numpy(), ref.cpu().numpy()) < TOL
    C = C0.clone()
    K.gemm(A, B, C_out=C, alpha=0.5, beta=-2.0)
    ref = -2.0 * C0.double() + 0.5 * (A.double() @ B.double())
    assert rel_err(C.cpu().numpy(), ref.cpu().numpy()) < TOL


@pytest.mark.parametrize("N", [36, 37, 300])
@pytest.mark.parametrize("beta", [0.0, 1.0])
def test_batched_edges_and_epilogue_modes(cuda, N, beta):
    """Batched GEMM whose tiles overhang M and N: the TMA-store / TMA-add
    epilogue (N = 36, 300: 16-byte rows) and the direct one (N = 37) give the
    same values, with beta = 0 (overwrite) and beta = 1 (accumulate)."""
    from tinytrain_b200 import kernels as K
    gen = torch.Generator(device=cuda).manual_seed(N + int(beta))
    A = torch.rand(3, 130, 70, device=cuda, generator=gen) * 2 - 1
    B = torch.rand(3, 70, N, device=cuda, generator=gen) * 2 - 1
    C0 = torch.rand(3, 130, N, device=cuda, generator=gen) * 2 - 1
    C = C0.clone()
    K.gemm(A, B, C_out=C, beta=beta)
    ref = beta * C0.double() + A.double() @ B.double()
    assert rel_err(C.cpu().numpy(), ref.cpu().numpy()) < TOL


@pytest.fixture
def pair_mode(cuda):
    """Sets the CTA-pair mode for one test and restores the previous one."""
    from tinytrain_b200 import _ttk
    old = _ttk.call("ttk_gemm_get_cta_pairs")

    def set_mode(m):
        _ttk.call("ttk_gemm_set_cta_pairs", m)
    yield set_mode
    _ttk.call("ttk_gemm_set_cta_pairs", old)


@pytest.mark.parametrize("tA,tB", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("batch,M,N,K", [(1, 300, 520, 200), (3, 130, 300, 70),
                                         (1, 2248, 1000, 1000), (2, 256, 256, 32)])
def test_cta_pair_tiles(cuda, pair_mode, tA, tB, batch, M, N, K):
    """256 x 256 tiles on CTA pairs (cta_group::2), forced onto small problems
    whose last tiles overhang M (a pair's second CTA partly or wholly past the
    last row) and N, with both operand orientations, several K chunks, and
    the three epilogue modes (TMA store for beta = 0, TMA reduce-add for
    beta = 1, direct stores otherwise). Equal to fp64 within the bound, and to
    the single-CTA kernel bit for bit (the same products summed in the same
    order)."""
    from tinytrain_b200 import kernels as Kn
    gen = torch.Generator(device=cuda).manual_seed(M + N + K + 10 * tA + tB)
    A = torch.rand((batch, K, M) if tA else (batch, M, K), device=cuda, generator=gen) * 2 - 1
    B = torch.rand((batch, N, K) if tB else (batch, K, N), device=cuda, generator=gen) * 2 - 1
    C0 = torch.rand(batch, M, N, device=cuda, generator=gen) * 2 - 1
    oA = A.double().transpose(1, 2) if tA else A.double()
    oB = B.double().transpose(1, 2) if tB else B.double()
    prod = oA @ oB
    for alpha, beta in [(1.0, 0.0), (1.0, 1.0), (0.5, -2.0)]:
        out = {}
        for mode in (2, 0):
            pair_mode(mode)
            C = C0.clone()
            Kn.gemm(A, B, transA=bool(tA), transB=bool(tB), C_out=C, alpha=alpha, beta=beta)
            torch.cuda.synchronize()
            out[mode] = C
        ref = alpha * prod + beta * C0.double()
        assert rel_err(out[2].cpu().numpy(), ref.cpu().numpy()) < TOL, (alpha, beta)
        assert torch.equal(out[2], out[0]), (alpha, beta)
    from tinytrain_b200 import _ttk
    assert _ttk.device_status() == 0


@pytest.mark.parametrize("M,K,N", [(2048, 256, 256), (2048, 256, 32000), (8192, 768, 2048),
                                   (16384, 2048, 5632)])
def test_sweep_shapes(cuda, M, K, N):
    """Linear forward (X W^T), dX (dY W) and dW (dY^T X) at the sweep shapes."""
    from tinytrain_b200 import kernels as Kn
    gen = torch.Generator(device=cuda).manual_seed(M + K + N)
    X = torch.rand(M, K, device=cuda, generator=gen) * 2 - 1
    W = torch.rand(N, K, device=cuda, generator=gen) * 2 - 1
    dY = torch.rand(M, N, device=cuda, generator=gen) * 2 - 1
    Y = Kn.linear_fwd(X, W)
    dX, dW = Kn.linear_bwd(X, W, dY)
    Xd, Wd, dYd = X.double(), W.double(), dY.double()
    for got, ref in ((Y, Xd @ Wd.T), (dX, dYd @ Wd), (dW, dYd.T @ Xd)):
        err = (got.double() - ref).abs().max().item() / ref.abs().max().item()
        assert err < TOL, err
    from tinytrain_b200 import _ttk
    assert _ttk.device_status() == 0


def test_rejects_bad_args(cuda):
    from tinytrain_b200 import _ttk
    with pytest.raises(_ttk.TtkError):
        _ttk.call("ttk_gemm", 0, 0, 1, 4, 4, 4, 1.0, None, 4, 16, None, 4, 16, 0.0, None, 4, 16,
                  None, 0, None)


@pytest.fixture
def split_k(cuda):
    from tinytrain_b200 import _ttk
    old = _ttk.call("ttk_gemm_get_split_k")

    def set_on(on):
        _ttk.call("ttk_gemm_set_split_k", int(on))
    yield set_on
    _ttk.call("ttk_gemm_set_split_k", old)


def _gemm_on_splits(A, B, tA, tB, M, N, K, alpha, beta, C):
    """The host path: operands split once (ttk_gemm_split), then ttk_gemm_splits."""
    from tinytrain_b200 import _ttk
    st = torch.cuda.current_stream().cuda_stream
    splits = []
    for X in (A, B):
        rows, cols = X.shape
        buf = torch.empty(_ttk.call("ttk_gemm_split_bytes", 1, rows, cols), dtype=torch.uint8,
                          device=X.device)
        _ttk.call("ttk_gemm_split", X.data_ptr(), rows, cols, cols, 0, 1, buf.data_ptr(), st)
        splits.append(buf)
    _ttk.call("ttk_gemm_splits", tA, tB, 1, M, N, K, alpha, splits[0].data_ptr(),
              splits[1].data_ptr(), beta, C.data_ptr(), N, 0, st)


@pytest.mark.parametrize("M,N,K,S,orients", [
    (2048, 2048, 16384, 8, [(1, 0)]),            # attention projection dW = dY^T X
    (5632, 2048, 16384, 2, [(1, 0)]),            # FFN dW
    (300, 260, 8192, 16, [(0, 0), (0, 1), (1, 0), (1, 1)])])
def test_split_k(cuda, split_k, M, N, K, S, orients):
    """Long-K GEMMs with few output tiles run as S K-slices plus an in-order
    sum of the partial products: equal to fp64 within the bound through both
    entry points (caller workspace; cached operand splits with pool-allocated
    partials), with beta = 0, 1 and other alpha / beta, and close to the
    unsplit result."""
    from tinytrain_b200 import _ttk
    from tinytrain_b200 import kernels as Kn
    for tA, tB in orients:
        split_k(True)
        assert _ttk.call("ttk_gemm_split_k_slices", tA, tB, 1, M, N, K) == S
        gen = torch.Generator(device=cuda).manual_seed(M + N + K + tA + 2 * tB)
        A = torch.rand((K, M) if tA else (M, K), device=cuda, generator=gen) * 2 - 1
        B = torch.rand((N, K) if tB else (K, N), device=cuda, generator=gen) * 2 - 1
        C0 = torch.rand(M, N, device=cuda, generator=gen) * 2 - 1
        prod = (A.double().T if tA else A.double()) @ (B.double().T if tB else B.double())
        for alpha, beta in [(1.0, 0.0), (1.0, 1.0), (0.5, -0.5)]:
            ref = (alpha * prod + beta * C0.double()).cpu().numpy()
            split_k(True)
            C1 = C0.clone()
            Kn.gemm(A, B, transA=bool(tA), transB=bool(tB), C_out=C1, alpha=alpha, beta=beta)
            C2 = C0.clone()
            _gemm_on_splits(A, B, tA, tB, M, N, K, alpha, beta, C2)
            split_k(False)
            assert _ttk.call("ttk_gemm_split_k_slices", tA, tB, 1, M, N, K) == 1
            C3 = C0.clone()
            Kn.gemm(A, B, transA=bool(tA), transB=bool(tB), C_out=C3, alpha=alpha, beta=beta)
            torch.cuda.synchronize()
            for got in (C1, C2):
                assert rel_err(got.cpu().numpy(), ref) < TOL, (tA, tB, alpha, beta)
            assert torch.equal(C1, C2)
            assert rel_err(C1.cpu().numpy(), C3.cpu().numpy()) < 1e-5
    assert _ttk.device_status() == 0
