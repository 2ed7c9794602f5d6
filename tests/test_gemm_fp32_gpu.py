"""The exact fp32 path of ttk_gemm for small problems (at most 2^24
multiply-adds by default): one fp32 fused multiply-add per product in
ascending k, the reference's sgemm arithmetic (ops.cpp:96-125).

Checked against the reference's own matmul fixtures (tests/golden/
ops_small.npz), against an fp64 product at 1e-6 (tighter than the split
GEMM's 1e-4 bound), and by the property the reference's gradient checks rely
on (tests/test_autograd.cpp, Autograd.Matmul): central differences of
sum(A @ B) with eps = 1e-3 reproduce the exact derivative within the
reference's tolerance, which the split's truncation steps break."""
import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_dispatch_rule(cuda):
    from tinytrain_b200 import _ttk
    old = _ttk.call("ttk_gemm_get_fp32_max_macs")
    assert old == 1 << 24
    assert _ttk.call("ttk_gemm_uses_fp32", 1, 4, 5, 3) == 1
    assert _ttk.call("ttk_gemm_uses_fp32", 4, 64, 256, 256) == 1      # 2^24 exactly
    assert _ttk.call("ttk_gemm_uses_fp32", 4, 65, 256, 256) == 0
    assert _ttk.call("ttk_gemm_uses_fp32", 1, 16384, 2048, 2048) == 0
    assert _ttk.call("ttk_gemm_workspace_size", 0, 0, 1, 4, 5, 3) == 0
    try:
        _ttk.call("ttk_gemm_set_fp32_max_macs", 0)
        assert _ttk.call("ttk_gemm_uses_fp32", 1, 4, 5, 3) == 0
        with pytest.raises(_ttk.TtkError):
            _ttk.call("ttk_gemm_set_fp32_max_macs", -1)
    finally:
        _ttk.call("ttk_gemm_set_fp32_max_macs", old)


@pytest.mark.parametrize("tag", ["a", "b", "c", "d"])
def test_matmul_golden(cuda, golden_ops, tag):
    from tinytrain_b200 import _ttk
    from tinytrain_b200 import kernels as K
    g = golden_ops
    A, B, G = (t(g[f"mm_{tag}_{n}"], cuda) for n in "ABG")
    assert _ttk.call("ttk_gemm_uses_fp32", 1, A.shape[0], B.shape[1], A.shape[1]) == 1
    C = K.gemm(A, B)
    dA = K.gemm(G, B, transB=True)
    dB = K.gemm(A, G, transA=True)
    torch.cuda.synchronize()
    assert rel_err(C.cpu().numpy(), g[f"mm_{tag}_C"]) < 1e-6
    assert rel_err(dA.cpu().numpy(), g[f"mm_{tag}_dA"]) < 1e-6
    assert rel_err(dB.cpu().numpy(), g[f"mm_{tag}_dB"]) < 1e-6


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("batch,M,N,K", [(1, 1, 1, 1), (3, 37, 45, 29), (1, 64, 64, 64),
                                         (2, 130, 7, 300), (1, 33, 1000, 65)])
def test_against_fp64(cuda, ta, tb, batch, M, N, K):
    from tinytrain_b200 import _ttk
    from tinytrain_b200 import kernels as K_
    assert _ttk.call("ttk_gemm_uses_fp32", batch, M, N, K) == 1
    rng = np.random.default_rng(M * 7 + N * 3 + K + ta * 2 + tb)
    a = rng.uniform(-1, 1, (batch, K, M) if ta else (batch, M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (batch, N, K) if tb else (batch, K, N)).astype(np.float32)
    c0 = rng.uniform(-1, 1, (batch, M, N)).astype(np.float32)
    oa = np.swapaxes(a, 1, 2) if ta else a
    ob = np.swapaxes(b, 1, 2) if tb else b
    prod = np.einsum("bmk,bkn->bmn", oa.astype(np.float64), ob.astype(np.float64))
    for alpha, beta in [(1.0, 0.0), (0.7, 1.0), (1.0, -0.5)]:
        C = t(c0, cuda)
        K_.gemm(t(a, cuda), t(b, cuda), transA=bool(ta), transB=bool(tb), C_out=C, alpha=alpha,
                beta=beta)
        ref = alpha * prod + beta * c0.astype(np.float64)
        torch.cuda.synchronize()
        assert rel_err(C.cpu().numpy(), ref) < 1e-6, (alpha, beta)


def test_finite_difference_gradients(cuda):
    """Central differences of sum(A @ B) in fp32 agree with the analytic
    derivative sum_j B[k, j] within the reference's gradcheck tolerance
    (atol 2e-3 + rtol 2e-2)."""
    from tinytrain_b200 import kernels as K
    rng = np.random.default_rng(18)
    a = rng.standard_normal((4, 5)).astype(np.float32)
    b = rng.standard_normal((5, 3)).astype(np.float32)
    B = t(b, cuda)
    eps = 1e-3

    def f(x):
        return float(K.gemm(t(x, cuda), B).sum(dtype=torch.float32).cpu())

    exact = np.broadcast_to(b.sum(1)[None, :], a.shape)
    worst = 0.0
    for i in range(4):
        for k in range(5):
            ap, am = a.copy(), a.copy()
            ap[i, k] += eps
            am[i, k] -= eps
            num = (f(ap) - f(am)) / (2 * eps)
            worst = max(worst, abs(num - exact[i, k]) / (2e-3 + 2e-2 * abs(exact[i, k])))
    assert worst <= 1.0, worst
