"""ttk_gemm_noalloc: the GEMM entry point for callers that cannot allocate.

Callers inside a fixed memory budget, or on paths that must not allocate
after start-up, cannot provide the device workspace ttk_gemm needs. This
entry point uses a fixed scratch array inside libttk.so instead. The test
calls it through the C ABI twice in a row (the second call on different
shapes and values, so anything left over from the first would show) and
checks each result against ttk_gemm on the same inputs, with the tolerance
of the GEMM tests (max|err| / max|ref| <= 1e-4; the two paths run the same
kernel, so the results are expected to be identical). It also checks that the
device pool's usage does not change across the calls and that an oversized
request is rejected. The file is named to be collected last.

One case has the shape of a weight gradient (A transposed, K = 4096 with a
256 x 256 output): ttk_gemm runs it as split-K slices, the no-alloc entry
never splits, so the case checks that the unsplit path fits the fixed
scratch and gives the same product. Besides the device pool's counters, the
device's free memory (cudaMemGetInfo) is compared across the calls, after
one warm-up round of the same calls has loaded every kernel they use.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.fixture(autouse=True)
def tensor_cores_at_every_size(cuda):
    """The cases below are small enough for ttk_gemm's exact fp32 path; send
    them to the tensor cores so that the split operands use the scratch."""
    from tinytrain_b200 import _ttk
    old = _ttk.call("ttk_gemm_get_fp32_max_macs")
    _ttk.call("ttk_gemm_set_fp32_max_macs", 0)
    yield
    _ttk.call("ttk_gemm_set_fp32_max_macs", old)


def _gemm_ref(A, B, tA, tB, M, N, K, stream):
    from tinytrain_b200 import _ttk
    Cm = torch.empty(M, N, device=A.device)
    ws_n = _ttk.call("ttk_gemm_workspace_size", tA, tB, 1, M, N, K)
    ws = torch.empty(max(ws_n, 16), dtype=torch.uint8, device=A.device)
    _ttk.call("ttk_gemm", tA, tB, 1, M, N, K, 1.0, A.data_ptr(), A.shape[1], 0, B.data_ptr(),
              B.shape[1], 0, 0.0, Cm.data_ptr(), N, 0, ws.data_ptr(), ws.numel(), stream)
    return Cm


def _noalloc(tA, tB, M, N, K, A, B, Cn, stream):
    from tinytrain_b200 import _ttk
    _ttk.call("ttk_gemm_noalloc", tA, tB, 1, M, N, K, 1.0, A.data_ptr(), A.shape[1], 0,
              B.data_ptr(), B.shape[1], 0, 0.0, Cn.data_ptr(), N, 0, stream)


def test_gemm_noalloc_matches_gemm(cuda):
    from tinytrain_b200 import _ttk
    _ttk.lib()
    stream = torch.cuda.current_stream().cuda_stream
    cases = [(0, 1, 300, 260, 200, 11), (1, 0, 128, 96, 384, 12), (1, 0, 256, 256, 4096, 13)]
    # The weight-gradient shape is one that ttk_gemm splits along K.
    assert _ttk.call("ttk_gemm_split_k_slices", 1, 0, 1, 256, 256, 4096) > 1
    cap = _ttk.call("ttk_gemm_noalloc_max_workspace")
    inputs = []
    for tA, tB, M, N, K, seed in cases:
        g = torch.Generator(device=cuda).manual_seed(seed)
        A = torch.rand((K, M) if tA else (M, K), device=cuda, generator=g) * 2 - 1
        B = torch.rand((N, K) if tB else (K, N), device=cuda, generator=g) * 2 - 1
        Cn = torch.full((M, N), float("nan"), device=cuda)
        inputs.append((tA, tB, M, N, K, A, B, Cn))
    # Warm-up round: loads every kernel these calls use, so that the memory
    # comparison below sees only what the calls themselves might allocate.
    warm = [torch.empty_like(x[7]) for x in inputs]
    for (tA, tB, M, N, K, A, B, _), Cw in zip(inputs, warm):
        _noalloc(tA, tB, M, N, K, A, B, Cw, stream)
    torch.cuda.synchronize()
    used0 = C.c_size_t(0)
    _ttk.call("ttk_pool_stats", None, C.byref(used0))
    free0, _ = torch.cuda.mem_get_info()
    for tA, tB, M, N, K, A, B, Cn in inputs:  # calls in a row
        _noalloc(tA, tB, M, N, K, A, B, Cn, stream)
    torch.cuda.synchronize()
    used1 = C.c_size_t(0)
    _ttk.call("ttk_pool_stats", None, C.byref(used1))
    free1, _ = torch.cuda.mem_get_info()
    assert used1.value == used0.value
    assert free1 == free0
    for tA, tB, M, N, K, A, B, Cn in inputs:
        assert _ttk.call("ttk_gemm_workspace_size", tA, tB, 1, M, N, K) <= cap
        ref = _gemm_ref(A, B, tA, tB, M, N, K, stream)
        torch.cuda.synchronize()
        assert rel_err(Cn.cpu().numpy(), ref.cpu().numpy()) < TOL
        exact = (A.double().T if tA else A.double()) @ (B.double().T if tB else B.double())
        assert rel_err(Cn.cpu().numpy(), exact.cpu().numpy()) < TOL
    assert _ttk.device_status() == 0


def test_gemm_noalloc_rejects_oversized(cuda):
    from tinytrain_b200 import _ttk
    cap = _ttk.call("ttk_gemm_noalloc_max_workspace")
    M = N = K = 4096  # split operands need 2 * 2 * 4096 * 4096 * 4 B = 256 MiB
    assert _ttk.call("ttk_gemm_workspace_size", 0, 0, 1, M, N, K) > cap
    # Real buffers of the full size: were the size check ever to let this
    # call through, the GEMM would read and write memory it owns.
    A = torch.zeros(M, K, device=cuda)
    B = torch.zeros(K, N, device=cuda)
    Cn = torch.zeros(M, N, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    with pytest.raises(_ttk.TtkError, match="fixed limit"):
        _ttk.call("ttk_gemm_noalloc", 0, 0, 1, M, N, K, 1.0, A.data_ptr(), K, 0, B.data_ptr(), N,
                  0, 0.0, Cn.data_ptr(), N, 0, stream)
    torch.cuda.synchronize()
