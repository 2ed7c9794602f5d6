"""Thin torch-tensor front end over the ttk C ABI (include/ttk.h).

torch provides device memory and the current stream; every computation is a
ttk_* call into libttk.so. Used by the parity tests and the benchmark to drive
single kernels; the training path itself runs in the C++ tt:: library.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _ttk
from ._ttk import call


def _s():
    return torch.cuda.current_stream().cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _chk(t, name):
    if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()):
        raise ValueError(f"{name}: expected a contiguous float32 CUDA tensor")


def workspace(nbytes: int, device=None) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device or "cuda")


def gemm(A, B, transA=False, transB=False, C_out=None, alpha=1.0, beta=0.0):
    """op(A) @ op(B) (+ beta*C) for 2-D or 3-D (batched) row-major tensors."""
    batched = A.dim() == 3
    if not batched:
        A, B = A.unsqueeze(0), B.unsqueeze(0)
    bt = A.shape[0]
    M, K = (A.shape[2], A.shape[1]) if transA else (A.shape[1], A.shape[2])
    N = B.shape[1] if transB else B.shape[2]
    if C_out is None:
        C_out = torch.empty((bt, M, N), dtype=torch.float32, device=A.device)
        beta = 0.0
    elif not batched:
        C_out = C_out.unsqueeze(0)
    ws_n = call("ttk_gemm_workspace_size", int(transA), int(transB), bt, M, N, K)
    ws = workspace(ws_n, A.device)
    call("ttk_gemm", int(transA), int(transB), bt, M, N, K, alpha, _p(A), A.shape[2],
         A.shape[1] * A.shape[2], _p(B), B.shape[2], B.shape[1] * B.shape[2], beta, _p(C_out),
         N, M * N, _p(ws), ws.numel(), _s())
    return C_out if batched else C_out[0]


def linear_fwd(X, W):
    """Y = X @ W^T (nn.cpp:23-26)."""
    return gemm(X, W, transB=True)


def linear_bwd(X, W, dY):
    """dX = dY @ W, dW = dY^T @ X (ops.cpp:672-694 through the transpose)."""
    return gemm(dY, W), gemm(dY, X, transA=True)


def rmsnorm_fwd(x, w, eps):
    R, D = x.shape
    y = torch.empty_like(x)
    rstd = torch.empty(R, dtype=torch.float32, device=x.device)
    call("ttk_rmsnorm_fwd", _p(x), _p(w), _p(y), _p(rstd), R, D, eps, _s())
    return y, rstd


def rmsnorm_fwd_split(x, w, eps):
    """(y, rstd, planes): the forward plus y's bf16x3 GEMM operand planes."""
    R, D = x.shape
    y = torch.empty_like(x)
    rstd = torch.empty(R, dtype=torch.float32, device=x.device)
    planes = workspace(call("ttk_gemm_split_bytes", 1, R, D), x.device)
    call("ttk_rmsnorm_fwd_split", _p(x), _p(w), _p(y), _p(rstd), R, D, eps, _p(planes), _s())
    return y, rstd, planes


def gemm_split(x):
    """bf16x3 operand planes of a 2-D fp32 tensor (ttk_gemm_split)."""
    R, D = x.shape
    planes = workspace(call("ttk_gemm_split_bytes", 1, R, D), x.device)
    call("ttk_gemm_split", _p(x), R, D, D, 0, 1, _p(planes), _s())
    return planes


def rmsnorm_bwd(x, w, rstd, dy, dx=None, dw=None, accumulate=False):
    R, D = x.shape
    if dx is None:
        dx = torch.empty_like(x)
    if dw is None:
        dw = torch.zeros_like(w)
    ws_n = call("ttk_rmsnorm_bwd_workspace_size", R, D)
    ws = workspace(ws_n, x.device)
    call("ttk_rmsnorm_bwd", _p(x), _p(w), _p(rstd), _p(dy), _p(dx), int(accumulate), _p(dw), R, D,
         _p(ws), ws.numel(), _s())
    return dx, dw


def swiglu_fwd(a, b):
    y = torch.empty_like(a)
    call("ttk_swiglu_fwd", _p(a), _p(b), _p(y), a.numel(), _s())
    return y


def swiglu_bwd(a, b, dy, da=None, db=None, accumulate=False):
    da = torch.empty_like(a) if da is None else da
    db = torch.empty_like(b) if db is None else db
    call("ttk_swiglu_bwd", _p(a), _p(b), _p(dy), _p(da), _p(db), int(accumulate), a.numel(), _s())
    return da, db


def cross_entropy(logits, targets, want_grad=True, dlogits=None):
    """Mean CE loss (ops.cpp:928-930) and d(loss)/d(logits) for d(loss) = 1."""
    N, Cn = logits.shape
    acc = torch.zeros(1, dtype=torch.float64, device=logits.device)
    if want_grad and dlogits is None:
        dlogits = torch.empty_like(logits)
    call("ttk_cross_entropy", _p(logits), _p(targets), N, Cn, _p(acc),
         _p(dlogits) if want_grad else None, 1.0 / N, _s())
    loss = torch.empty(1, dtype=torch.float32, device=logits.device)
    call("ttk_loss_finalize", _p(acc), 1.0 / N, _p(loss), _s())
    return loss, dlogits


def embedding_fwd(W, idx):
    V, D = W.shape
    N = idx.numel()
    out = torch.empty((N, D), dtype=torch.float32, device=W.device)
    call("ttk_embedding_fwd", _p(W), _p(idx), _p(out), N, D, V, _s())
    return out


def embedding_bwd(dout, idx, dW):
    V, D = dW.shape
    N = idx.numel()
    ws = workspace(call("ttk_embedding_bwd_workspace_size", N), dW.device)
    call("ttk_embedding_bwd", _p(dout), _p(idx), _p(dW), N, D, V, _p(ws), ws.numel(), _s())
    return dW


def rope_fwd(x, cos, sin):
    B, T, H, D = x.shape
    y = torch.empty_like(x)
    call("ttk_rope_fwd", _p(x), _p(cos), _p(sin), _p(y), B, T, H, D, _s())
    return y


def rope_bwd(dy, cos, sin, dx=None, accumulate=False):
    B, T, H, D = dy.shape
    dx = torch.empty_like(dy) if dx is None else dx
    call("ttk_rope_bwd", _p(dy), _p(cos), _p(sin), _p(dx), int(accumulate), B, T, H, D, _s())
    return dx


def softmax_fwd(x, log=False):
    R, Cn = x.shape
    y = torch.empty_like(x)
    call("ttk_softmax_fwd", _p(x), _p(y), R, Cn, int(log), _s())
    return y


def softmax_bwd(y, dy, log=False, dx=None, accumulate=False):
    R, Cn = y.shape
    dx = torch.empty_like(y) if dx is None else dx
    call("ttk_softmax_bwd", _p(y), _p(dy), _p(dx), int(accumulate), R, Cn, int(log), _s())
    return dx


def rope_tables(T, hd, theta, device):
    """model.cpp:43-53 in float32 (computed on the host, as the model does)."""
    import numpy as np
    i = np.arange(hd // 2, dtype=np.float32)
    inv = np.float32(1) / np.power(np.float32(theta), (np.float32(2) * i) / np.float32(hd),
                                   dtype=np.float32)
    ang = np.arange(T, dtype=np.float32)[:, None] * inv[None, :]
    return (torch.from_numpy(np.cos(ang).astype(np.float32)).to(device),
            torch.from_numpy(np.sin(ang).astype(np.float32)).to(device))


def attention_fwd(q, k, v, cos, sin, scale=None, keep_ws=False):
    """(o, lse); with keep_ws also the workspace (q, k, v planes) for attention_bwd(fwd_ws=)."""
    B, T, H, hd = q.shape
    scale = float(hd) ** -0.5 if scale is None else scale
    o = torch.empty_like(q)
    lse = torch.empty((B, H, T), dtype=torch.float32, device=q.device)
    ws = workspace(call("ttk_attention_fwd_workspace_size", B, T, H, hd), q.device)
    call("ttk_attention_fwd", _p(q), _p(k), _p(v), _p(cos), _p(sin), _p(o), _p(lse), B, T, H, hd,
         scale, _p(ws), ws.numel(), _s())
    return (o, lse, ws) if keep_ws else (o, lse)


def attention_fwd_split(q, k, v, cos, sin, scale=None):
    """(o, lse, planes): the forward plus o's bf16x3 operand planes ([B*T, H*hd])."""
    B, T, H, hd = q.shape
    scale = float(hd) ** -0.5 if scale is None else scale
    o = torch.empty_like(q)
    lse = torch.empty((B, H, T), dtype=torch.float32, device=q.device)
    ws = workspace(call("ttk_attention_fwd_workspace_size", B, T, H, hd), q.device)
    planes = workspace(call("ttk_gemm_split_bytes", 1, B * T, H * hd), q.device)
    call("ttk_attention_fwd_split", _p(q), _p(k), _p(v), _p(cos), _p(sin), _p(o), _p(lse),
         _p(planes), B, T, H, hd, scale, _p(ws), ws.numel(), _s())
    return o, lse, planes


def attention_bwd(q, k, v, cos, sin, o, lse, do, scale=None, out=None, accumulate=False,
                  fwd_ws=None):
    """dq, dk, dv; with `out` = (dq, dk, dv) writes (or, with accumulate, adds) into them.
    fwd_ws: the forward's workspace (attention_fwd(keep_ws=True)), whose q, k, v planes are
    reused."""
    B, T, H, hd = q.shape
    scale = float(hd) ** -0.5 if scale is None else scale
    dq, dk, dv = out if out is not None else (torch.empty_like(q), torch.empty_like(k),
                                               torch.empty_like(v))
    if fwd_ws is not None and fwd_ws.numel() > 0:
        ws = workspace(call("ttk_attention_bwd_ex_workspace_size", B, T, H, hd), q.device)
        call("ttk_attention_bwd_ex", _p(q), _p(k), _p(v), _p(cos), _p(sin), _p(o), _p(lse),
             _p(do), _p(dq), _p(dk), _p(dv), int(accumulate), B, T, H, hd, scale, _p(fwd_ws),
             _p(ws), ws.numel(), _s())
        return dq, dk, dv
    ws = workspace(call("ttk_attention_bwd_workspace_size", B, T, H, hd), q.device)
    call("ttk_attention_bwd", _p(q), _p(k), _p(v), _p(cos), _p(sin), _p(o), _p(lse), _p(do),
         _p(dq), _p(dk), _p(dv), int(accumulate), B, T, H, hd, scale, _p(ws), ws.numel(), _s())
    return dq, dk, dv


def attention_bwd_split(q, k, v, cos, sin, o, lse, do, scale=None, out=None, accumulate=False,
                        fwd_ws=None):
    """(dq, dk, dv, planes): the backward plus the bf16x3 operand planes of dq,
    dk, dv, each as [B*T, H*hd] rows."""
    B, T, H, hd = q.shape
    scale = float(hd) ** -0.5 if scale is None else scale
    dq, dk, dv = out if out is not None else (torch.empty_like(q), torch.empty_like(k),
                                               torch.empty_like(v))
    reuse = fwd_ws is not None and fwd_ws.numel() > 0
    ws = workspace(call("ttk_attention_bwd_ex_workspace_size" if reuse else
                        "ttk_attention_bwd_workspace_size", B, T, H, hd), q.device)
    pb = call("ttk_gemm_split_bytes", 1, B * T, H * hd)
    planes = [workspace(pb, q.device) for _ in range(3)]
    call("ttk_attention_bwd_split", _p(q), _p(k), _p(v), _p(cos), _p(sin), _p(o), _p(lse),
         _p(do), _p(dq), _p(dk), _p(dv), int(accumulate), B, T, H, hd, scale,
         _p(fwd_ws) if reuse else None, _p(ws), ws.numel(), *(_p(x) for x in planes), _s())
    return dq, dk, dv, planes


def sumsq(tensors):
    acc = torch.zeros(1, dtype=torch.float64, device=tensors[0].device)
    ptrs = _ttk.ptr_array([t.data_ptr() for t in tensors])
    sizes = _ttk.i64_array([t.numel() for t in tensors])
    call("ttk_sumsq_multi", ptrs, sizes, len(tensors), _p(acc), _s())
    return acc


def adamw(params, grads, ms, vs, lr, b1, b2, eps, wd, step, sumsq_acc=None, max_norm=0.0,
          grad_scale=1.0):
    n = len(params)
    call("ttk_adamw_multi", _ttk.ptr_array([p.data_ptr() for p in params]),
         _ttk.ptr_array([g.data_ptr() for g in grads]), _ttk.ptr_array([m.data_ptr() for m in ms]),
         _ttk.ptr_array([v.data_ptr() for v in vs]), _ttk.i64_array([p.numel() for p in params]),
         n, lr, b1, b2, eps, wd, step, _p(sumsq_acc), max_norm, grad_scale, _s())
