"""Op-level benchmark of the device kernels (one JSON line per op).

    python -m tinytrain_b200.opbench                 # the whole sweep
    python -m tinytrain_b200.opbench --only gemm --shape 16384,2048,5632
    python -m tinytrain_b200.opbench --only ce --rows 16384

Workloads (fp32, seeded):
  gemm       matmul forward (X W^T), dX (dY W) and dW (dY^T X) at
             (M, K, N) in {(2048,256,256), (2048,256,32000), (8192,768,2048),
             (16384,2048,5632)}, inputs U(-1, 1)
  rmsnorm / swiglu / ce
             forward + backward at rows = one micro-batch of the bench's 13M,
             110M and 1B configs (2048, 65536, 32768), d / F of the config,
             vocab 32000 for CE
  hbm        AdamW + global-norm clip over the 1B model's 887.7M parameters,
             embedding gather / scatter-add and the residual add at 16384 x 2048
  attention  fused causal attention with RoPE, forward + backward, B 8, H 12,
             hd 64, S in {128, 512, 1024, 2048}, inputs N(0, 1) (--hd 128:
             B 8, H 16, the 1B layer; --hd 32: B 16, H 8, the 13M default
             model; --batch / --heads override)
Each line: median of `--iters` timed launches (CUDA events, after warm-up, L2
flushed by a 256 MB write before each), the algorithmic work (FLOPs, or bytes
that must cross HBM), achieved rate and fraction of the measured peak
(MEASURED_PEAKS.json, else the pool's earlier figures: bf16 burst for tensor
work, HBM copy bandwidth for memory-bound kernels). The bf16x3 GEMM's
fp32-accurate ceiling is the bf16 peak / 3.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import numpy as np
import torch

from . import _ttk, kernels as K

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GEMM_SHAPES = [(2048, 256, 256), (2048, 256, 32000), (8192, 768, 2048), (16384, 2048, 5632)]
# (rows, d, F): rows = one micro-batch of the bench's configs (13M 16 x 128,
# 110M 64 x 1024, 1B 16 x 2048)
ROWS = [(2048, 256, 768), (65536, 768, 2048), (32768, 2048, 5632)]
ATTN_S = [128, 512, 1024, 2048]


def peaks():
    try:
        d = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


_FLUSH = None


def flush_l2():
    """Writes 256 MB (twice the 126 MB L2) so the next launch starts cold."""
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    _FLUSH.fill_(1.0)


def timed(fn, iters, warmup=3):
    """Median of `iters` CUDA-event timings of fn, L2 flushed before each."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush_l2()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def emit(rec):
    print(json.dumps(rec), flush=True)


def bench_gemm(shapes, iters):
    hbm, bf16, src = peaks()
    s = torch.cuda.current_stream().cuda_stream
    for (M, Kd, N) in shapes:
        g = torch.Generator(device="cuda").manual_seed(M + Kd + N)
        X = torch.rand(M, Kd, device="cuda", generator=g) * 2 - 1
        W = torch.rand(N, Kd, device="cuda", generator=g) * 2 - 1
        dY = torch.rand(M, N, device="cuda", generator=g) * 2 - 1
        for name, (tA, tB, A, B, m, n, k) in {
                "fwd": (0, 1, X, W, M, N, Kd), "dX": (0, 0, dY, W, M, Kd, N),
                "dW": (1, 0, dY, X, N, Kd, M)}.items():
            C = torch.empty(m, n, device="cuda")
            wsn = _ttk.call("ttk_gemm_workspace_size", tA, tB, 1, m, n, k)
            ws = torch.empty(wsn, dtype=torch.uint8, device="cuda")

            def run():
                _ttk.call("ttk_gemm", tA, tB, 1, m, n, k, 1.0, A.data_ptr(), A.shape[1], 0,
                          B.data_ptr(), B.shape[1], 0, 0.0, C.data_ptr(), n, 0, ws.data_ptr(),
                          wsn, s)
            ms = timed(run, iters)
            tf = 2 * m * n * k / ms / 1e9
            prec = "tf32x3" if _ttk.call("ttk_gemm_get_precision") == 1 else "bf16x3"
            div = 6 if prec == "tf32x3" else 3
            emit({"op": "gemm", "pass": name, "M": m, "N": n, "K": k, "ms": ms, "split": prec,
                  "tflops_fp32_accurate": tf, "peak_bf16": bf16, "peak_src": src,
                  "frac_of_split3_ceiling": tf / (bf16 / div), "frac_of_bf16_peak": tf / bf16,
                  "includes": "operand split (hi/lo) + tcgen05 kernel"})


def bench_rows(rows, iters, ops=("rmsnorm", "swiglu", "ce")):
    hbm, _, src = peaks()
    for (R, D, F) in rows:
        if "rmsnorm" in ops:
            bench_rmsnorm(R, D, iters, hbm, src)
        if "swiglu" in ops:
            bench_swiglu(R, F, iters, hbm)
        if "ce" in ops:
            bench_ce(R, iters, hbm)


def bench_rmsnorm(R, D, iters, hbm, src):
    x = torch.rand(R, D, device="cuda") * 2 - 1
    w = torch.rand(D, device="cuda")
    dy = torch.rand(R, D, device="cuda") * 2 - 1
    y, rstd = K.rmsnorm_fwd(x, w, 1e-5)
    ms = timed(lambda: K.rmsnorm_fwd(x, w, 1e-5), iters)
    emit({"op": "rmsnorm", "pass": "fwd", "rows": R, "d": D, "ms": ms,
          "gbs": 8 * R * D / ms / 1e6, "frac_hbm": 8 * R * D / ms / 1e6 / hbm,
          "peak_src": src})
    dx, dw = torch.empty_like(x), torch.zeros_like(w)
    ms = timed(lambda: K.rmsnorm_bwd(x, w, rstd, dy, dx=dx, dw=dw), iters)
    emit({"op": "rmsnorm", "pass": "bwd", "rows": R, "d": D, "ms": ms,
          "gbs": 12 * R * D / ms / 1e6, "frac_hbm": 12 * R * D / ms / 1e6 / hbm})


def bench_swiglu(R, F, iters, hbm):
    a = torch.rand(R, F, device="cuda") * 8 - 4
    b = torch.rand(R, F, device="cuda") * 2 - 1
    g = torch.rand(R, F, device="cuda") * 2 - 1
    ms = timed(lambda: K.swiglu_fwd(a, b), iters)
    emit({"op": "swiglu", "pass": "fwd", "rows": R, "F": F, "ms": ms,
          "gbs": 12 * R * F / ms / 1e6, "frac_hbm": 12 * R * F / ms / 1e6 / hbm})
    da, db = torch.empty_like(a), torch.empty_like(b)
    ms = timed(lambda: K.swiglu_bwd(a, b, g, da=da, db=db), iters)
    emit({"op": "swiglu", "pass": "bwd", "rows": R, "F": F, "ms": ms,
          "gbs": 20 * R * F / ms / 1e6, "frac_hbm": 20 * R * F / ms / 1e6 / hbm})


def bench_ce(R, iters, hbm):
    V = 32000
    L = torch.randn(R, V, device="cuda") * 3
    t = torch.randint(0, V, (R,), device="cuda", dtype=torch.int64)
    dL = torch.empty_like(L)
    ms = timed(lambda: K.cross_entropy(L, t, dlogits=dL), iters)
    emit({"op": "cross_entropy", "pass": "fwd+bwd fused", "rows": R, "vocab": V, "ms": ms,
          "gbs": 8 * R * V / ms / 1e6, "frac_hbm": 8 * R * V / ms / 1e6 / hbm})
    del L, dL


def llama1b_param_shapes(d=2048, layers=16, ffn=5632, vocab=32000):
    """Parameter sizes of the 1B model in parameters() order (tied head)."""
    sizes = [vocab * d]
    for _ in range(layers):
        sizes += [d, d * d, d * d, d * d, d * d, d, ffn * d, ffn * d, d * ffn]
    return sizes + [d]


def bench_hbm(iters):
    """The remaining bandwidth kernels at the 1B sizes: AdamW with global-norm
    clipping over all 887.7M parameters (32 B / parameter: the norm reads g;
    the update reads p, g, m, v and writes p, m, v), the embedding gather and
    scatter-add (8 B per row element each way) and the residual add (12 B /
    element)."""
    hbm, _, src = peaks()
    sizes = llama1b_param_shapes()
    n = sum(sizes)
    flat = [torch.empty(n, device="cuda") for _ in range(4)]
    for t in flat:
        t.uniform_(-0.01, 0.01)
    flat[3].abs_()

    def views(buf):
        out, off = [], 0
        for k in sizes:
            out.append(buf[off:off + k])
            off += k
        return out
    P, G, M, V = (views(b) for b in flat)
    step = [0]

    def adamw_clip():
        step[0] += 1
        acc = K.sumsq(G)
        K.adamw(P, G, M, V, 3e-4, 0.9, 0.95, 1e-8, 0.1, step[0], sumsq_acc=acc, max_norm=1.0)
    ms = timed(adamw_clip, iters)
    emit({"op": "adamw_clip", "params": n, "tensors": len(sizes), "ms": ms,
          "gbs": 32 * n / ms / 1e6, "frac_hbm": 32 * n / ms / 1e6 / hbm, "peak_src": src})
    del P, G, M, V, flat
    R, D, Vv = 16384, 2048, 32000
    W = torch.randn(Vv, D, device="cuda")
    idx = torch.randint(0, Vv, (R,), device="cuda", dtype=torch.int64)
    ms = timed(lambda: K.embedding_fwd(W, idx), iters)
    emit({"op": "embedding", "pass": "fwd", "rows": R, "d": D, "ms": ms,
          "gbs": 8 * R * D / ms / 1e6, "frac_hbm": 8 * R * D / ms / 1e6 / hbm})
    dout = torch.randn(R, D, device="cuda")
    dW = torch.zeros_like(W)
    ms = timed(lambda: K.embedding_bwd(dout, idx, dW), iters)
    emit({"op": "embedding", "pass": "bwd (sort + segmented sum)", "rows": R, "d": D, "ms": ms,
          "gbs": 8 * R * D / ms / 1e6, "frac_hbm": 8 * R * D / ms / 1e6 / hbm})
    a, b = torch.randn(R, D, device="cuda"), torch.randn(R, D, device="cuda")
    out = torch.empty_like(a)
    shape = _ttk.i64_array([R, D])
    st = _ttk.i64_array([D, 1])

    def add():
        _ttk.call("ttk_binary", 0, a.data_ptr(), st, b.data_ptr(), st, out.data_ptr(), shape, 2,
                  torch.cuda.current_stream().cuda_stream)
    ms = timed(add, iters)
    emit({"op": "residual_add", "rows": R, "d": D, "ms": ms,
          "gbs": 12 * R * D / ms / 1e6, "frac_hbm": 12 * R * D / ms / 1e6 / hbm})


def bench_attention(seqs, iters, B=8, H=12, hd=64):
    """Forward + backward; fwd FLOPs 2*B*H*S^2*hd (causal half of 4*B*H*S^2*hd),
    backward counted as 2x forward (dQ, dK, dV; recomputation not credited)."""
    _, bf16, src = peaks()
    for S in seqs:
        q, k, v, do = (torch.randn(B, S, H, hd, device="cuda") for _ in range(4))
        cs, sn = K.rope_tables(S, hd, 10000.0, "cuda")
        o, lse = K.attention_fwd(q, k, v, cs, sn)
        ms_f = timed(lambda: K.attention_fwd(q, k, v, cs, sn), iters)
        ms_b = timed(lambda: K.attention_bwd(q, k, v, cs, sn, o, lse, do), iters)
        fl_f = 2 * B * H * S * S * hd  # causal half of 4*B*H*S^2*hd
        fl_b = 2 * fl_f
        eng = {0: "tcgen05 fwd + bwd, bf16x3 split",
               2: "mma.sync m16n8k16 bf16x3 split"}[_ttk.call("ttk_attention_get_impl")]
        emit({"op": "attention", "B": B, "H": H, "hd": hd, "S": S, "ms_fwd": ms_f,
              "ms_bwd": ms_b, "tflops_fwd": fl_f / ms_f / 1e9, "tflops_bwd": fl_b / ms_b / 1e9,
              "tflops_fwd_bwd": (fl_f + fl_b) / (ms_f + ms_b) / 1e9, "engine": eng})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", choices=["gemm", "rows", "ce", "hbm", "attention"], default=None)
    ap.add_argument("--shape", default=None, help="M,K,N for --only gemm")
    ap.add_argument("--rows", type=int, default=None)
    ap.add_argument("--dims", default=None,
                    help="R,D,F: one row shape for --only rows (e.g. a capture-sized case)")
    ap.add_argument("--ops", default="rmsnorm,swiglu,ce",
                    help="row kernels for --only rows: any of rmsnorm, swiglu, ce")
    ap.add_argument("--seq", type=int, default=None)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--hd", type=int, default=64)
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--heads", type=int, default=None)
    a = ap.parse_args()
    torch.cuda.set_device(0)
    _ttk.call("ttk_init", 0)
    shapes = [tuple(int(x) for x in a.shape.split(","))] if a.shape else GEMM_SHAPES
    rows = [r for r in ROWS if a.rows is None or r[0] == a.rows] or ROWS
    if a.dims:
        rows = [tuple(int(x) for x in a.dims.split(","))]
    if a.only in (None, "gemm"):
        bench_gemm(shapes, a.iters)
    if a.only in (None, "rows", "ce"):
        ops = ("ce",) if a.only == "ce" else tuple(a.ops.split(","))
        bench_rows(rows, a.iters, ops)
    if a.only in (None, "hbm"):
        bench_hbm(a.iters)
    if a.only in (None, "attention"):
        B0, H0 = {64: (8, 12), 128: (8, 16), 32: (16, 8)}.get(a.hd, (8, 2048 // a.hd))
        bench_attention([a.seq] if a.seq else ATTN_S, a.iters, B=a.batch or B0,
                        H=a.heads or H0, hd=a.hd)
    assert _ttk.device_status() == 0


if __name__ == "__main__":
    main()
