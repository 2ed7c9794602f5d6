"""numpy restatement of the tinytrain reference's training hot path.

TEST INFRASTRUCTURE ONLY (imported by tests/ and the smoke check, never by
the product). Each function restates one reference algorithm, citing the
file:line of seampm/tinytrain it follows, in float32 with float64 where the
reference accumulates in double. It is pinned against the reference itself:
tests/test_oracle.py compares it with oracle/_ref/libttref.so (the reference
sources compiled unchanged) and with the fixtures in tests/golden/ that the
reference produced.

Gradient clipping is not in the reference (no clip symbol exists in its
sources); clip_grad_norm below restates the conventional global-norm rule and
is marked as such.
"""
from __future__ import annotations

import numpy as np

f32 = np.float32


def matmul(A, B):
    """ops.cpp:96-125 sgemm / :661-697 matmul: C = A @ B (float32)."""
    return (A.astype(np.float64) @ B.astype(np.float64)).astype(f32)


def matmul_bwd(A, B, G):
    """ops.cpp:672-694: dA = G @ B^T, dB = A^T @ G."""
    A64, B64, G64 = A.astype(np.float64), B.astype(np.float64), G.astype(np.float64)
    return (G64 @ B64.T).astype(f32), (A64.T @ G64).astype(f32)


def rmsnorm(x, w, eps):
    """ops.cpp:932-942: r = (sum(x^2,-1)/D + eps)^-1/2 ; y = x*r*w.
    Returns (y, r) with r per row."""
    D = x.shape[-1]
    ms = (x.astype(f32) * x).sum(-1, keepdims=True, dtype=f32) / f32(D)
    r = (ms + f32(eps)) ** f32(-0.5)
    return (x * r * w).astype(f32), r.astype(f32)


def rmsnorm_bwd(x, w, r, g):
    """Backward of the composite rmsnorm (ops.cpp:934-941 chain):
    dw = sum_rows(g*x*r); dx = r*g*w - x*r^3/D * sum(g*w*x, -1)."""
    D = x.shape[-1]
    x64, w64, r64, g64 = (a.astype(np.float64) for a in (x, w, r, g))
    gw = g64 * w64
    dot = (gw * x64).sum(-1, keepdims=True)
    dx = r64 * gw - x64 * (r64 ** 3) / D * dot
    dw = (g64 * x64 * r64).reshape(-1, D).sum(0)
    return dx.astype(f32), dw.astype(f32)


def silu(a):
    """ops.cpp:324: x / (1 + exp(-x))."""
    return (a / (f32(1) + np.exp(-a, dtype=f32))).astype(f32)


def swiglu(a, b):
    """model.cpp:149-151: y = silu(a) * b."""
    return (silu(a) * b).astype(f32)


def swiglu_bwd(a, b, g):
    """ops.cpp:325-328 b_silu and ops.cpp:256 bwd_mul:
    da = g*b*s*(1+a*(1-s)), db = g*silu(a)."""
    s = f32(1) / (f32(1) + np.exp(-a, dtype=f32))
    da = g * b * (s * (f32(1) + a * (f32(1) - s)))
    db = g * (a * s)
    return da.astype(f32), db.astype(f32)


def softmax(x):
    """ops.cpp:777-815: max-subtracted exp, double sum, scale by 1/sum."""
    m = x.max(-1, keepdims=True)
    e = np.exp((x - m).astype(f32), dtype=f32)
    s = e.astype(np.float64).sum(-1, keepdims=True)
    return (e * (1.0 / s).astype(f32)).astype(f32)


def softmax_bwd(y, g):
    """ops.cpp:816-838: dx = y * (g - sum(g*y))."""
    dot = (g.astype(np.float64) * y).sum(-1, keepdims=True).astype(f32)
    return (y * (g - dot)).astype(f32)


def log_softmax(x):
    """ops.cpp:840-868: x - (max + log(sum exp(x - max))), sum in double."""
    m = x.max(-1, keepdims=True)
    s = np.exp((x - m).astype(f32), dtype=f32).astype(np.float64).sum(-1, keepdims=True)
    lse = m + np.log(s).astype(f32)
    return (x - lse).astype(f32), lse.astype(f32)


def cross_entropy(logits, targets):
    """ops.cpp:898-930: loss = mean_i(-log_softmax(x)[i, t_i]) (double acc);
    dlogits = (softmax - onehot) / N for d(loss)=1 (ops.cpp:869-893, :918-923)."""
    N = logits.shape[0]
    lp, _ = log_softmax(logits)
    loss = -lp[np.arange(N), targets].astype(np.float64).sum() / N
    d = np.exp(lp, dtype=f32)
    d[np.arange(N), targets] -= f32(1)
    return f32(loss), (d / f32(N)).astype(f32)


def embedding(W, idx):
    """ops.cpp:746-759: out[i] = W[idx[i]]."""
    return W[idx].astype(f32)


def embedding_bwd(shape, idx, g):
    """ops.cpp:761-772: dW[idx[i]] += g[i], i ascending (float32 adds)."""
    dW = np.zeros(shape, f32)
    for i, t in enumerate(idx):
        dW[t] += g[i]
    return dW


def rope_tables(T, hd, theta):
    """model.cpp:43-53: angle = pos * (1 / theta^(2i/hd)) in float32."""
    i = np.arange(hd // 2, dtype=f32)
    inv = f32(1) / np.power(f32(theta), (f32(2) * i) / f32(hd), dtype=f32)
    ang = np.arange(T, dtype=f32)[:, None] * inv[None, :]
    return np.cos(ang).astype(f32), np.sin(ang).astype(f32)


def rope(x, cos, sin):
    """ops.cpp:970-999: half-split rotation on x [B,T,H,D]."""
    Dh = x.shape[-1] // 2
    x1, x2 = x[..., :Dh], x[..., Dh:]
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    return np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], -1).astype(f32)


def rope_bwd(g, cos, sin):
    """ops.cpp:1011-1023: the transpose rotation."""
    Dh = g.shape[-1] // 2
    g1, g2 = g[..., :Dh], g[..., Dh:]
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    return np.concatenate([g1 * c + g2 * s, -g1 * s + g2 * c], -1).astype(f32)


def attention(q, k, v, theta):
    """model.cpp:127-141 on q,k,v [B,T,H,hd] (pre-RoPE) -> [B,T,H*hd].
    Returns (out, cache) for attention_bwd."""
    B, T, H, hd = q.shape
    cos, sin = rope_tables(T, hd, theta)
    qr, kr = rope(q, cos, sin), rope(k, cos, sin)
    scale = f32(1.0 / np.sqrt(np.float32(hd)))
    qb = qr.transpose(0, 2, 1, 3).astype(np.float64)
    kb = kr.transpose(0, 2, 1, 3).astype(np.float64)
    vb = v.transpose(0, 2, 1, 3).astype(np.float64)
    s = (qb @ kb.transpose(0, 1, 3, 2)).astype(f32) * scale
    mask = np.triu(np.full((T, T), -1e9, f32), 1)
    p = softmax((s + mask).astype(f32))
    o = (p.astype(np.float64) @ vb).astype(f32)
    out = o.transpose(0, 2, 1, 3).reshape(B, T, H * hd)
    return out, (qb, kb, vb, p, cos, sin, scale)


def attention_bwd(g, cache):
    qb, kb, vb, p, cos, sin, scale = cache
    B, H, T, hd = qb.shape
    go = g.reshape(B, T, H, hd).transpose(0, 2, 1, 3).astype(np.float64)
    dv = p.astype(np.float64).transpose(0, 1, 3, 2) @ go
    dp = (go @ vb.transpose(0, 1, 3, 2)).astype(f32)
    ds = softmax_bwd(p, dp).astype(np.float64) * scale
    dq = ds @ kb
    dk = ds.transpose(0, 1, 3, 2) @ qb
    to_bthd = lambda a: a.transpose(0, 2, 1, 3).astype(f32)
    return (rope_bwd(to_bthd(dq), cos, sin), rope_bwd(to_bthd(dk), cos, sin), to_bthd(dv))


def adamw_step(p, g, m, v, step, lr, b1, b2, eps, wd):
    """optim.cpp:17-48, one step in place: decoupled decay with lr (before
    the moments), bias correction folded into lr_t, eps added to sqrt(v)."""
    bc1 = f32(1) - np.power(f32(b1), f32(step), dtype=f32)
    bc2 = f32(1) - np.power(f32(b2), f32(step), dtype=f32)
    lr_t = f32(lr) * np.sqrt(bc2, dtype=f32) / bc1
    p -= f32(lr) * f32(wd) * p
    m[:] = f32(b1) * m + (f32(1) - f32(b1)) * g
    v[:] = f32(b2) * v + (f32(1) - f32(b2)) * g * g
    p -= lr_t * m / (np.sqrt(v, dtype=f32) + f32(eps))


def clip_grad_norm(grads, max_norm):
    """Not in the reference: global-norm clipping restated from the
    conventional rule (torch.nn.utils.clip_grad_norm_):
    total = ||g||_2 over all grads (double), coef = max_norm/(total+1e-6),
    grads *= coef if coef < 1. Returns total."""
    ss = sum(float((g.astype(np.float64) ** 2).sum()) for g in grads)
    total = np.sqrt(ss)
    coef = f32(max_norm / (total + 1e-6))
    if max_norm > 0 and coef < 1:
        for g in grads:
            g *= coef
    return total


_M64 = (1 << 64) - 1


def xorshift_stream(seed, n):
    """n outputs of the xorshift64* generator shared by tensor.cpp's Rng, the
    dropout mask (ops.cpp:949-963) and apps/train.cpp:145-153 (seed 0 ->
    0x9E3779B97F4A7C15). Pure Python: small n only."""
    s = seed if seed else 0x9E3779B97F4A7C15
    out = []
    for _ in range(n):
        s ^= s >> 12
        s ^= (s << 25) & _M64
        s ^= s >> 27
        out.append((s * 0x2545F4914F6CDD1D) & _M64)
    return out


def dropout_mask(n, p, seed):
    """ops.cpp:949-963: element i kept when ((r_i >> 11) * 2^-53) >= p."""
    r = xorshift_stream(seed, n)
    return np.array([1.0 if (x >> 11) * (1.0 / 9007199254740992.0) >= float(np.float32(p)) else 0.0
                     for x in r], np.float32)


def sample_windows(seed, ntok, T, count):
    """apps/train.cpp:225-232: `count` window starts rng.next() % (ntok - T - 1)
    from Rng(seed); returns (starts, next seed state is not exposed)."""
    return [x % (ntok - T - 1) for x in xorshift_stream(seed, count)]


def lr_scale(gstep, warmup, total_steps):
    """apps/train.cpp:214-222: linear warmup then cosine to 10% of peak."""
    if gstep < warmup:
        return f32(gstep + 1) / f32(warmup)
    prog = f32(gstep - warmup) / f32(max(total_steps - warmup, 1))
    return f32(0.1) + f32(0.9) * f32(0.5) * (f32(1) + np.cos(f32(3.14159265) * prog, dtype=f32))


# ---------------------------------------------------------------------------
# Whole model (model.cpp:87-160) with its backward, on the flat parameter list
# in GPTModel::parameters() order (model.cpp:56-85).
# ---------------------------------------------------------------------------

def param_shapes(vocab, dim, layers, heads, ffn):
    shapes = [(vocab, dim)]
    for _ in range(layers):
        shapes += [(dim,), (dim, dim), (dim, dim), (dim, dim), (dim, dim), (dim,),
                   (ffn, dim), (ffn, dim), (dim, ffn)]
    shapes.append((dim,))
    return shapes


def split_params(flat, shapes):
    out, off = [], 0
    for s in shapes:
        n = int(np.prod(s))
        out.append(flat[off:off + n].reshape(s))
        off += n
    return out


def model_fwd_bwd(flat, idx, targets, B, T, vocab, dim, layers, heads, ffn, eps=1e-5,
                  theta=10000.0):
    """Forward (model.cpp:87-160) + cross-entropy + full backward.
    Returns (loss, logits, flat_grads)."""
    shapes = param_shapes(vocab, dim, layers, heads, ffn)
    P = split_params(np.asarray(flat, f32), shapes)
    G = [np.zeros(s, f32) for s in shapes]
    hd = dim // heads
    R = B * T
    E = P[0]
    x = embedding(E, idx)
    caches = []
    for l in range(layers):
        base = 1 + 9 * l
        w_an, wq, wk, wv, wo, w_fn, wg, wu, wd = P[base:base + 9]
        h, r1 = rmsnorm(x, w_an, eps)
        q, k, v = matmul(h, wq.T), matmul(h, wk.T), matmul(h, wv.T)
        att, acache = attention(q.reshape(B, T, heads, hd), k.reshape(B, T, heads, hd),
                                v.reshape(B, T, heads, hd), theta)
        att = att.reshape(R, dim)
        x1 = (x + matmul(att, wo.T)).astype(f32)
        h2, r2 = rmsnorm(x1, w_fn, eps)
        a, u = matmul(h2, wg.T), matmul(h2, wu.T)
        act = swiglu(a, u)
        x2 = (x1 + matmul(act, wd.T)).astype(f32)
        caches.append((x, h, r1, acache, att, x1, h2, r2, a, u, act))
        x = x2
    hn, rf = rmsnorm(x, P[-1], eps)
    logits = matmul(hn, E.T)
    loss, dlog = cross_entropy(logits, targets)
    # backward
    dhn, dE_head = matmul_bwd(hn, E.T, dlog)
    G[0] += dE_head.T
    dx, dwf = rmsnorm_bwd(x, P[-1], rf, dhn)
    G[-1] += dwf
    for l in reversed(range(layers)):
        base = 1 + 9 * l
        w_an, wq, wk, wv, wo, w_fn, wg, wu, wd = P[base:base + 9]
        xin, h, r1, acache, att, x1, h2, r2, a, u, act = caches[l]
        dact, dwdT = matmul_bwd(act, wd.T, dx)
        G[base + 8] += dwdT.T
        da, du = swiglu_bwd(a, u, dact)
        dh2a, dwgT = matmul_bwd(h2, wg.T, da)
        dh2u, dwuT = matmul_bwd(h2, wu.T, du)
        G[base + 6] += dwgT.T
        G[base + 7] += dwuT.T
        dx1_n, dwfn = rmsnorm_bwd(x1, w_fn, r2, (dh2a + dh2u).astype(f32))
        G[base + 5] += dwfn
        dx1 = (dx + dx1_n).astype(f32)
        datt, dwoT = matmul_bwd(att, wo.T, dx1)
        G[base + 4] += dwoT.T
        dq, dk, dv = attention_bwd(datt.reshape(B, T, heads * hd), acache)
        dhq, dwqT = matmul_bwd(h, wq.T, dq.reshape(R, dim))
        dhk, dwkT = matmul_bwd(h, wk.T, dk.reshape(R, dim))
        dhv, dwvT = matmul_bwd(h, wv.T, dv.reshape(R, dim))
        G[base + 1] += dwqT.T
        G[base + 2] += dwkT.T
        G[base + 3] += dwvT.T
        dxn, dwan = rmsnorm_bwd(xin, w_an, r1, (dhq + dhk + dhv).astype(f32))
        G[base] += dwan
        dx = (dx1 + dxn).astype(f32)
    G[0] += embedding_bwd(E.shape, idx, dx)
    return loss, logits, np.concatenate([g.ravel() for g in G]).astype(f32)
