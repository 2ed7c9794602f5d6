"""ctypes binding of oracle/_ref/libttref.so (the reference's own CPU library).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the product package. Each function
takes numpy arrays, runs the reference op chain named in its docstring, and
returns numpy results. See oracle/ref_harness.cpp for the op chains.
"""
from __future__ import annotations

import contextlib
import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libttref.so")
# The same harness with the reference's src/model.cpp, compiled against this
# repository's headers and library (the drop-in on the device).
LIB_B200_PATH = os.path.join(_HERE, "_ref", "libttref_b200.so")
_libs = {}
_active = LIB_PATH


class RefCfg(C.Structure):
    _fields_ = [("vocab", C.c_int64), ("dim", C.c_int64), ("layers", C.c_int64),
                ("heads", C.c_int64), ("ffn", C.c_int64), ("max_seq", C.c_int64),
                ("norm_eps", C.c_float), ("rope_theta", C.c_float)]


def available(path=None) -> bool:
    return os.path.exists(path or LIB_PATH)


def lib():
    path = _active
    if path not in _libs:
        if not available(path):
            raise FileNotFoundError(
                f"{path} missing: build it with `make -C oracle` where the reference sources exist")
        L = C.CDLL(path)
        L.ref_last_error.restype = C.c_char_p
        L.ref_param_count.restype = C.c_int64
        L.ref_param_shapes.restype = C.c_int64
        _libs[path] = L
    return _libs[path]


@contextlib.contextmanager
def on_device():
    """Inside the block every function of this module runs the harness built
    against this repository's library (oracle/_ref/libttref_b200.so): the
    reference's own model.cpp and op chains, unmodified, executing on the
    device. Not for the oracle's role: its results are what gets checked."""
    global _active
    prev, _active = _active, LIB_B200_PATH
    try:
        yield
    finally:
        _active = prev


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i(a):
    return np.ascontiguousarray(a, dtype=np.int64)


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _check(rc):
    if rc != 0:
        raise ValueError(lib().ref_last_error().decode())


def cfg(vocab=32000, dim=256, layers=6, heads=8, ffn=768, max_seq=256, norm_eps=1e-5,
        rope_theta=10000.0) -> RefCfg:
    return RefCfg(vocab, dim, layers, heads, ffn, max_seq, norm_eps, rope_theta)


def matmul(A, B, G=None):
    A, B = _f(A), _f(B)
    M, K = A.shape
    N = B.shape[1]
    Cm = np.empty((M, N), np.float32)
    dA = np.empty_like(A) if G is not None else None
    dB = np.empty_like(B) if G is not None else None
    G = None if G is None else _f(G)
    _check(lib().ref_matmul(C.c_int64(M), C.c_int64(K), C.c_int64(N), _p(A), _p(B), _p(G),
                            _p(Cm), _p(dA), _p(dB)))
    return (Cm, dA, dB) if G is not None else Cm


def linear(X, W, G=None):
    X, W = _f(X), _f(W)
    R, n_in = X.shape
    n_out = W.shape[0]
    Y = np.empty((R, n_out), np.float32)
    dX = np.empty_like(X) if G is not None else None
    dW = np.empty_like(W) if G is not None else None
    G = None if G is None else _f(G)
    _check(lib().ref_linear(C.c_int64(R), C.c_int64(n_in), C.c_int64(n_out), _p(X), _p(W),
                            _p(G), _p(Y), _p(dX), _p(dW)))
    return (Y, dX, dW) if G is not None else Y


def bmm(A, B, G=None):
    A, B = _f(A), _f(B)
    Bt, M, K = A.shape
    N = B.shape[2]
    Cm = np.empty((Bt, M, N), np.float32)
    dA = np.empty_like(A) if G is not None else None
    dB = np.empty_like(B) if G is not None else None
    G = None if G is None else _f(G)
    _check(lib().ref_bmm(C.c_int64(Bt), C.c_int64(M), C.c_int64(K), C.c_int64(N), _p(A), _p(B),
                         _p(G), _p(Cm), _p(dA), _p(dB)))
    return (Cm, dA, dB) if G is not None else Cm


def rmsnorm(X, W, eps, G=None):
    X, W = _f(X), _f(W)
    R, D = X.shape
    Y = np.empty_like(X)
    dX = np.empty_like(X) if G is not None else None
    dW = np.empty_like(W) if G is not None else None
    G = None if G is None else _f(G)
    _check(lib().ref_rmsnorm(C.c_int64(R), C.c_int64(D), _p(X), _p(W), C.c_float(eps), _p(G),
                             _p(Y), _p(dX), _p(dW)))
    return (Y, dX, dW) if G is not None else Y


def swiglu(A, Bm, G=None):
    A, Bm = _f(A), _f(Bm)
    R, F = A.shape
    Y = np.empty_like(A)
    dA = np.empty_like(A) if G is not None else None
    dB = np.empty_like(A) if G is not None else None
    G = None if G is None else _f(G)
    _check(lib().ref_swiglu(C.c_int64(R), C.c_int64(F), _p(A), _p(Bm), _p(G), _p(Y), _p(dA),
                            _p(dB)))
    return (Y, dA, dB) if G is not None else Y


def cross_entropy(logits, targets, grad=True):
    logits, targets = _f(logits), _i(targets)
    N, Cn = logits.shape
    loss = C.c_float(0)
    dl = np.empty_like(logits) if grad else None
    _check(lib().ref_cross_entropy(C.c_int64(N), C.c_int64(Cn), _p(logits), _p(targets),
                                   C.byref(loss), _p(dl)))
    return (loss.value, dl) if grad else loss.value


def embedding(W, idx, G=None):
    W, idx = _f(W), _i(idx)
    V, D = W.shape
    N = idx.shape[0]
    out = np.empty((N, D), np.float32)
    dW = np.empty_like(W) if G is not None else None
    G = None if G is None else _f(G)
    _check(lib().ref_embedding(C.c_int64(V), C.c_int64(D), _p(W), C.c_int64(N), _p(idx), _p(G),
                               _p(out), _p(dW)))
    return (out, dW) if G is not None else out


def rope(X, cos, sin, G=None):
    X, cos, sin = _f(X), _f(cos), _f(sin)
    B, T, H, D = X.shape
    Y = np.empty_like(X)
    dX = np.empty_like(X) if G is not None else None
    G = None if G is None else _f(G)
    _check(lib().ref_rope(C.c_int64(B), C.c_int64(T), C.c_int64(H), C.c_int64(D), _p(X),
                          _p(cos), _p(sin), _p(G), _p(Y), _p(dX)))
    return (Y, dX) if G is not None else Y


def dropout_mask(n, p, seed):
    """Mask of the reference's dropout (ops.cpp:944-968) for n elements."""
    m = np.empty(n, np.float32)
    _check(lib().ref_dropout_mask(C.c_int64(n), C.c_float(p), C.c_uint64(seed), _p(m)))
    return m


def softmax(X, G=None):
    X = _f(X)
    R, Cn = X.shape
    Y = np.empty_like(X)
    dX = np.empty_like(X) if G is not None else None
    G = None if G is None else _f(G)
    _check(lib().ref_softmax(C.c_int64(R), C.c_int64(Cn), _p(X), _p(G), _p(Y), _p(dX)))
    return (Y, dX) if G is not None else Y


def attention(Q, K, V, theta=10000.0, G=None):
    """model.cpp:127-141 on q/k/v [B,T,H,hd] (pre-RoPE); out [B,T,H*hd]."""
    Q, K, V = _f(Q), _f(K), _f(V)
    B, T, H, hd = Q.shape
    O = np.empty((B, T, H * hd), np.float32)
    dQ = np.empty_like(Q) if G is not None else None
    dK = np.empty_like(K) if G is not None else None
    dV = np.empty_like(V) if G is not None else None
    G = None if G is None else _f(G)
    _check(lib().ref_attention(C.c_int64(B), C.c_int64(T), C.c_int64(H), C.c_int64(hd),
                               C.c_float(theta), _p(Q), _p(K), _p(V), _p(G), _p(O), _p(dQ),
                               _p(dK), _p(dV)))
    return (O, dQ, dK, dV) if G is not None else O


def adamw(p, grads, lr, b1, b2, eps, wd):
    """len(grads) steps of the reference AdamW on one flat parameter."""
    p = _f(p).copy()
    grads = _f(grads)
    K, n = grads.shape
    _check(lib().ref_adamw(C.c_int64(n), _p(p), _p(grads), C.c_int64(K), C.c_float(lr),
                           C.c_float(b1), C.c_float(b2), C.c_float(eps), C.c_float(wd)))
    return p


def param_count(c: RefCfg) -> int:
    return int(lib().ref_param_count(C.byref(c)))


def param_shapes(c: RefCfg):
    cap = 4096
    buf = np.zeros(2 * cap, np.int64)
    n = lib().ref_param_shapes(C.byref(c), _p(buf), C.c_int64(cap))
    if n < 0:
        raise ValueError(lib().ref_last_error().decode())
    out = []
    for i in range(n):
        r, c2 = int(buf[2 * i]), int(buf[2 * i + 1])
        out.append((r,) if c2 == 0 else (r, c2))
    return out


def init_params(c: RefCfg, seed: int):
    out = np.empty(param_count(c), np.float32)
    _check(lib().ref_init_params(C.byref(c), C.c_uint64(seed), _p(out)))
    return out


def load_checkpoint(c: RefCfg, path: str):
    """Flat parameters after the reference's GPTModel::load_checkpoint(path)."""
    out = np.empty(param_count(c), np.float32)
    _check(lib().ref_load_checkpoint(C.byref(c), os.fsencode(path), _p(out)))
    return out


def model_fwd_bwd(c: RefCfg, params, idx, targets, B, T, want_grads=True):
    params, idx = _f(params), _i(idx)
    logits = np.empty((B * T, c.vocab), np.float32)
    loss = C.c_float(0)
    grads = np.empty_like(params) if want_grads else None
    tg = None if targets is None else _i(targets)
    _check(lib().ref_model_fwd_bwd(C.byref(c), _p(params), _p(idx), _p(tg), C.c_int64(B),
                                   C.c_int64(T), _p(logits), C.byref(loss), _p(grads)))
    return logits, loss.value, grads


def train(c: RefCfg, params, idx, targets, B, T, lrs, b1=0.9, b2=0.95, eps=1e-8, wd=0.1,
          clip=1.0):
    """apps/train.cpp:212-256 loop on fixed batches; returns (losses, norms, params)."""
    params = _f(params).copy()
    idx, targets = _i(idx), _i(targets)
    lrs = _f(lrs)
    steps = lrs.shape[0]
    losses = np.empty(steps, np.float32)
    norms = np.empty(steps, np.float32)
    _check(lib().ref_train(C.byref(c), _p(params), _p(idx), _p(targets), C.c_int64(B),
                           C.c_int64(T), C.c_int64(steps), _p(lrs), C.c_float(b1), C.c_float(b2),
                           C.c_float(eps), C.c_float(wd), C.c_float(clip), _p(losses),
                           _p(norms)))
    return losses, norms, params


def time_train(c: RefCfg, B, T, warmup, steps, seed=42) -> float:
    """Mean seconds per reference training step (forward+CE+backward+clip+AdamW)."""
    secs = C.c_double(0)
    _check(lib().ref_time_train(C.byref(c), C.c_int64(B), C.c_int64(T), C.c_int64(warmup),
                                C.c_int64(steps), C.c_uint64(seed), C.byref(secs)))
    return secs.value


def time_phases(c: RefCfg, B, T, warmup, steps, seed=42):
    """(mean seconds of forward+CE+backward per B x T micro-step, seconds of
    one clip + AdamW step) of the reference on random tokens."""
    fb, op = C.c_double(0), C.c_double(0)
    _check(lib().ref_time_phases(C.byref(c), C.c_int64(B), C.c_int64(T), C.c_int64(warmup),
                                 C.c_int64(steps), C.c_uint64(seed), C.byref(fb), C.byref(op)))
    return fb.value, op.value
