"""Seeded synthetic inputs shared by the fixture generator and the tests.

Weights: every matrix (embedding and Linear weights) ~ N(0, 0.02), every
RMSNorm weight = 1, in GPTModel::parameters() order. Tokens: uniform in
[0, vocab); each sequence is a window of T+1 tokens, idx = window[:T],
targets = window[1:] (next-token prediction, as apps/train.cpp:225-232).
No dataset is involved: these stand in for the reference's TinyStories run.
"""
from __future__ import annotations

import numpy as np


def param_shapes(vocab, dim, layers, heads, ffn):
    shapes = [(vocab, dim)]
    for _ in range(layers):
        shapes += [(dim,), (dim, dim), (dim, dim), (dim, dim), (dim, dim), (dim,),
                   (ffn, dim), (ffn, dim), (dim, ffn)]
    shapes.append((dim,))
    return shapes


def make_weights(shapes, seed, std=0.02):
    rng = np.random.default_rng(seed)
    parts = []
    for s in shapes:
        if len(s) == 1:
            parts.append(np.ones(s, np.float32))
        else:
            parts.append((rng.standard_normal(s, dtype=np.float32) * np.float32(std)))
    return np.concatenate([p.ravel() for p in parts]).astype(np.float32)


def make_tokens(steps, B, T, vocab, seed):
    rng = np.random.default_rng(seed)
    w = rng.integers(0, vocab, size=(steps, B, T + 1), dtype=np.int64)
    idx = w[:, :, :T].reshape(steps, B * T)
    tgt = w[:, :, 1:].reshape(steps, B * T)
    return np.ascontiguousarray(idx), np.ascontiguousarray(tgt)


def checksum(a):
    return float(np.asarray(a, np.float64).sum())
