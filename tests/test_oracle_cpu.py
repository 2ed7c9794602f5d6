"""The oracle pinned: the numpy restatement (oracle/restate.py) against the
fixtures the reference's own CPU library produced (tests/golden/), and, where
the compiled reference (oracle/_ref) is present, against the reference
directly. Runs on CPU."""
import numpy as np
import pytest

from conftest import GOLDEN, rel_err
from oracle import restate as rs

TOL = 1e-5  # restatement vs reference: same fp32 arithmetic up to summation order


def test_matmul(golden_ops):
    g = golden_ops
    for tag in "abcd":
        A, B, G = g[f"mm_{tag}_A"], g[f"mm_{tag}_B"], g[f"mm_{tag}_G"]
        assert rel_err(rs.matmul(A, B), g[f"mm_{tag}_C"]) < TOL
        dA, dB = rs.matmul_bwd(A, B, G)
        assert rel_err(dA, g[f"mm_{tag}_dA"]) < TOL
        assert rel_err(dB, g[f"mm_{tag}_dB"]) < TOL


def test_rmsnorm(golden_ops):
    g = golden_ops
    y, r = rs.rmsnorm(g["rms_X"], g["rms_W"], 1e-5)
    dx, dw = rs.rmsnorm_bwd(g["rms_X"], g["rms_W"], r, g["rms_G"])
    assert rel_err(y, g["rms_Y"]) < TOL
    assert rel_err(dx, g["rms_dX"]) < TOL
    assert rel_err(dw, g["rms_dW"]) < TOL


def test_swiglu(golden_ops):
    g = golden_ops
    assert rel_err(rs.swiglu(g["swi_A"], g["swi_B"]), g["swi_Y"]) < TOL
    da, db = rs.swiglu_bwd(g["swi_A"], g["swi_B"], g["swi_G"])
    assert rel_err(da, g["swi_dA"]) < TOL
    assert rel_err(db, g["swi_dB"]) < TOL


def test_softmax(golden_ops):
    g = golden_ops
    y = rs.softmax(g["sm_X"])
    assert rel_err(y, g["sm_Y"]) < TOL
    assert rel_err(rs.softmax_bwd(y, g["sm_G"]), g["sm_dX"]) < TOL


def test_cross_entropy(golden_ops):
    g = golden_ops
    loss, d = rs.cross_entropy(g["ce_L"], g["ce_t"])
    assert abs(loss - g["ce_loss"]) <= 1e-6 * abs(g["ce_loss"])
    assert rel_err(d, g["ce_dL"]) < TOL


def test_embedding_bitexact(golden_ops):
    g = golden_ops
    assert np.array_equal(rs.embedding(g["emb_W"], g["emb_idx"]), g["emb_out"])
    assert np.array_equal(rs.embedding_bwd(g["emb_W"].shape, g["emb_idx"], g["emb_G"]), g["emb_dW"])


def test_rope(golden_ops):
    g = golden_ops
    assert rel_err(rs.rope(g["rope_X"], g["rope_cos"], g["rope_sin"]), g["rope_Y"]) < TOL
    assert rel_err(rs.rope_bwd(g["rope_G"], g["rope_cos"], g["rope_sin"]), g["rope_dX"]) < TOL


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_attention(golden_ops, tag):
    g = golden_ops
    q, k, v, G = (g[f"att_{tag}_{s}"] for s in ("q", "k", "v", "G"))
    o, cache = rs.attention(q, k, v, 10000.0)
    assert rel_err(o, g[f"att_{tag}_O"]) < TOL
    for got, ref in zip(rs.attention_bwd(G, cache), ("dq", "dk", "dv")):
        assert rel_err(got, g[f"att_{tag}_{ref}"]) < TOL


def test_adamw(golden_ops):
    g = golden_ops
    p = g["adam_p"].copy()
    m, v = np.zeros_like(p), np.zeros_like(p)
    for s in range(g["adam_g"].shape[0]):
        rs.adamw_step(p, g["adam_g"][s], m, v, s + 1, 1e-2, 0.9, 0.95, 1e-8, 0.1)
    assert rel_err(p, g["adam_out"]) < 1e-6


def test_model_tiny_fwd_bwd():
    d = dict(np.load(f"{GOLDEN}/model_tiny.npz"))
    v, dim, L, H, F, _ = (int(x) for x in d["cfg"])
    loss, logits, grads = rs.model_fwd_bwd(d["weights"], d["idx"][0], d["tgt"][0], 2, 16, v, dim,
                                           L, H, F)
    assert abs(loss - d["loss"]) <= 1e-5 * abs(d["loss"])
    assert rel_err(logits, d["logits"]) < TOL
    assert rel_err(grads, d["grads"]) < 1e-5


def test_lr_schedule():
    """apps/train.cpp:214-222: linear warmup then cosine to 10%."""
    assert rs.lr_scale(0, 100, 1000) == np.float32(0.01)
    assert rs.lr_scale(99, 100, 1000) == np.float32(1.0)
    assert abs(rs.lr_scale(100, 100, 1000) - 1.0) < 1e-6
    assert abs(rs.lr_scale(1000, 100, 1000) - 0.1) < 1e-6


@pytest.mark.parametrize("n,p,seed", [(1, 0.5, 0), (97, 0.1, 7), (5000, 0.3, 12345),
                                      (2048, 0.9, (1 << 63) + 5)])
def test_dropout_mask_restatement_bitexact(n, p, seed):
    """The restated mask stream equals the reference's dropout (ops.cpp:944-968)."""
    from oracle import refbind as rb
    if not rb.available():
        pytest.skip("oracle/_ref not built (needs the reference sources)")
    assert np.array_equal(rs.dropout_mask(n, p, seed), rb.dropout_mask(n, p, seed))


def test_window_sampler_uses_the_shared_generator():
    """apps/train.cpp's Rng is the dropout generator: the first window start
    is the first output modulo the window range."""
    r = rs.xorshift_stream(1041, 3)
    assert rs.sample_windows(1041, 20000, 64, 3) == [x % (20000 - 64 - 1) for x in r]


def test_clip_rule():
    gs = [np.full(4, 3.0, np.float32), np.full(9, 1.0, np.float32)]
    total = rs.clip_grad_norm(gs, 1.0)
    assert abs(total - np.sqrt(36 + 9)) < 1e-9
    scaled = np.sqrt(sum(float((g.astype(np.float64) ** 2).sum()) for g in gs))
    assert abs(scaled - 1.0) < 1e-5
    gs2 = [np.full(4, 0.01, np.float32)]
    assert rs.clip_grad_norm(gs2, 1.0) < 1.0 and gs2[0][0] == np.float32(0.01)


def test_restatement_vs_compiled_reference():
    from oracle import refbind as rb
    if not rb.available():
        pytest.skip("oracle/_ref not built (needs the reference sources)")
    rng = np.random.default_rng(3)
    c = rb.cfg(vocab=50, dim=32, layers=2, heads=2, ffn=40, max_seq=12)
    shapes = rs.param_shapes(50, 32, 2, 2, 40)
    assert rb.param_shapes(c) == shapes
    w = np.concatenate([np.ones(s, np.float32).ravel() if len(s) == 1 else
                        (rng.standard_normal(s) * 0.2).astype(np.float32).ravel() for s in shapes])
    idx, tgt = rng.integers(0, 50, 24), rng.integers(0, 50, 24)
    lg, l, g = rb.model_fwd_bwd(c, w, idx, tgt, 2, 12)
    l2, lg2, g2 = rs.model_fwd_bwd(w, idx, tgt, 2, 12, 50, 32, 2, 2, 40)
    assert abs(l - l2) <= 1e-5 * abs(l)
    assert rel_err(lg2, lg) < TOL
    assert rel_err(g2, g) < 1e-5


def test_reference_reproduces_tiny_fixture():
    """The fixture is reproducible from the reference (10 AdamW+clip steps)."""
    from oracle import refbind as rb
    if not rb.available():
        pytest.skip("oracle/_ref not built (needs the reference sources)")
    d = dict(np.load(f"{GOLDEN}/model_tiny.npz"))
    v, dim, L, H, F, ms = (int(x) for x in d["cfg"])
    c = rb.cfg(vocab=v, dim=dim, layers=L, heads=H, ffn=F, max_seq=ms)
    losses, norms, final = rb.train(c, d["weights"], d["idx"], d["tgt"], 2, 16, d["lrs"])
    assert np.array_equal(losses, d["losses"])
    assert np.array_equal(final, d["final"])
