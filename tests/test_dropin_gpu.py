"""The drop-in boundary end to end: the reference's training program
(apps/train.cpp, unmodified) built twice, against the reference's CPU library
(oracle/_ref/train_ref, the oracle) and against this repository's library
(oracle/_ref/train_b200, every op on the B200). Both read the same int32
token file with the same flags; their logged per-step losses (which cover the
window sampler, the LR schedule, model init, forward, backward and AdamW)
must agree within 1e-3, and both final checkpoints must load in the
reference. With --dropout the masks come from the device generator and must
equal the reference's for the losses to agree."""
import os
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_BIN = os.path.join(ROOT, "oracle", "_ref", "train_ref")
B200_BIN = os.path.join(ROOT, "oracle", "_ref", "train_b200")
ARGS = ["--steps", "5", "--batch-size", "4", "--seq-len", "64", "--dim", "128", "--layers", "2",
        "--heads", "2", "--ffn", "256", "--max-seq", "64", "--warmup", "2", "--lr", "1e-3",
        "--seed", "5", "--ckpt-every", "1000"]


def _losses(out):
    rows = [ln.split() for ln in open(os.path.join(out, "losses.txt")) if ln.strip()]
    return np.array([float(r[1]) for r in rows])


def _run(binary, tokens, out, extra):
    r = subprocess.run([binary, "--tokens", tokens, "--out", out] + ARGS + extra,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (binary, r.stdout[-2000:], r.stderr[-2000:])
    return _losses(out)


@pytest.mark.parametrize("extra", [[], ["--dropout", "0.1"]], ids=["plain", "dropout"])
def test_reference_train_program_on_b200(cuda, tmp_path, extra):
    if not (os.path.exists(REF_BIN) and os.path.exists(B200_BIN)):
        pytest.skip("oracle/_ref train binaries not built (they need the reference sources)")
    from oracle import refbind as rb
    tokens = str(tmp_path / "tokens.bin")
    np.random.default_rng(11).integers(0, 32000, 20000).astype(np.int32).tofile(tokens)
    ref = _run(REF_BIN, tokens, str(tmp_path / "ref"), extra)
    ours = _run(B200_BIN, tokens, str(tmp_path / "b200"), extra)
    assert ref.shape == ours.shape == (5,)
    assert np.abs(ref - ours).max() <= 1e-3, (ref, ours)
    c = rb.cfg(vocab=32000, dim=128, layers=2, heads=2, ffn=256, max_seq=64)
    w_ref = rb.load_checkpoint(c, str(tmp_path / "ref" / "ckpt-final"))
    w_ours = rb.load_checkpoint(c, str(tmp_path / "b200" / "ckpt-final"))
    assert w_ref.shape == w_ours.shape
    assert np.abs(w_ref - w_ours).max() <= 1e-2


REF_TESTS_B200 = os.path.join(ROOT, "oracle", "_ref", "ref_tests_b200")


def test_reference_unit_tests_on_b200(cuda, tmp_path):
    """The reference's own unit tests (tests/test_scaffold.cpp,
    tests/test_autograd.cpp, tests/test_model.cpp: finite-difference
    gradchecks of every op and of a tiny transformer, AdamW/SGD convergence,
    the checkpoint format), compiled unmodified against this library on the
    gtest-compatible harness, pass with every op on the device."""
    if not os.path.exists(REF_TESTS_B200):
        pytest.skip("oracle/_ref/ref_tests_b200 not built (it needs the reference sources)")
    r = subprocess.run([REF_TESTS_B200], capture_output=True, text=True, timeout=600,
                       cwd=str(tmp_path))
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "[  PASSED  ] 22 tests." in r.stdout, r.stdout[-2000:]
