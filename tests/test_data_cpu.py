"""Host logic of the data feed and the learning-rate schedule, no device
needed: the native window sampler (tt_sample_windows) against the restated
apps/train.cpp:145-153, 225-232 sampler, and tt_lr_at against the restated
apps/train.cpp:214-222 schedule."""
import numpy as np
import pytest

from oracle import restate as rs


@pytest.fixture(scope="module")
def tr():
    from tinytrain_b200 import trainer
    try:
        trainer.lib()
    except (ImportError, OSError) as e:
        pytest.skip(f"libtinytrain not built: {e}")
    return trainer


@pytest.mark.parametrize("seed", [0, 1041, (1 << 64) - 3])
def test_sampler_continues_the_reference_stream(tr, seed):
    """Consecutive draws continue one xorshift64* stream, as consecutive
    training steps of apps/train.cpp do."""
    s = tr.WindowSampler(seed)
    a = s.draw(20000, 64, 5)
    b = s.draw(20000, 64, 7)
    assert list(a) + list(b) == rs.sample_windows(seed, 20000, 64, 12)
    assert all(0 <= x < 20000 - 64 - 1 for x in list(a) + list(b))


def test_sampler_rejects_a_too_short_stream(tr):
    with pytest.raises(tr.TrainerError):
        tr.WindowSampler(1).draw(10, 9, 1)


def test_lr_schedule_matches_restatement(tr):
    base = 3e-4
    for step in list(range(0, 30)) + list(range(30, 1200, 37)) + [1199, 1200, 5000]:
        want = np.float32(base) * rs.lr_scale(step, 20, 1200)
        got = tr.lr_at(base, step, 20, 1200)
        assert abs(got - float(want)) <= 1e-6 * float(want), step
    assert tr.lr_at(1.0, 0, 10, 100) == np.float32(0.1)
    assert abs(tr.lr_at(1.0, 100, 10, 100) - 0.1) < 1e-6
