"""The collective watchdog's wait loop (tt_watchdog_selftest: the code that
guards every distributed step's NCCL collectives) on fake probes, no GPU:
  - completion before the deadline: no abort;
  - an asynchronous communicator error: abort called once, outcome 1;
  - a collective that never completes (a peer left): abort called once
    after the deadline, outcome 2.
"""
import time

from tinytrain_b200 import trainer as trn


class Fake:
    def __init__(self, done_after=None, error_after=None):
        self.polls = 0
        self.aborts = 0
        self.done_after, self.error_after = done_after, error_after

    def done(self):
        self.polls += 1
        return int(self.done_after is not None and self.polls >= self.done_after)

    def error(self):
        return int(self.error_after is not None and self.polls >= self.error_after)

    def abort(self):
        self.aborts += 1
        return 0


def test_completes_without_abort():
    f = Fake(done_after=5)
    assert trn.watchdog_selftest(f.done, f.error, f.abort, 10.0) == 0
    assert f.aborts == 0 and f.polls == 5


def test_async_error_aborts_once():
    f = Fake(error_after=3)
    assert trn.watchdog_selftest(f.done, f.error, f.abort, 10.0) == 1
    assert f.aborts == 1 and f.polls == 3


def test_deadline_aborts_once():
    f = Fake()
    t0 = time.time()
    assert trn.watchdog_selftest(f.done, f.error, f.abort, 0.2) == 2
    dt = time.time() - t0
    assert f.aborts == 1
    assert 0.2 <= dt < 5.0
