"""The per-GPU batch scheduler (rokoko_b200.boxbench.run_batches) on the host
with fake contexts (no GPU): every batch runs once, a context that raises is
taken out of service and its batch runs on another context, and the call
fails when a batch keeps failing or no context is left."""
import time

import numpy as np
import pytest

from rokoko_b200 import boxbench


class FakeUtt:
    def __init__(self, i):
        self.i = i


class FakeCtx:
    """encode -> (None, lengths); decode -> one array per utterance; fail_on: the
    n-th encode (0-based) raises, or every one when fail_on == 'always'."""

    def __init__(self, name, fail_on=None, delay=0.0):
        self.name, self.fail_on, self.delay = name, fail_on, delay
        self.calls = 0
        self.pending = None
        self.batches = []

    def encode(self, utts):
        n = self.calls
        self.calls += 1
        time.sleep(self.delay)
        if self.fail_on == "always" or self.fail_on == n:
            raise RuntimeError(f"{self.name}: device error on batch {n}")
        self.pending = [u.i for u in utts]
        self.batches.append(list(self.pending))
        return None, [u.i + 1 for u in utts]

    def decode(self, Ls):
        return [np.full(L, i, np.float32) for i, L in zip(self.pending, Ls)]


def _batches(n_utts=40, b=4):
    idx = list(range(n_utts))
    return [idx[k:k + b] for k in range(0, n_utts, b)]


def _check(res, n_utts=40):
    got = sorted(i for i, _ in res)
    assert got == list(range(n_utts))
    for i, pcm in res:
        assert pcm.shape == (i + 1,) and np.all(pcm == i)


def test_all_batches_run_once():
    utts = [FakeUtt(i) for i in range(40)]
    ctxs = [FakeCtx(f"c{k}", delay=0.001) for k in range(3)]
    tim = []
    res = boxbench.run_batches(ctxs, utts, _batches(), tim)
    _check(res)
    assert sum(len(c.batches) for c in ctxs) == 10 and len(tim) == 3


def test_failed_context_leaves_service_and_batch_is_retried():
    utts = [FakeUtt(i) for i in range(40)]
    ctxs = [FakeCtx("good0", delay=0.002), FakeCtx("bad", fail_on=1, delay=0.002), FakeCtx("good1", delay=0.002)]
    failures = []
    res = boxbench.run_batches(ctxs, utts, _batches(), failures=failures)
    _check(res)
    assert len(failures) == 1 and failures[0][0] == 1
    assert ctxs[1].calls == 2  # no batch after the failing one
    assert sum(len(c.batches) for c in ctxs) == 10


def test_failed_batch_is_picked_up_by_a_waiting_context():
    # two batches: the good context finishes its own and waits (queue empty, one batch in
    # flight) until the bad context's batch comes back
    utts = [FakeUtt(i) for i in range(8)]
    ctxs = [FakeCtx("bad", fail_on=0, delay=0.05), FakeCtx("good", delay=0.01)]
    failures = []
    res = boxbench.run_batches(ctxs, utts, _batches(8, 4), failures=failures)
    _check(res, 8)
    assert [f[0] for f in failures] == [0] and len(ctxs[1].batches) == 2


class BadInputCtx(FakeCtx):
    """Fails on any batch holding utterance 5 (a batch that fails wherever it runs)."""

    def encode(self, utts):
        if any(u.i == 5 for u in utts):
            self.calls += 1
            raise RuntimeError(f"{self.name}: bad input")
        return super().encode(utts)


def test_a_batch_that_keeps_failing_raises():
    utts = [FakeUtt(i) for i in range(8)]
    ctxs = [BadInputCtx("a"), BadInputCtx("b"), BadInputCtx("c")]
    failures = []
    with pytest.raises(RuntimeError, match="bad input"):
        boxbench.run_batches(ctxs, utts, _batches(8, 4), failures=failures, max_tries=2)
    assert len(failures) == 2 and all(f[1] == 1 for f in failures)


def test_no_context_left_raises():
    utts = [FakeUtt(i) for i in range(8)]
    ctxs = [FakeCtx("a", fail_on="always")]
    with pytest.raises(RuntimeError, match="device error"):
        boxbench.run_batches(ctxs, utts, _batches(8, 4), max_tries=3)


def test_run_share_two_contexts_in_plan_order():
    # the call shape tests/test_box_gpu.py and bench.py use: a share in plan order, batches of 8
    utts = [FakeUtt(i) for i in range(32)]
    order = list(range(31, -1, -1))
    ctxs = [FakeCtx("c0", delay=0.001), FakeCtx("c1", delay=0.001)]
    tim = []
    res = boxbench.run_share(ctxs, utts, order, 8, tim)
    _check(res, 32)
    taken = sorted(b for c in ctxs for b in map(tuple, c.batches))
    assert taken == sorted(tuple(order[k:k + 8]) for k in range(0, 32, 8))
    assert len(tim) == 2 and all(t[0] >= 0 and t[1] >= 0 for t in tim)
