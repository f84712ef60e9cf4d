"""CPU: the multi-GPU dynamic batcher (malaga_b200/server.py) with fake backends
standing in for the per-GPU engines: the reference's drain-and-group policy
(crates/malaga/src/server.rs:74-112), least-loaded dispatch, and a worker that
fails on the host while the others finish."""
import threading
import time

import pytest

from malaga_b200.server import Server


class FakeBackend:
    """translate(): the "translation" of a sentence is its ids without the tags,
    prefixed by the target token; records the groups it ran."""

    def __init__(self, delay=0.01, fail=False):
        self.delay, self.fail, self.groups, self.lock = delay, fail, [], threading.Lock()

    def translate(self, srcs, tgt, beam):
        time.sleep(self.delay)
        if self.fail:
            raise RuntimeError("injected worker failure (CUDA_ERROR_LAUNCH_FAILED)")
        with self.lock:
            self.groups.append((len(srcs), tgt, beam))
        return [[tgt] + s[1:-1] for s in srcs]


def _want(srcs, tgt):
    return [[tgt] + s[1:-1] for s in srcs]


def test_every_job_gets_its_own_translation_in_order():
    backs = [FakeBackend(), FakeBackend(), FakeBackend()]
    srv = Server(backs)
    jobs = [srv.submit([[9, i, i + 1, 2], [9, 7, 2]], tgt=100 + i % 2, beam=1 + i % 2) for i in range(60)]
    for i, j in enumerate(jobs):
        assert j.future.result(timeout=10) == _want([[9, i, i + 1, 2], [9, 7, 2]], 100 + i % 2)
    srv.close()
    # drained jobs were decoded together, each group one (target, beam)
    groups = [g for b in backs for g in b.groups]
    assert sum(n for n, _, _ in groups) == 120
    assert any(n > 2 for n, _, _ in groups)
    # least-loaded dispatch used every worker
    assert all(b.groups for b in backs)


def test_a_failing_worker_is_retired_and_its_jobs_finish_elsewhere():
    backs = [FakeBackend(fail=True), FakeBackend(), FakeBackend()]
    srv = Server(backs)
    jobs = [srv.submit([[9, i, 2]], tgt=5) for i in range(40)]
    for i, j in enumerate(jobs):
        assert j.future.result(timeout=10) == [[5, i]]
    assert not srv.workers[0].alive and "injected" in str(srv.workers[0].error)
    assert srv.workers[1].alive and srv.workers[2].alive
    srv.close()


def test_no_worker_left_fails_the_jobs_without_hanging():
    srv = Server([FakeBackend(fail=True), FakeBackend(fail=True)])
    jobs = [srv.submit([[9, i, 2]], tgt=5) for i in range(6)]
    for j in jobs:
        with pytest.raises(RuntimeError):
            j.future.result(timeout=10)
    srv.close()
