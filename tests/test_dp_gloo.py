"""CPU: the data-parallel plan with 2 gloo ranks (no GPU)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from malaga_b200 import dp


def test_batches_are_length_sorted_chunks():
    lens = [5, 9, 3, 9, 7, 1, 4]
    bs = dp.batches(lens, 3)
    assert bs == [[1, 3, 4], [0, 6, 2], [5]]


def test_lpt_assignment_balances_and_covers():
    costs = [10, 9, 8, 7, 6, 5, 4, 3, 2, 1]
    parts = dp.assign(costs, 3)
    assert sorted(i for p in parts for i in p) == list(range(10))
    loads = [sum(costs[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= max(costs)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, lens, q, fail_rank):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        mine = dp.shard(lens, world, rank, 4, lambda b: 8)
        if rank == fail_rank:
            raise RuntimeError("injected rank failure")
        # stand-in decode: the "translation" of sentence i is [i] * len
        local = {i: [i] * lens[i] for b in mine for i in b}
        out = dp.gather(local, len(lens))
        q.put((rank, out))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _run(world, lens, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, lens, q, fail_rank)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    return res


def test_two_ranks_gather_every_sentence_in_order():
    lens = [3, 11, 7, 2, 9, 5, 8, 1, 6, 4]
    res = _run(2, lens)
    want = [[i] * lens[i] for i in range(len(lens))]
    assert res[0] == want and res[1] == want


def test_a_failing_rank_is_reported_not_hung():
    """A rank that raises before the gather: the other rank's collective ends
    with an error within the process-group timeout instead of hanging."""
    res = _run(2, [3, 4, 5, 6], fail_rank=1)
    assert "injected rank failure" in res[1]
    assert isinstance(res[0], str)  # the surviving rank saw an error, not results


class _FakeEngine:
    def __init__(self, k, fail_on=None):
        self.k, self.fail_on, self.seen = k, fail_on, []
        self.kernel_launches = 0

    def close(self):
        pass


def _pool(n, fail_on=None):
    pool = dp.StreamPool.__new__(dp.StreamPool)
    pool.engines = [_FakeEngine(k, fail_on) for k in range(n)]
    return pool


def test_stream_pool_maps_item_i_to_context_i_mod_n_in_order():
    import threading

    pool = _pool(3)
    tids = {}

    def fn(e, x):
        e.seen.append(x)
        tids.setdefault(e.k, set()).add(threading.get_ident())
        return (e.k, x * x)

    out = pool.map(fn, list(range(10)))
    assert out == [(i % 3, i * i) for i in range(10)]
    assert [e.seen for e in pool.engines] == [[0, 3, 6, 9], [1, 4, 7], [2, 5, 8]]
    assert all(len(t) == 1 for t in tids.values())  # each context's items on one host thread


def test_stream_pool_reraises_a_context_failure():
    pool = _pool(2)

    def fn(e, x):
        if x == 3:
            raise RuntimeError("context 1 failed")
        return x

    with pytest.raises(RuntimeError, match="context 1 failed"):
        pool.map(fn, list(range(6)))
