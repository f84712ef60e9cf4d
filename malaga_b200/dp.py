"""Data-parallel decoding across the GPUs of one box.

Sentences are independent (the reference requires batch invariance:
spec/specification.md:35, crates/malaga-core/tests/pipeline.rs:45-57), so the
multi-GPU plan has no collective on the data path: each rank owns full weights
and decodes its own length-sorted batches; results are gathered on the host.

  batches   length-sorted chunks of max_batch (translator.rs:140-147)
  assign    longest-processing-time-first placement of batches on ranks by
            their decode cost, so the slowest rank finishes as early as possible
  decode    one rank's share through its own Engine (one process per GPU)
  StreamPool  several decode contexts (CUDA streams) on one GPU, each driven by
            its own host thread, decoding independent batches concurrently
"""
from __future__ import annotations

import heapq
import threading


def batches(lens: list[int], max_batch: int) -> list[list[int]]:
    """Indices sorted by descending length, cut into chunks of max_batch."""
    order = sorted(range(len(lens)), key=lambda i: -lens[i])
    return [order[i: i + max_batch] for i in range(0, len(order), max(1, max_batch))]


def batch_cost(batch: list[int], lens: list[int], steps: int) -> float:
    """Decode cost model: every step of a batch reads the weights once (a constant
    per step) plus attention over (source + generated) keys per row."""
    return steps * (1.0 + 1e-3 * sum(lens[i] + steps / 2 for i in batch))


def assign(costs: list[float], world: int) -> list[list[int]]:
    """LPT: batches in descending cost, each to the currently least-loaded rank.
    Returns per-rank lists of batch indices (ties go to the lower rank)."""
    heap = [(0.0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for b in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        load, r = heapq.heappop(heap)
        out[r].append(b)
        heapq.heappush(heap, (load + costs[b], r))
    return out


def shard(lens: list[int], world: int, rank: int, max_batch: int, steps_of) -> list[list[int]]:
    """The batches (lists of sentence indices) rank `rank` decodes."""
    bs = batches(lens, max_batch)
    costs = [batch_cost(b, lens, steps_of(b)) for b in bs]
    return [bs[i] for i in assign(costs, world)[rank]]


def decode_rank(engine, sources: list[list[int]], tgt: int, opts, world: int, rank: int) -> dict[int, list[int]]:
    """Decodes this rank's share through `engine`; returns {sentence index: ids}."""
    from .translator import Translator

    t = Translator(engine)
    lens = [len(s) for s in sources]
    out: dict[int, list[int]] = {}
    for b in shard(lens, world, rank, opts.max_batch, lambda b: max(t.budget(lens[i], opts) for i in b)):
        for i, ids in zip(b, t.generate([sources[i] for i in b], tgt, opts)):
            out[i] = ids
    return out


class StreamPool:
    """`streams` decode contexts on one GPU, each with its own CUDA stream,
    weight copy and graph cache, each driven by its own host thread (the C ABI
    calls release the GIL): independent batches decode concurrently. A decode
    step at batch sizes up to 64 is a chain of dependent, latency-bound launches
    that leaves SMs idle between kernels; the chains of a few batches
    interleave on the SMs (measured on B200 at batch 64, 16 batches: 1.25x the
    tokens/s with 2 streams, 1.33x with 3, 1.40x with 4). With more than one
    context open on a device the tensor-core matmuls pick SM-time-efficient
    token tiles (at least 32 tokens), which takes 4 streams to 1.56x and 8 to
    1.85x the one-stream rate. Item i of a map runs on context i % streams."""

    def __init__(self, gguf_path: str, device: int = 0, streams: int = 3, **engine_kw):
        from .translator import Engine

        self.engines = [Engine(gguf_path, device=device, **engine_kw) for _ in range(max(1, streams))]

    def __len__(self) -> int:
        return len(self.engines)

    def map(self, fn, items: list) -> list:
        """fn(engine, item) for every item, in order per context; results in input order."""
        n = len(self.engines)
        out: list = [None] * len(items)
        errors: list[BaseException] = []

        def work(k: int):
            try:
                for i in range(k, len(items), n):
                    out[i] = fn(self.engines[k], items[i])
            except BaseException as e:  # noqa: BLE001 - re-raised on the caller's thread
                errors.append(e)

        threads = [threading.Thread(target=work, args=(k,)) for k in range(min(n, len(items)))]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]
        return out

    @property
    def kernel_launches(self) -> int:
        return sum(e.kernel_launches for e in self.engines)

    def close(self):
        for e in self.engines:
            e.close()


def gather(local: dict[int, list[int]], n: int) -> list[list[int]] | None:
    """all_gather of every rank's results (torch.distributed must be initialised);
    returns the outputs in input order on every rank."""
    import torch.distributed as dist

    parts: list = [None] * dist.get_world_size()
    dist.all_gather_object(parts, local)
    merged: dict[int, list[int]] = {}
    for p in parts:
        merged.update(p)
    if sorted(merged) != list(range(n)):
        raise RuntimeError("data-parallel decode lost or duplicated sentences")
    return [merged[i] for i in range(n)]
