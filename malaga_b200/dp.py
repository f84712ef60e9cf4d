"""Data-parallel decoding across the GPUs of one box.

Sentences are independent (the reference requires batch invariance:
spec/specification.md:35, crates/malaga-core/tests/pipeline.rs:45-57), so the
multi-GPU plan has no collective on the data path: each rank owns full weights
and decodes its own length-sorted batches; results are gathered on the host.

  batches   length-sorted chunks of max_batch (translator.rs:140-147)
  assign    longest-processing-time-first placement of batches on ranks by
            their decode cost, so the slowest rank finishes as early as possible
  decode    one rank's share through its own Engine (one process per GPU)
"""
from __future__ import annotations

import heapq


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
