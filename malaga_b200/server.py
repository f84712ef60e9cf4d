"""Dynamic batching of translation requests over the GPUs of one box.

The reference serves requests from one inference thread (crates/malaga/src/
server.rs:72-112, 344-367): the HTTP handlers push a job into a channel, the
thread blocks on the first job, drains every job already queued, groups them by
(source language, target language, beam) and runs each group as one batched
translation, then replies to each job. The HTTP surface itself is outside the
decode path and is not rebuilt here; requests are token ids.

B200 layout: one worker thread per GPU, each owning its own engine (context,
weights, static states and CUDA graphs), each applying the reference's
drain-and-group policy to its own queue; a dispatcher sends every request to the
alive worker with the fewest decode tokens outstanding. Worker failures are
handled on the host: a worker whose backend raises stops taking work, and the
jobs of its failed group are sent to the other workers (once); a job that fails
twice, or when no worker is left, completes with the error.
"""
from __future__ import annotations

import concurrent.futures as cf
import dataclasses
import queue
import threading
import time
from typing import Callable, Protocol


@dataclasses.dataclass
class Job:
    srcs: list[list[int]]          # the request's sentences (token ids, src tag ... </s>)
    tgt: int                       # target language token
    beam: int = 1
    future: cf.Future = dataclasses.field(default_factory=cf.Future)
    t_submit: float = 0.0
    t_done: float = 0.0
    cost: int = 0                  # decode tokens this job adds to a worker's queue
    attempts: int = 0


class Backend(Protocol):
    """What a worker drives: translate_batch(srcs, tgt, beam) -> target ids per
    sentence (malaga_b200.translator.Translator with its GenOptions)."""

    def translate(self, srcs: list[list[int]], tgt: int, beam: int) -> list[list[int]]: ...


class TranslatorBackend:
    """A worker's backend on one GPU: an Engine and a Translator with fixed options."""

    def __init__(self, gguf_path: str, device: int, opts):
        from .translator import Engine, Translator

        self.engine = Engine(gguf_path, device=device)
        self.t = Translator(self.engine)
        self.opts = opts

    def budget(self, n: int) -> int:
        return self.t.budget(n, self.opts)

    def translate(self, srcs, tgt, beam):
        opts = dataclasses.replace(self.opts, beam_size=beam)
        return self.t.translate_batch(srcs, tgt, opts)

    def close(self):
        self.engine.close()


class Worker(threading.Thread):
    """One GPU's inference loop (server.rs:74-89 per queue)."""

    def __init__(self, index: int, backend: Backend, server: "Server"):
        super().__init__(daemon=True, name=f"malaga-gpu{index}")
        self.index, self.backend, self.server = index, backend, server
        self.q: queue.Queue = queue.Queue()
        self.outstanding = 0           # decode tokens queued or running (dispatcher's load measure)
        self.alive = True
        self.error: BaseException | None = None
        self.lock = threading.Lock()

    def submit(self, job: Job):
        with self.lock:
            self.outstanding += job.cost
        self.q.put(job)

    def run(self):
        while True:
            first = self.q.get()
            if first is None:
                return
            jobs = [first]
            while True:  # take every job already queued (try_recv)
                try:
                    j = self.q.get_nowait()
                except queue.Empty:
                    break
                if j is None:
                    self.q.put(None)  # stop after this batch
                    break
                jobs.append(j)
            while jobs:  # group by (target, beam) in arrival order of the first job
                key = (jobs[0].tgt, jobs[0].beam)
                group = [j for j in jobs if (j.tgt, j.beam) == key]
                jobs = [j for j in jobs if (j.tgt, j.beam) != key]
                if not self.alive:
                    self.server.redispatch(group, self)
                    continue
                self.run_group(group, key)

    def run_group(self, group: list[Job], key):
        srcs = [s for j in group for s in j.srcs]
        try:
            out = self.backend.translate(srcs, key[0], key[1])
        except BaseException as e:  # noqa: BLE001 - any backend failure takes this worker out
            self.alive = False
            self.error = e
            with self.lock:
                self.outstanding -= sum(j.cost for j in group)
            self.server.redispatch(group, self, e)
            return
        now = time.perf_counter()
        k = 0
        for j in group:
            n = len(j.srcs)
            j.t_done = now
            with self.lock:
                self.outstanding -= j.cost
            j.future.set_result(out[k: k + n])
            k += n


class Server:
    """Least-loaded dispatch over per-GPU workers."""

    def __init__(self, backends: list[Backend], cost: Callable[[list[list[int]]], int] | None = None):
        self.workers = [Worker(i, b, self) for i, b in enumerate(backends)]
        self.cost = cost or (lambda srcs: sum(2 * len(s) + 16 for s in srcs))
        self.lock = threading.Lock()
        for w in self.workers:
            w.start()

    def submit(self, srcs: list[list[int]], tgt: int, beam: int = 1) -> Job:
        job = Job(srcs=srcs, tgt=tgt, beam=beam, t_submit=time.perf_counter(), cost=self.cost(srcs))
        self._dispatch(job)
        return job

    def _dispatch(self, job: Job, exclude: Worker | None = None, err: BaseException | None = None):
        with self.lock:
            alive = [w for w in self.workers if w.alive and w is not exclude]
        if not alive or job.attempts >= 2:
            job.t_done = time.perf_counter()
            job.future.set_exception(err or RuntimeError("no inference worker left"))
            return
        job.attempts += 1
        min(alive, key=lambda w: w.outstanding).submit(job)

    def redispatch(self, group: list[Job], failed: Worker, err: BaseException | None = None):
        for j in group:
            self._dispatch(j, exclude=failed, err=err)

    def close(self):
        for w in self.workers:
            w.q.put(None)
        for w in self.workers:
            w.join(timeout=60)
