"""Benchmark of the NLLB decoder token loop (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload dp600|c2q4|c2|c1] [--impl ours|reference]

Metric: decoded tokens/s, NLLB-600M q4_k_m, batch 64, on
1/2/4/8 B200; p50 ms/sentence at batch 1.

Headline (default workload dp600): a fixed set of 1024 synthetic sentences
(config 2's lengths, uniform in [8, 64]) cut into 16 length-sorted batches of
64 (translator.rs:140-147) and placed on the ranks longest-processing-time
first (malaga_b200/dp.py): one process per GPU, no collective on the data
path, strong scaling (the total work is fixed as N grows). One bench step = one
pass of the hot path over every batch of the rank's share: the greedy decode
of each encoded batch, forced to 64 tokens per row (EOS ignored), through
mgb_greedy (CUDA-graph replay of the fused step). `value` = tokens of all
ranks / the slowest rank's device time (CUDA events on the engine's stream,
max over ranks).

`e2e`: the same metric through the public API from host buffers (token ids in
host memory -> mgb_encode -> mgb_greedy -> token ids back in host memory), per
step, for every batch of the share. `b1` (rank 0, N = 1): config 1 (batch 1,
34-token source, 32 forced steps) timed as the reference's `malaga bench`
(crates/malaga/src/main.rs:409-436: 3 warm-ups, p50 over 20 runs of a whole
sentence: encode + decode from host ids).

`roofline`: the dominant kernel (the fused LM head + argmax), its algorithmic
bytes over its launch time measured live (CUDA events, mgb_profile_step);
`step_roofline`: weight + KV bytes actually read per decode over the decode's
device time (north_star's definition).

`--impl reference`: the CPU restatement of the reference's algorithm (oracle/,
compiled C with OpenMP on every host core) on a bounded sample of the same
workload; the reference's own Rust/candle build cannot be compiled here.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

from malaga_b200 import dp, models  # noqa: E402

METRIC = "decoded tokens/s NLLB-600M q4_k_m b64 @1/2/4/8 B200; p50 ms/sentence b1"
C4_METRIC = "C4: decoded tokens/s NLLB-3.3B q4_k_m b128 @1/2/4/8 B200"
C5_METRIC = "C5 server: sustained decoded tokens/s; p50/p99 ms request latency"


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device, self.rows, self.stop = device, [], threading.Event()
        self.t = threading.Thread(target=self.run, daemon=True)

    def run(self):
        while not self.stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                if out.returncode == 0 and out.stdout.strip():
                    self.rows.append([x.strip() for x in out.stdout.strip().split(",")])
            except Exception:
                return
            self.stop.wait(0.2)

    def __enter__(self):
        self.t.start()
        return self

    def __exit__(self, *a):
        self.stop.set()
        self.t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 5 + i and "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


DESCRIBE = {
    "dp600": "1024 sentences (source lengths U[8,64]) in 16 length-sorted batches of 64, "
             "64 forced greedy steps per batch, batches placed on the ranks by LPT",
    "c1": "batch 1, source 32 random ids + language tag + </s>, 32 forced greedy steps",
    "c2": "batch 64 (q8_0 weights), source lengths U[8,64], 64 forced greedy steps",
    "c2q4": "batch 64, source lengths U[8,64], 64 forced greedy steps",
    "c4": "1024 sentences (source lengths lognormal, median 28, 8-128) in 8 length-sorted batches of 128, "
          "128 forced greedy steps per batch, batches placed on the ranks by LPT",
}
MODEL_NAMES = {"600m": "NLLB-600M", "3.3b": "NLLB-3.3B"}

# The LM-head kernel each batch size runs (the roofline's dominant kernel).
def lm_kernel(rows: int, preset: str) -> str:
    t = "Q6_K" if preset == "q4_k_m" else "Q8_0"
    if rows <= 8:
        return f"small_mm_kernel<{t}, ARGMAX, LN> (MMVQ LM head + argmax, {rows} row(s))"
    return f"gemm_tc_kernel<{t}, ARGMAX, 64> (tcgen05 MMQ LM head + argmax)"


def measured_traffic(key: str):
    """DRAM bytes per launch of a workload's LM-head kernel from the ncu capture
    summarized in profiles/traffic.txt (lines: key bytes_per_launch)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.txt")) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 2 and parts[0] == key and not line.startswith("#"):
                    return int(parts[1])
    except OSError:
        pass
    return None


def kv_bytes(info: dict, src_lens: list[int], steps: int) -> int:
    """K/V bytes the attention reads in one decode of a batch (f16 caches): at
    step t (0..steps, the start step included) every layer reads t+1 self-attention
    keys and values and the row's source-length cross keys and values."""
    per_key = info["decoder_layers"] * 2 * info["d_model"] * 2
    self_keys = (steps + 1) * (steps + 2) // 2
    return per_key * sum(self_keys + (steps + 1) * s for s in src_lens)


def cpu_sample(w) -> tuple[int, int]:
    """Rows and forced steps of the CPU baseline's bounded sample (about 10 s of
    work on 16 host threads for a batch of 64)."""
    rows = min(w.batch, len(w.sources))
    if w.model == "3.3b":
        return 16, 2
    return rows, (6 if rows > 8 else 16)


def cpu_baseline(w):
    """The oracle (CPU restatement, OpenMP on every host core) on a bounded
    sample of the workload: one batch of it decoding a few forced steps (plus
    the start step) from synthetic cross K/V."""
    import oracle

    path = models.model_path(w.model, w.preset, w.seed)
    # every host core (torchrun sets OMP_NUM_THREADS=1 for its processes)
    oracle.lib().orc_set_threads(len(os.sched_getaffinity(0)))
    orc = oracle.Oracle(path)
    rows, sample_steps = cpu_sample(w)
    src = sorted(w.sources, key=len, reverse=True)[:rows]
    t0 = time.perf_counter()
    orc.decode_timing_sample(src, models.TGT_TAG, sample_steps)
    dt = time.perf_counter() - t0
    toks = len(src) * sample_steps
    return {"value": toks / dt, "unit": "tokens/s", "cores": oracle.lib().orc_threads(), "kind": "port",
            "sample": f"{len(src)} rows x {sample_steps} forced decode steps (+1 start step) of {w.name} "
                      f"from synthetic cross K/V, {dt:.1f} s", "seconds": dt}


def run_reference(args, w):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    results = [cpu_baseline(w) for _ in range(args.warmup + args.steps)][args.warmup:]
    vals = [r["value"] for r in results]
    v = statistics.median(vals)
    cb = dict(results[-1])
    cb["value"] = v
    rows, sample_steps = cpu_sample(w)
    line = {"impl": "reference",
            "metric": C5_METRIC if w.name == "c5" else (METRIC if w.model == "600m" else C4_METRIC),
            "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * rows * sample_steps / v,
            "higher_is_better": True, "scaling": "strong" if w.name in ("dp600", "c4") else "weak",
            "vs_baseline": None,
            "dtype": "int8 dot / f32", "data": "synthetic",
            "config": {"workload": w.name, "model": f"nllb-{w.model}-{w.preset} (random init)", "sample_rows": rows,
                       "decode_steps_sampled": sample_steps},
            "cpu_baseline": cb, "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def bench_b1(eng, torch, stream, info, hbm, sl=-1):
    """Config 1 as the reference's bench: p50 over 20 whole sentences (host ids ->
    encode -> 32 forced steps -> host ids) after 3 warm-ups; also the device time."""
    w = models.workload("c1")
    src = w.sources
    ids = np.array(src, np.uint32)
    lens = np.array([len(s) for s in src], np.uint32)
    out = np.empty((1, w.steps), np.uint32)
    wall, dev = [], []
    for it in range(3 + 20):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e0.record(stream)
        b = eng.encode_array(ids, lens)
        eng.greedy(b, models.TGT_TAG, w.steps, sync_every=4, force=True, out=out, shortlist=sl)
        e1.record(stream)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        b.free()
        if it >= 3:
            wall.append((t1 - t0) * 1e3)
            dev.append(e0.elapsed_time(e1))
    # the decode alone (graph replay), for the per-step roofline
    b = eng.encode_array(ids, lens)
    eng.greedy(b, models.TGT_TAG, w.steps, sync_every=4, force=True, out=out, shortlist=sl)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(5):
        eng.greedy(b, models.TGT_TAG, w.steps, sync_every=4, force=True, out=out, shortlist=sl)
    e1.record(stream)
    torch.cuda.synchronize()
    dec_ms = e0.elapsed_time(e1) / 5
    lm_ms, _ = eng.profile_step(b, models.TGT_TAG, 8)
    b.free()
    steps = w.steps + 1  # the start step runs the whole decoder too
    by = steps * info["decoder_step_bytes"] + kv_bytes(info, [len(s) for s in src], w.steps)
    lm_bytes = info["lm_head_bytes"]
    return {
        "workload": f"c1: NLLB-600M q4_k_m (random init, seed 0), {DESCRIBE['c1']}",
        "p50_ms_per_sentence": statistics.median(wall), "p90_ms_per_sentence": float(np.percentile(wall, 90)),
        "p50_device_ms_per_sentence": statistics.median(dev), "iterations": len(wall), "warmup": 3,
        "decode_ms": dec_ms, "ms_per_decoder_step": dec_ms / steps, "tokens_per_s": w.steps / (dec_ms / 1e3),
        "step_roofline": {"bytes_per_decode": by, "achieved_gbs": by / (dec_ms / 1e3) / 1e9, "peak": hbm,
                          "frac": by / (dec_ms / 1e3) / 1e9 / hbm},
        "lm_head": {"kernel": lm_kernel(1, "q4_k_m"), "launch_ms": lm_ms, "algorithmic_bytes": lm_bytes,
                    "achieved_gbs": lm_bytes / (lm_ms / 1e3) / 1e9,
                    "frac": lm_bytes / (lm_ms / 1e3) / 1e9 / hbm, "traffic": measured_traffic("b1")},
    }


def run_c3(args):
    """Config 3: beam search (beam 4, length penalty 1.0) over 16 sources of 48
    tokens, at most 96 steps, NLLB-1.3B q4_k_m (random init, seed 2), through
    Engine.encode_array + Engine.beam (mgb_encode + mgb_beam) from host ids: the
    best hypotheses' tokens per second of device time (events around each whole
    call pair on the engine's stream), after --warmup untimed runs."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import torch

    from malaga_b200 import Engine

    w = models.workload("c3")
    path = models.model_path(w.model, w.preset, w.seed)
    eng = Engine(path)
    stream = torch.cuda.ExternalStream(eng.stream)
    ids = np.array(w.sources, np.uint32)
    lens = np.array([len(r) for r in w.sources], np.uint32)

    def once():
        b = eng.encode_array(ids, lens)
        out, olens = eng.beam(b, models.TGT_TAG, 4, w.steps, 1.0)
        b.free()
        return int(olens.sum())

    for _ in range(max(3, args.warmup)):
        once()
    ms, toks, wall = [], 0, time.perf_counter()
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        toks += once()
        e1.record(stream)
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1))
    wall = time.perf_counter() - wall
    total = sum(ms) / 1e3
    line = {"metric": C3_METRIC, "value": toks / total, "unit": "tokens/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.median(ms),
            "higher_is_better": True, "data": "synthetic",
            "beam_rows_steps_per_s": 16 * 4 * w.steps * args.steps / total,
            "e2e": {"value": toks / wall, "unit": "tokens/s", "h2d_bytes_per_step": int(ids.nbytes + lens.nbytes),
                    "d2h_bytes_per_step": int(16 * w.steps * 4 + 16 * 4)},
            "config": {"workload": "c3: NLLB-1.3B q4_k_m (random init, seed 2), beam 4, length penalty 1.0, 16 "
                                   "sources of 48 ids, at most 96 steps (64 beam rows per step)",
                       "step": "ms_per_step = one encode + beam search of the batch"}}
    eng.close()
    if not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = c3_cpu_sample()
        except Exception as e:  # reported, never fatal
            line["cpu_baseline"] = {"error": str(e)}
    print(json.dumps(line), flush=True)


C3_METRIC = "C3: beam-4 decoded tokens/s NLLB-1.3B q4_k_m b16"


def c3_cpu_sample() -> dict:
    """Config 3 on the oracle (the CPU restatement of encode + beam search,
    translator.rs:250-358, OpenMP on every host core): a bounded sample of the
    workload -- its first source, beam 4, at most 3 tokens -- timed whole; value
    = the best hypothesis' tokens per second."""
    import oracle

    w = models.workload("c3")
    path = models.model_path(w.model, w.preset, w.seed)
    oracle.lib().orc_set_threads(len(os.sched_getaffinity(0)))
    orc = oracle.Oracle(path)
    src, max_new = w.sources[:1], 3
    t0 = time.perf_counter()
    out = orc.beam(src, models.TGT_TAG, 4, max_new)
    dt = time.perf_counter() - t0
    return {"value": max(1, sum(len(r) for r in out)) / dt, "unit": "tokens/s", "cores": oracle.lib().orc_threads(),
            "kind": "port", "sample": f"1 source of {len(src[0])} ids, beam 4, at most {max_new} tokens "
                                      f"(encode + beam), {dt:.1f} s", "seconds": dt}


def run_reference_c3(args):
    """Config 3's reference arm, rank 0 only: c3_cpu_sample per step, the
    median over --steps after --warmup."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    results = [c3_cpu_sample() for _ in range(args.warmup + args.steps)][args.warmup:]
    v = statistics.median(r["value"] for r in results)
    cb = dict(results[-1])
    cb["value"] = v
    line = {"impl": "reference", "metric": C3_METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * statistics.median(r["seconds"] for r in results),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot / f32",
            "data": "synthetic",
            "config": {"workload": "c3", "model": "nllb-1.3b-q4_k_m (random init)", "sample": cb["sample"]},
            "cpu_baseline": cb, "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_c5(args):
    """Config 5: server dynamic batching (malaga_b200/server.py) on NLLB-600M
    q4_k_m over --gpus GPUs of one process (--streams worker threads, each with
    its own engine, per GPU): 4096 single-sentence requests arriving as a Poisson process at 2000
    requests/s, source lengths lognormal (median 24, 4-96), greedy decode with a
    budget of 1.5 x source length + 8. The stream runs once to capture every
    shape's CUDA graphs, then again timed: end-to-end latency per request (host
    clock from arrival to its reply) and sustained decoded tokens/s."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from malaga_b200.server import Server, TranslatorBackend
    from malaga_b200.translator import GenOptions

    w = models.workload("c5")
    path = models.model_path(w.model, w.preset, w.seed)
    arrivals = models.poisson_arrivals(len(w.sources), 2000.0, 4)
    opts = GenOptions(max_batch=64, budget_scale=1.5, budget_extra=8)
    backends = [TranslatorBackend(path, d, opts) for d in range(args.gpus) for _ in range(max(1, args.streams))]
    srv = Server(backends, cost=lambda srcs: sum(backends[0].budget(len(s)) for s in srcs))

    def stream():
        t0 = time.perf_counter()
        jobs = []
        for src, at in zip(w.sources, arrivals):
            while True:
                dt = at - (time.perf_counter() - t0)
                if dt <= 0:
                    break
                time.sleep(min(dt, 0.0005))
            jobs.append(srv.submit([src], models.TGT_TAG))
        outs = [j.future.result() for j in jobs]
        lat = np.array([j.t_done - j.t_submit for j in jobs]) * 1e3
        span = max(j.t_done for j in jobs) - t0
        toks = sum(len(o[0]) for o in outs)
        return lat, span, toks

    stream()  # warm-up: graph capture of every (batch, source, output) bucket
    lat, span, toks = stream()
    srv.close()
    line = {"metric": C5_METRIC, "value": toks / span,
            "unit": "tokens/s", "n_gpus": args.gpus, "higher_is_better": True, "data": "synthetic",
            "p50_ms": float(np.percentile(lat, 50)), "p99_ms": float(np.percentile(lat, 99)),
            "mean_ms": float(lat.mean()), "requests": len(lat), "decoded_tokens": toks, "seconds": span,
            "offered_rps": 2000.0, "achieved_rps": len(lat) / span,
            "config": {"workload": "c5: NLLB-600M q4_k_m (random init, seed 0), 4096 Poisson requests at 2000/s, "
                                   "lognormal lengths (median 24, 4-96), greedy, budget 1.5*len+8, max_batch 64",
                       "workers_per_gpu": max(1, args.streams),
                       "dispatch": "least outstanding decode tokens; per-worker drain-and-group (server.rs:74-89)"}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="dp600", choices=["dp600", "c2q4", "c2", "c1", "c5", "c4", "c3"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-b1", action="store_true")
    ap.add_argument("--fast-vocab", type=int, default=0, metavar="N",
                    help="decode over a synthetic vocabulary shortlist of N ids (--fast-vocab: not exact, "
                         "off by default); the LM-head roofline stays the full head's")
    ap.add_argument("--streams", type=int, default=None,
                    help="decode contexts (CUDA streams) per GPU for independent batches (dp.StreamPool); "
                         "default 8, 4 for c4 (3.3B: larger states)")
    args = ap.parse_args()
    if args.workload == "c5" and args.impl == "ours":
        return run_c5(args)
    if args.workload == "c3":
        return run_c3(args) if args.impl == "ours" else run_reference_c3(args)
    w = models.workload(args.workload)
    if args.impl == "reference":
        return run_reference(args, w)

    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    def model_file():
        if not args.fast_vocab:
            return models.model_path(w.model, w.preset, w.seed)
        # the same weights plus a synthetic shortlist holding the forced tokens
        V = models.config_of(w.model).vocab_size
        return models.shortlist_model_path(
            w.model, w.preset, w.seed,
            {"syn_Latn": models.synthetic_shortlist(V, args.fast_vocab, 11, [models.TGT_TAG])})

    # rank 0 generates the model file; the others wait for it
    if rank == 0:
        model_file()
    if world > 1:
        dist.barrier()
    path = model_file()
    sl = 0 if args.fast_vocab else -1

    # this rank's share: length-sorted batches of w.batch placed by LPT (a
    # single-batch workload is replicated on every rank instead)
    lens_all = [len(s) for s in w.sources]
    if w.name in ("dp600", "c4"):
        share = dp.shard(lens_all, world, rank, w.batch, lambda b: w.steps)
        scaling = "strong"
    else:
        share = [list(range(len(w.sources)))]
        scaling = "weak"
    srcs = [[w.sources[i] for i in b] for b in share]
    # independent batches decode on `streams` contexts of this GPU at once
    # (dp.StreamPool); batch i belongs to context i % streams
    streams = max(1, min(args.streams or (4 if w.model == "3.3b" else 8), len(srcs)))
    # (3.3B states at batch 128 are ~7 GB each: room for every source-length bucket)
    pool = dp.StreamPool(path, device=local, streams=streams, graph_cache_mb=65536 if w.model == "3.3b" else 8192)
    eng = pool.engines[0]
    info = eng.info
    cur = torch.cuda.current_stream()
    estreams = [torch.cuda.ExternalStream(e.stream, device=torch.device("cuda", local)) for e in pool.engines]
    stream = estreams[0]
    tgt, steps = models.TGT_TAG, w.steps
    batches = pool.map(lambda e, s: e.encode(s), srcs)
    outs = [np.empty((len(s), steps), np.uint32) for s in srcs]
    my_tokens = sum(len(s) for s in srcs) * steps
    total_tokens = (len(w.sources) if scaling == "strong" else world * len(w.sources)) * steps

    def decode_step():
        pool.map(lambda e, bo: e.greedy(bo[0], tgt, steps, sync_every=4, force=True, out=bo[1], shortlist=sl),
                 list(zip(batches, outs)))

    for _ in range(max(3, args.warmup)):
        decode_step()

    def timed(fn, k):
        """Device time of k calls of fn: an event on this thread's stream before,
        and after it one that waits for every context's stream."""
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        for _ in range(k):
            fn()
        for es in estreams:
            ev = torch.cuda.Event()
            ev.record(es)
            cur.wait_event(ev)
        e1.record(cur)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    l0 = pool.kernel_launches
    with ClockSampler(local) as clk:
        ms = timed(decode_step, args.steps)
    launches = pool.kernel_launches - l0
    ms_step = ms / args.steps
    value = total_tokens / (ms_step / 1e3)

    # e2e: host ids -> encode -> greedy -> host ids, every batch of the share, every step
    hosts = []
    for s in srcs:
        ids_host = np.full((len(s), max(len(r) for r in s)), 1, np.uint32)
        for i, r in enumerate(s):
            ids_host[i, : len(r)] = r
        hosts.append((ids_host, np.array([len(r) for r in s], np.uint32)))

    def e2e_one(e, item):
        (ih, lh), o = item
        b = e.encode_array(ih, lh)
        e.greedy(b, tgt, steps, sync_every=4, force=True, out=o, shortlist=sl)
        b.free()

    def e2e_step():
        pool.map(e2e_one, list(zip(hosts, outs)))

    e2e_step()
    k_e2e = max(1, min(args.steps, 3))
    ms_e2e = timed(e2e_step, k_e2e)
    e2e_value = total_tokens / (ms_e2e / k_e2e / 1e3)

    # roofline of the dominant kernel (fused LM head + argmax), timed live with events
    hbm, peak_kind = peaks()
    lm_ms, eager_step_ms = eng.profile_step(batches[0], tgt, 8)
    lm_bytes = info["lm_head_bytes"]
    achieved = lm_bytes / (lm_ms / 1e3) / 1e9
    step_bytes = info["decoder_step_bytes"]
    # weight + KV bytes of this rank's decodes per bench step
    rank_bytes = sum((steps + 1) * step_bytes + kv_bytes(info, [len(r) for r in s], steps) for s in srcs)
    rank_dev_ms = ms_step  # (max over ranks: the slowest rank's time)

    b1 = None
    if rank == 0 and world == 1 and not args.no_b1:
        if w.model == "600m" and w.preset == "q4_k_m":
            b1 = bench_b1(eng, torch, stream, info, hbm, sl)

    if rank == 0:
        line = {
            "metric": METRIC if w.model == "600m" else C4_METRIC,
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": "int8 dot / f32 (q8_1 activations x GGUF blocks)", "data": "synthetic",
            "config": {"workload": f"{w.name}: {MODEL_NAMES[w.model]} {w.preset} (random init, seed {w.seed}), "
                                   f"{DESCRIBE[w.name]}",
                       "global_batch": w.batch, "sentences": len(w.sources) * (1 if scaling == "strong" else world),
                       "decode_steps": steps, "parallelism": f"dp{world}",
                       "step": "ms_per_step = one pass over the rank's batches (each a whole forced decode)",
                       "batches_this_rank": len(srcs), "streams_per_gpu": streams,
                       **({"fast_vocab": f"shortlist of {args.fast_vocab} synthetic ids + source tokens (not exact)"}
                          if args.fast_vocab else {}),
                       "l2": "weights (%.0f MB per decoder step) exceed the 126 MB L2" % (step_bytes / 1e6)},
            "gpu_launches": launches,
            "e2e": {"value": e2e_value, "unit": "tokens/s",
                    "h2d_bytes_per_step": int(sum(ih.nbytes + lh.nbytes for ih, lh in hosts)),
                    "d2h_bytes_per_step": int(sum(o.nbytes for o in outs))},
            "roofline": {"bound": "hbm", "kernel": lm_kernel(len(srcs[0]), w.preset),
                         "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_source": peak_kind, "traffic": measured_traffic(f"b{len(srcs[0])}"),
                         "algorithmic_bytes": lm_bytes, "launch_ms": lm_ms},
            "step_roofline": {"bytes_per_step_rank0": rank_bytes, "weight_bytes_per_decoder_step": step_bytes,
                              "achieved_gbs": rank_bytes / (rank_dev_ms / 1e3) / 1e9,
                              "frac": rank_bytes / (rank_dev_ms / 1e3) / 1e9 / hbm,
                              "ms_per_decoder_step": ms_step / len(srcs) / (steps + 1),
                              "eager_step_ms": eager_step_ms},
            "clocks": clk.summary(),
        }
        if b1:
            line["b1"] = b1
        if not args.no_cpu_baseline and world == 1:
            try:
                line["cpu_baseline"] = cpu_baseline(w)
            except Exception as e:  # reported, never fatal
                line["cpu_baseline"] = {"error": str(e)}
        print(json.dumps(line), flush=True)
    for b in batches:
        b.free()
    pool.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
