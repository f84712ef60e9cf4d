"""Benchmark of the NLLB decoder token loop (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c2q4|c2|c1] [--impl ours|reference]

Metric: decoded tokens/s, NLLB-600M, batch 64, on 1/2/4/8 B200.
One bench step = one pass of the hot path over one batch: the greedy decode of
an encoded batch of 64 sentences, forced to 64 steps (EOS ignored), through
mgb_greedy (CUDA-graph replay of the fused step). Inputs are synthetic: a
random-init NLLB-600M converted to GGUF, and seeded token ids (config 2's
batch: lengths uniform in [8, 64]). Each rank decodes its own batch ("weak"
scaling, no collective on the data path); `value` = tokens of all ranks / the
slowest rank's device time.

`e2e`: the same metric through the public API from host buffers (token ids in
host memory -> mgb_encode -> mgb_greedy -> token ids back in host memory) per
step. `--impl reference`: the CPU restatement of the reference's algorithm
(oracle/, compiled C with OpenMP on every host core) on a bounded sample of the
same workload; the reference's own Rust/candle build cannot be compiled here.
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

from malaga_b200 import models  # noqa: E402

METRIC = "decoded tokens/s NLLB-600M q4_k_m b64 @1/2/4/8 B200; p50 ms/sentence b1"


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
    "c1": "batch 1, source 32 random ids + language tag + </s>, 32 forced greedy steps",
    "c2": "batch 64 (q8_0 weights), source lengths U[8,64], 64 forced greedy steps",
    "c2q4": "batch 64, source lengths U[8,64], 64 forced greedy steps",
}

# The LM-head kernel each workload runs (the roofline's dominant kernel).
LM_KERNEL = {
    "c1": "gemv_fused_kernel<Q6_K, ARGMAX, LN, 1> (small-batch LM head + argmax)",
    "c2": "gemm_tc_kernel<Q8_0, ARGMAX, 64> (tcgen05 LM head + argmax)",
    "c2q4": "gemm_tc_kernel<Q6_K, ARGMAX, 64> (tcgen05 LM head + argmax)",
}


def measured_traffic(workload: str):
    """DRAM bytes per launch of the workload's LM-head kernel from the ncu capture
    summarized in profiles/traffic.txt (lines: workload bytes_per_launch)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.txt")) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 2 and parts[0] == workload and not line.startswith("#"):
                    return int(parts[1])
    except OSError:
        pass
    return None


def cpu_baseline(w, max_seconds: float = 20.0):
    """The oracle (CPU restatement, OpenMP on every host core) on a bounded sample:
    the workload's full batch decoding 2 steps from synthetic cross K/V."""
    import oracle

    path = models.model_path(w.model, w.preset, w.seed)
    orc = oracle.Oracle(path)
    sample_steps = 4
    t0 = time.perf_counter()
    orc.decode_timing_sample(w.sources, models.TGT_TAG, sample_steps)
    dt = time.perf_counter() - t0
    # the discarded decoder-start step is timed too, as on the GPU path; count generated tokens
    toks = len(w.sources) * sample_steps
    return {"value": toks / dt, "unit": "tokens/s", "cores": oracle.lib().orc_threads(), "kind": "port",
            "sample": f"{len(w.sources)} rows x {sample_steps} decode steps (+1 start step) of {w.name} "
                      f"from synthetic cross K/V, {dt:.1f} s"}


def run_reference(args, w):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    results = [cpu_baseline(w) for _ in range(args.warmup + args.steps)][args.warmup:]
    vals = [r["value"] for r in results]
    v = statistics.median(vals)
    cb = dict(results[-1])
    cb["value"] = v
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * len(w.sources) * 4 / v,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot / f32",
            "data": "synthetic", "config": {"workload": w.name, "model": f"nllb-600m-{w.preset} (random init)",
                                            "batch": len(w.sources), "decode_steps_sampled": 4},
            "cpu_baseline": cb, "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="c2q4", choices=["c2q4", "c2", "c1"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
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
    # rank 0 generates the model file; the others wait for it
    if rank == 0:
        path = models.model_path(w.model, w.preset, w.seed)
    if world > 1:
        dist.barrier()
    path = models.model_path(w.model, w.preset, w.seed)

    from malaga_b200 import Engine

    eng = Engine(path, device=local)
    stream = torch.cuda.ExternalStream(eng.stream, device=torch.device("cuda", local))
    tgt = models.TGT_TAG
    src = w.sources
    batch = eng.encode(src)
    rows, steps = len(src), w.steps
    tokens_per_step = rows * steps
    out = np.empty((rows, steps), np.uint32)

    def decode_step():
        eng.greedy(batch, tgt, steps, sync_every=4, force=True, out=out)

    for _ in range(max(3, args.warmup)):
        decode_step()

    def timed(fn, k):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    l0 = eng.kernel_launches
    with ClockSampler(local) as clk:
        ms = timed(decode_step, args.steps)
    launches = eng.kernel_launches - l0
    ms_step = ms / args.steps
    value = world * tokens_per_step / (ms_step / 1e3)

    # e2e: host ids -> encode -> greedy -> host ids, every step
    ids_host = np.full((rows, max(len(s) for s in src)), 1, np.uint32)
    for i, s in enumerate(src):
        ids_host[i, : len(s)] = s
    lens_host = np.array([len(s) for s in src], np.uint32)

    def e2e_step():
        b = eng.encode_array(ids_host, lens_host)
        eng.greedy(b, tgt, steps, sync_every=4, force=True, out=out)
        b.free()

    e2e_step()
    ms_e2e = timed(e2e_step, max(1, min(args.steps, 3)))
    e2e_value = world * tokens_per_step / (ms_e2e / max(1, min(args.steps, 3)) / 1e3)

    # roofline of the dominant kernel (fused LM head + argmax), timed live with events
    lm_ms, step_ms = eng.profile_step(batch, tgt, 8)
    lm_bytes = eng.info["lm_head_bytes"]
    hbm, peak_kind = peaks()
    achieved = lm_bytes / (lm_ms / 1e3) / 1e9
    step_bytes = eng.info["decoder_step_bytes"]

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 dot / f32 (q8 activations x GGUF blocks)", "data": "synthetic",
            "config": {"workload": f"{w.name}: NLLB-600M {w.preset} (random init, seed {w.seed}), {DESCRIBE[w.name]}",
                       "global_batch": rows * world, "decode_steps": steps, "parallelism": f"dp{world}",
                       "l2": "weights (%.0f MB/step) exceed the 126 MB L2" % (step_bytes / 1e6)},
            "gpu_launches": launches,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": int(ids_host.nbytes + lens_host.nbytes),
                    "d2h_bytes_per_step": int(out.nbytes)},
            "roofline": {"bound": "hbm", "kernel": LM_KERNEL[w.name],
                         "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_source": peak_kind, "traffic": measured_traffic(w.name),
                         "algorithmic_bytes": lm_bytes, "launch_ms": lm_ms},
            "step_roofline": {"weight_bytes_per_step": step_bytes, "eager_step_ms": step_ms,
                              "graph_step_ms": ms_step / steps,
                              "frac_of_hbm": step_bytes / (ms_step / steps / 1e3) / 1e9 / hbm},
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline and world == 1:
            try:
                line["cpu_baseline"] = cpu_baseline(w)
            except Exception as e:  # reported, never fatal
                line["cpu_baseline"] = {"error": str(e)}
        print(json.dumps(line), flush=True)
    batch.free()
    eng.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
