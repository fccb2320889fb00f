"""Benchmark of the batched sampling step (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg2]

A step samples one token for every row of one batch of logits: at N=1 the headline
configuration, [256, 128256] fp32 logits, temperature 0.7, top_k 50, top_p 0.95 (the metric's
configuration). Logits are seeded synthetic data with the benchmark's shape and distribution
(pagedbatch_b200.workloads). Under torchrun each rank samples its own batch on its own GPU
(rows shard with no communication: weak scaling) and the step time is the max over ranks.

* value: sampled rows/s over the whole job, inputs resident in HBM. K steps are captured in one
  CUDA graph and replayed between CUDA events; each step reads one of 4 rotating input copies
  (4 x 131 MB > 126 MB L2), so every step streams its logits from HBM.
* e2e: the same metric through the public API ``sample_tokens`` with the logits in pinned host
  memory: host->device copy of the logits and parameters, the launch, device->host tokens.
* roofline: algorithmic bytes (B*V*elem read once) per launch / average launch time, against
  the measured HBM copy bandwidth in MEASURED_PEAKS.json.
* cpu_baseline: the reference's own torch operations (oracle/torch_port.py, the calls of
  pagedbatch/sampling.py:12-27) timed per row on this host's cores over a bounded sample.

``--impl reference`` times only that CPU implementation (rank 0; other ranks exit at once).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

from pagedbatch_b200 import _lib, ops, sampling, workloads  # noqa: E402

METRIC = "sampled rows/s and us/step at B=256,V=128256 fp32; % HBM peak; 1/2/4/8 GPU"
FALLBACK_HBM_GBS = 6650.0
NROT = 4


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def make_workload(name: str, rank: int):
    fn = {"cfg0": workloads.config0, "cfg1": workloads.config1, "cfg2": workloads.config2,
          "cfg2flat": workloads.config2_flat, "cfg3": workloads.config3}[name]
    return fn(seed=rank)


class ClockSampler:
    """nvidia-smi clock / throttle samples while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""
        return False

    def summary(self):
        rows = [r.split(", ") for r in self.out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_baseline(w, budget_s: float = 10.0, min_rows: int = 8):
    """The reference's per-row torch calls over a bounded sample of the workload's rows."""
    from oracle import torch_port

    torch.set_num_threads(os.cpu_count() or 1)
    x = w.logits
    params = [(p.temperature, p.top_k, p.top_p) for p in w.params]
    done, t0 = 0, time.perf_counter()
    while True:
        r = done % w.rows
        torch_port.sample_row(x[r], *params[r], torch.Generator().manual_seed(w.seeds[r]))
        done += 1
        el = time.perf_counter() - t0
        if done >= min_rows and el >= budget_s:
            break
    return done / el, done, el


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = make_workload(args.workload, 0)
    # one timing of a few rows sizes each step's sample to keep the whole run to ~2 minutes
    rate, _, _ = cpu_baseline(w, budget_s=1.0, min_rows=2)
    per_step = max(1, int(120.0 * rate / max(1, args.steps + args.warmup)))
    per_step = min(per_step, w.rows)
    from oracle import torch_port

    params = [(p.temperature, p.top_k, p.top_p) for p in w.params]
    times = []
    for s in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        for j in range(per_step):
            r = (s * per_step + j) % w.rows
            torch_port.sample_row(w.logits[r], *params[r], torch.Generator().manual_seed(w.seeds[r]))
        if s >= args.warmup:
            times.append(time.perf_counter() - t0)
    tot = sum(times)
    value = per_step * args.steps / tot
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": w.name, "rows_per_step_sampled": per_step, "full_batch_rows": w.rows},
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{per_step} rows per step of {w.name}, reference torch ops per row"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_vocab_parallel(args):
    """Config 3: each rank holds a column slice of [1024, 128256] bf16; shard candidates, one NCCL
    all-gather of the per-row records, merge. Strong scaling (the job is fixed as N grows)."""
    from pagedbatch_b200.vocab_parallel import CudaKernels, record_cap

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    _lib.load()
    w = workloads.config3(seed=0)
    B, V = w.logits.shape
    lo, hi = V * rank // world, V * (rank + 1) // world
    xs = [w.logits[:, lo:hi].contiguous().to(dev) for _ in range(NROT)]
    rec = sampling.pack_rows(w.params, np.array(w.uniforms()))
    dparams = ops.params_tensor(rec, dev)
    cap = record_cap(w.params)
    kern = CudaKernels()
    rb = _lib.record_bytes(cap)
    gathered = torch.empty((world, B, rb), dtype=torch.uint8, device=dev)

    def step(i):
        mine = kern.candidates(xs[i % NROT], dparams, lo, cap)
        if dist:
            dist.all_gather_into_tensor(gathered.view(world * B, rb), mine)
            return kern.merge(gathered, dparams, cap)
        return kern.merge(mine.unsqueeze(0), dparams, cap)

    for i in range(args.warmup):
        tok, info = step(i)
    torch.cuda.synchronize(dev)
    fallback = int((ops.info_records(info)["status"] == _lib.ROW_FALLBACK).sum())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        if dist:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev0.record()
        for i in range(args.steps):
            step(i)
        ev1.record()
        torch.cuda.synchronize(dev)
        if dist:
            dist.barrier()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    step_ms = ms_max / args.steps
    peak, peak_kind = load_peaks()
    shard_bytes = B * (hi - lo) * 2
    line = {
        "metric": "vocab-parallel sampled rows/s at B=1024,V=128256 bf16 (config 3); 1/2/4/8 GPU",
        "value": B * args.steps / (ms_max / 1e3), "unit": "rows/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "us_per_step": step_ms * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": w.name, "rows": B, "vocab": V, "shard_vocab": hi - lo,
                   "parallelism": f"vocab-parallel over {world} rank(s): one NCCL all-gather of {rb} B per row per rank",
                   "l2": f"{NROT} rotating input copies ({NROT * shard_bytes / 1e6:.0f} MB per rank)",
                   "timing": "eager launches between CUDA events, max over ranks", "fallback_rows": fallback},
        "roofline": {"bound": "hbm", "achieved": shard_bytes / (step_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": shard_bytes / (step_ms / 1e3) / 1e9 / peak, "peak_source": f"{peak_kind} hbm_gbs",
                     "traffic": None, "alg_bytes_per_launch": shard_bytes},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_ours(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    _lib.load()
    w = make_workload(args.workload, rank)
    B, V = w.logits.shape
    elem = w.logits.element_size()
    rec = sampling.pack_rows(w.params, np.array(w.uniforms()))
    params = ops.params_tensor(rec, dev)
    bufs = [w.logits.to(dev) for _ in range(NROT)]
    stream = torch.cuda.Stream(dev)

    # warm-up (also sets the kernel's shared-memory attribute before capture)
    with torch.cuda.stream(stream):
        for i in range(max(3, args.warmup)):
            ops.sample_op(bufs[i % NROT], params)
    stream.synchronize()
    if args.profile:
        # profiling mode: a few eager launches for ncu, no timing and no JSON line
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                ops.sample_op(bufs[i % NROT], params)
        torch.cuda.synchronize(dev)
        print(f"profile launches done: {args.warmup} warm-up + {args.steps} on {w.name}", flush=True)
        return

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(args.steps):
            out = ops.sample_op(bufs[i % NROT], params)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize(dev)

    # keep the GPU busy for ~1 s around the timed region so the clock samples mean something
    soak = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    soak[0].record(stream)
    with torch.cuda.stream(stream):
        graph.replay()
    soak[1].record(stream)
    torch.cuda.synchronize(dev)
    per_replay_ms = max(soak[0].elapsed_time(soak[1]), 1e-3)
    n_soak = max(1, int(600.0 / per_replay_ms))

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            for _ in range(n_soak):
                graph.replay()
        if dist:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev0.record(stream)
        with torch.cuda.stream(stream):
            graph.replay()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
        if dist:
            dist.barrier()
        with torch.cuda.stream(stream):
            for _ in range(n_soak // 2):
                graph.replay()
        torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    step_ms = ms_max / args.steps
    value = world * B * args.steps / (ms_max / 1e3)

    # end to end through the public API, logits in pinned host memory
    host = w.logits.pin_memory()
    gens = [torch.Generator().manual_seed(s) for s in w.seeds]
    for _ in range(2):
        sampling.sample_tokens(host, w.params, gens)
    torch.cuda.synchronize(dev)
    e2e_steps = max(3, min(20, args.steps))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        toks = sampling.sample_tokens(host, w.params, gens)
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    et = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
    if dist:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_s = float(et.item())
    assert len(toks) == B

    peak, peak_kind = load_peaks()
    alg_bytes = B * V * elem
    achieved = alg_bytes / (step_ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "us_per_step": step_ms * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": {4: "f32", 2: "bf16"}[elem], "data": "synthetic",
        "config": {"workload": w.name, "rows": B, "vocab": V, "rows_per_gpu": B,
                   "parallelism": f"rows sharded over {world} GPU(s), no collective",
                   "l2": f"{NROT} rotating input copies ({NROT * alg_bytes / 1e6:.0f} MB > 126 MB L2)",
                   "timing": "CUDA graph of K launches between CUDA events, max over ranks"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} hbm_gbs", "traffic": load_traffic(w.name),
                     "alg_bytes_per_launch": alg_bytes},
        "e2e": {"value": world * B / e2e_s, "unit": "rows/s", "ms_per_step": e2e_s * 1e3,
                "h2d_bytes_per_step": alg_bytes + rec.nbytes, "d2h_bytes_per_step": 8 * B,
                "api": "pagedbatch_b200.sample_tokens(pinned host logits)"},
        # one launch per step; PB_PATH=pass makes it two (the persistent pass, then the full-row
        # kernel on the rows the pass could not settle) after a memset of the pass's row counters
        "gpu_launches": args.steps * (2 if ops._pass_path() else 1),
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, n, el = cpu_baseline(w)
        line["cpu_baseline"] = {"value": rate, "unit": "rows/s", "cores": torch.get_num_threads(), "kind": "port",
                                "sample": f"{n} rows of {w.name} in {el:.1f} s, reference torch ops per row"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def load_traffic(workload):
    """DRAM bytes (read + write) of one launch on this workload, from a committed ncu summary."""
    path = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(workload, {}).get("dram_bytes_per_launch")
    except (OSError, ValueError):
        return None


def run_calibration(args):
    """Plain torch reductions over the same logits, timed like the sampler (rotating input copies,
    one CUDA graph of K launches between CUDA events): what one read-once pass over this tensor
    costs at this size on this GPU, beside the sampler itself. One JSON line, 1 GPU."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    w = make_workload(args.workload, 0)
    rec = sampling.pack_rows(w.params, np.array(w.uniforms()))
    params = ops.params_tensor(rec, dev)
    bufs = [w.logits.to(dev) for _ in range(NROT)]
    nbytes = w.logits.numel() * w.logits.element_size()
    stream = torch.cuda.Stream(dev)

    def graph_us(f):
        with torch.cuda.stream(stream):
            for i in range(args.warmup):
                f(bufs[i % NROT])
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(args.steps):
                f(bufs[i % NROT])
        g.replay()
        torch.cuda.synchronize(dev)
        times = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            with torch.cuda.stream(stream):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            times.append(e0.elapsed_time(e1) * 1e3 / args.steps)
        us = sorted(times)[2]
        return {"us_per_launch": us, "read_GBps": nbytes / (us * 1e-6) / 1e9}

    line = {
        "calibration": w.name,
        "bytes_per_launch": nbytes,
        "timing": "CUDA graph of K launches between CUDA events, median of 5 replays; "
                  f"{NROT} rotating input copies",
        "torch_sum": graph_us(lambda a: a.sum()),
        "torch_amax_rows": graph_us(lambda a: torch.amax(a, dim=1)),
        "torch_max_argmax_rows": graph_us(lambda a: torch.max(a, dim=1)),
        "pb_sample": graph_us(lambda a: ops.sample_op(a, params)),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="cfg2", choices=["cfg0", "cfg1", "cfg2", "cfg2flat", "cfg3"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true", help="eager launches only (for ncu), no timing")
    ap.add_argument("--calibrate", action="store_true",
                    help="time plain torch reductions over the same logits beside the sampler (1 GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.calibrate:
        run_calibration(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload == "cfg3":
        run_vocab_parallel(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
