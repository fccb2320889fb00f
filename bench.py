"""Benchmark of the batched sampling step (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg2]

A step samples one token for every row of one batch of logits: at N=1 the headline
configuration, [256, 128256] fp32 logits, temperature 0.7, top_k 50, top_p 0.95 (the metric's
configuration). Logits are seeded synthetic data with the benchmark's shape and distribution
(pagedbatch_b200.workloads). Under torchrun each rank samples its own batch on its own GPU
(rows shard with no communication: weak scaling) and the step time is the max over ranks; with
N > 1 the line also carries the vocabulary-parallel configuration (config 3: [1024, 128256] bf16
split by columns over the N ranks, one NCCL all-gather per step).

* value: sampled rows/s over the whole job, inputs resident in HBM. K steps are captured in one
  CUDA graph and the graph is replayed until at least 200 ms of steps are timed, each replay
  between CUDA events; value and ms_per_step come from the median replay (max over ranks);
  timing_stats adds the per-launch median and p99 (from a copy of the graph with an event between
  launches). Each step reads one of 4 rotating input copies (4 x 131 MB > 126 MB L2), so every
  step streams from HBM.
* e2e: the same metric through the public API ``sample_tokens`` with the logits in pinned host
  memory: host->device copy of the logits and parameters, the launch, device->host tokens.
* roofline: algorithmic bytes (B*V*elem read once) per step / median step time, against the
  measured HBM copy bandwidth in MEASURED_PEAKS.json.
* cpu_baseline: the reference's own sample_token (pagedbatch.sampling, installed in baseline/_ref)
  per row on this host's cores over a bounded sample (the restated torch port if it is absent).
* extra_configs (N=1): configs 0, 1, 2-flat and 3 timed the same way, each with its CPU baseline.

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
MIN_TIMED_MS = 200.0
WORKLOADS = {"cfg0": workloads.config0, "cfg1": workloads.config1, "cfg2": workloads.config2,
             "cfg2flat": workloads.config2_flat, "cfg3": workloads.config3}


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def make_workload(name: str, rank: int):
    return WORKLOADS[name](seed=rank)


def workload_config(w) -> dict:
    """The workload description both arms print (the same dict, so their lines compare)."""
    p = w.params[0]
    dtype = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}[w.logits.dtype]
    return {"workload": w.name, "rows_per_gpu": w.rows, "vocab": w.vocab, "logits_dtype": dtype,
            "sampling": "mixed" if len({(q.temperature, q.top_k, q.top_p) for q in w.params}) > 1
            else f"T {p.temperature}, top_k {p.top_k}, top_p {p.top_p}"}


class ClockSampler:
    """nvidia-smi clock / throttle samples while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.out = ""

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


# ---- the reference's CPU implementation -------------------------------------------------------

def reference_sampler():
    """(row sampler, kind, description): the reference's own sample_token from baseline/_ref when it
    is installed there (``kind`` "reference"), else its restatement oracle/torch_port ("port")."""
    path = os.path.join(REPO, "baseline", "_ref")
    if os.path.isdir(os.path.join(path, "pagedbatch")):
        if path not in sys.path:
            sys.path.insert(0, path)
        from pagedbatch.config import SamplingParams as RefParams
        from pagedbatch.sampling import sample_token

        def f(row, t, k, p, g):
            return sample_token(row, RefParams(temperature=t, top_k=k, top_p=p), g)

        return f, "reference", "pagedbatch.sampling.sample_token (reference, baseline/_ref)"
    from oracle import torch_port

    return torch_port.sample_row, "port", "oracle/torch_port.sample_row (restated reference torch calls)"


def cpu_baseline(w, budget_s: float = 10.0, min_rows: int = 8):
    """The reference's sampler per row (as the engine calls it) over a bounded sample of the rows."""
    fn, kind, desc = reference_sampler()
    torch.set_num_threads(os.cpu_count() or 1)
    x = w.logits
    params = [(p.temperature, p.top_k, p.top_p) for p in w.params]
    done, t0 = 0, time.perf_counter()
    while True:
        r = done % w.rows
        fn(x[r], *params[r], torch.Generator().manual_seed(w.seeds[r]))
        done += 1
        el = time.perf_counter() - t0
        if done >= min_rows and el >= budget_s:
            break
    rate = done / el
    return {"value": rate, "unit": "rows/s", "cores": torch.get_num_threads(), "kind": kind,
            "sample": f"{done} rows of {w.name} in {el:.1f} s, {desc}, one call per row"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = make_workload(args.workload, 0)
    fn, kind, desc = reference_sampler()
    torch.set_num_threads(os.cpu_count() or 1)
    params = [(p.temperature, p.top_k, p.top_p) for p in w.params]
    # one timing of a few rows sizes each step's sample to keep the whole run to ~2 minutes
    t0 = time.perf_counter()
    for j in range(2):
        fn(w.logits[j], *params[j], torch.Generator().manual_seed(w.seeds[j]))
    rate = 2 / (time.perf_counter() - t0)
    per_step = max(1, min(w.rows, int(120.0 * rate / max(1, args.steps + args.warmup))))
    times = []
    for s in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        for j in range(per_step):
            r = (s * per_step + j) % w.rows
            fn(w.logits[r], *params[r], torch.Generator().manual_seed(w.seeds[r]))
        if s >= args.warmup:
            times.append(time.perf_counter() - t0)
    tot = sum(times)
    value = per_step * args.steps / tot
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(w),
        "method": {"rows_per_step_sampled": per_step, "calls": "one sample_token call per row, each with its "
                   "own seeded torch.Generator (pagedbatch/engine.py:133-139)"},
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": torch.get_num_threads(), "kind": kind,
                         "sample": f"{per_step} rows per step of {w.name}, {desc}"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- device timing helpers --------------------------------------------------------------------

def timed_graph(fn, bufs, steps: int, stream, dev, dist=None, min_ms: float = MIN_TIMED_MS, soak_ms: float = 600.0):
    """Capture `steps` calls fn(buf) in one CUDA graph, soak the GPU (so clock samples mean
    something), then replay it until `min_ms` of steps are timed, each replay between CUDA events.
    A second graph of the same calls with a timing event between calls gives the per-launch
    distribution (its event nodes cost a little time between launches, so it does not set the
    value). Returns (median replay ms, per-replay ms list, per-launch us list, clock summary)."""
    with torch.cuda.stream(stream):
        for i in range(3):
            fn(bufs[i % NROT])
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(steps):
            fn(bufs[i % NROT])
    evs = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(steps + 1)]
    g_ev = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_ev, stream=stream):
        evs[0].record(stream)
        for i in range(steps):
            fn(bufs[i % NROT])
            evs[i + 1].record(stream)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    per_replay = max(e0.elapsed_time(e1), 1e-3)
    n_soak = max(1, int(soak_ms / per_replay))
    n_timed = max(5, int(min_ms / per_replay) + 1)
    if dist:
        t = torch.tensor([n_timed], device=dev, dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)  # every rank replays as often
        n_timed = int(t.item())
    reps, launches = [], []
    rec = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_timed)]
    with ClockSampler(dev.index or 0) as clk:
        with torch.cuda.stream(stream):
            for _ in range(n_soak):
                graph.replay()
        if dist:
            dist.barrier()
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(stream):
            for a, b in rec:
                a.record(stream)
                graph.replay()
                b.record(stream)
        torch.cuda.synchronize(dev)
        if dist:
            dist.barrier()
    for a, b in rec:
        reps.append(a.elapsed_time(b))
    for _ in range(min(20, n_timed)):
        with torch.cuda.stream(stream):
            g_ev.replay()
        torch.cuda.synchronize(dev)
        launches += [evs[i].elapsed_time(evs[i + 1]) * 1e3 for i in range(steps)]
    del graph, g_ev
    return statistics.median(reps), reps, launches, clk.summary()


def pct(xs, q):
    return float(np.percentile(np.asarray(xs, dtype=np.float64), q)) if xs else None


def launches_per_step(L, logits, params) -> int:
    """Kernel launches of one sample_op on these logits (the path the ops layer takes)."""
    B, V = logits.shape
    code = ops._DTYPE_CODE[logits.dtype]
    if ops._ws_path(params, V):
        return L.pb_sample_ws_launches(logits.data_ptr(), B, V, logits.stride(0), code)
    return L.pb_sample_launches(B, V, code, 0)


def device_config_measure(w, dev, stream, steps: int):
    """One workload on one GPU: median step time and its clocks (for extra_configs)."""
    rec = sampling.pack_rows(w.params, np.array(w.uniforms()))
    params = ops.params_tensor(rec, dev)
    bufs = [w.logits.to(dev) for _ in range(NROT)]
    med, reps, launches, clocks = timed_graph(lambda b: ops.sample_op(b, params), bufs, steps, stream, dev,
                                              min_ms=100.0, soak_ms=300.0)
    B, V = w.logits.shape
    elem = w.logits.element_size()
    step_ms = med / steps
    peak, _ = load_peaks()
    L = _lib.load()
    out = {"us_per_step": step_ms * 1e3, "rows_per_s": B / (step_ms / 1e3),
           "per_launch_us": {"p50": pct(launches, 50), "p99": pct(launches, 99)},
           "hbm_frac": B * V * elem / (step_ms / 1e3) / 1e9 / peak,
           "gpu_launches_per_step": launches_per_step(L, bufs[0], params),
           "clocks": clocks, "config": workload_config(w)}
    del bufs
    torch.cuda.empty_cache()
    return out


# ---- vocabulary-parallel (config 3) ------------------------------------------------------------

def measure_vocab_parallel(world, rank, local, dist, steps: int, warmup: int):
    """Config 3 over this process group: per step, pb_candidates on this rank's column slice, one
    NCCL all-gather of the per-row records, pb_merge. Eager launches, CUDA events per phase; the
    step time is the max over ranks (strong scaling: the job is fixed as N grows)."""
    from pagedbatch_b200.vocab_parallel import CudaKernels, record_cap

    dev = torch.device("cuda", local)
    w = workloads.config3(seed=0)
    B, V = w.logits.shape
    lo, hi = V * rank // world, V * (rank + 1) // world
    xs = [w.logits[:, lo:hi].contiguous().to(dev) for _ in range(NROT)]
    xs_ptr = xs[0].data_ptr()
    rec = sampling.pack_rows(w.params, np.array(w.uniforms()))
    dparams = ops.params_tensor(rec, dev)
    cap = record_cap(w.params)
    kern = CudaKernels()
    rb = _lib.record_bytes(cap)
    gathered = torch.empty((world, B, rb), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]

    def step(i, marks=None):
        if marks:
            marks[0].record(stream)
        mine = kern.candidates(xs[i % NROT], dparams, lo, cap)
        if marks:
            marks[1].record(stream)
        if dist:
            dist.all_gather_into_tensor(gathered.view(world * B, rb), mine)
        else:
            gathered[0].copy_(mine)
        if marks:
            marks[2].record(stream)
        tok, info = kern.merge(gathered, dparams, cap)
        if marks:
            marks[3].record(stream)
        return tok, info

    for i in range(max(3, warmup)):
        tok, info = step(i)
    torch.cuda.synchronize(dev)
    fallback = int((ops.info_records(info)["status"] == _lib.ROW_FALLBACK).sum())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        # soak ~0.6 s (the same number of steps on every rank) so the clock samples mean something
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < 0.3:
            step(n)
            n += 1
            if n % 50 == 0:
                torch.cuda.synchronize(dev)
        cnt = torch.tensor([2 * n], device=dev, dtype=torch.int64)
        if dist:
            dist.all_reduce(cnt, op=dist.ReduceOp.MAX)
        for i in range(int(cnt.item()) - n):
            step(i)
        if dist:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for i in range(steps):
            step(i, ev[i])
        e1.record(stream)
        torch.cuda.synchronize(dev)
        if dist:
            dist.barrier()
    ms = e0.elapsed_time(e1)
    phases = {"candidates": [], "all_gather": [], "merge": []}
    for m in ev:
        phases["candidates"].append(m[0].elapsed_time(m[1]) * 1e3)
        phases["all_gather"].append(m[1].elapsed_time(m[2]) * 1e3)
        phases["merge"].append(m[2].elapsed_time(m[3]) * 1e3)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    step_ms = ms_max / steps
    peak, _ = load_peaks()
    shard_bytes = B * (hi - lo) * 2
    L = _lib.load()
    out = {
        "workload": w.name, "rows": B, "vocab": V, "ranks": world, "shard_vocab": hi - lo,
        "us_per_step": step_ms * 1e3, "rows_per_s": B / (step_ms / 1e3), "scaling": "strong",
        "phase_us_median_rank0": {k: statistics.median(v) for k, v in phases.items()},
        "record_bytes_per_row": rb, "all_gather_bytes_per_rank": B * rb,
        "fallback_rows": fallback,
        "shard_hbm_frac": shard_bytes / (step_ms / 1e3) / 1e9 / peak,
        "kernels": (f"pb_candidates_ws ({L.pb_sample_ws_launches(xs_ptr, B, hi - lo, hi - lo, 1)} launches)"
                    if ops._ws_path(dparams, hi - lo) else
                    f"pb_candidates ({L.pb_sample_launches(B, hi - lo, 1, 0)} launch(es))")
                   + " + NCCL all_gather_into_tensor + pb_merge (1 launch)",
        "timing": "eager launches between CUDA events, max over ranks; per-phase medians from rank 0",
        "clocks": clk.summary(),
    }
    del xs, gathered
    torch.cuda.empty_cache()
    return out


def run_vocab_parallel(args):
    """Config 3 alone (``--workload cfg3``): the vocabulary-parallel line."""
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
    vp = measure_vocab_parallel(world, rank, local, dist, args.steps, args.warmup)
    peak, peak_kind = load_peaks()
    line = {
        "metric": "vocab-parallel sampled rows/s at B=1024,V=128256 bf16 (config 3); 1/2/4/8 GPU",
        "value": vp["rows_per_s"], "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": vp["us_per_step"] / 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic", "config": {"workload": vp["workload"], "rows": vp["rows"],
                                                         "vocab": vp["vocab"]},
        "vocab_parallel": vp, "clocks": vp["clocks"], "gpu_launches": 3 * args.steps,
        "roofline": {"bound": "hbm", "achieved": vp["shard_hbm_frac"] * peak, "peak": peak, "unit": "GB/s",
                     "frac": vp["shard_hbm_frac"], "peak_source": f"{peak_kind} hbm_gbs", "traffic": None,
                     "alg_bytes_per_launch_per_rank": vp["rows"] * vp["shard_vocab"] * 2},
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# ---- config 4: the reference engine end to end ---------------------------------------------------

def _cfg4_params(RefSP, i: int, rows: int = 256):
    """Config 1's mix for request i of 256: greedy, temperature-only, top-k, top-p blocks of 64."""
    q = rows // 4
    blk, j = divmod(i, q)
    kw = dict(max_tokens=256, ignore_eos=True, seed=i)
    if blk == 0:
        return RefSP(temperature=0.0, **kw)
    if blk == 1:
        return RefSP(temperature=(0.5, 1.0, 1.5)[j % 3], **kw)
    if blk == 2:
        return RefSP(temperature=1.0, top_k=(1, 20, 100, 1000)[j % 4], **kw)
    return RefSP(temperature=1.0, top_p=(0.5, 0.9, 0.99)[j % 3], **kw)


def engine_decode_config4(dev, steps_ours: int = 48, steps_ref: int = 6) -> dict:
    """Config 4: the reference's LLMEngine (pagedbatch/engine.py) with its smollm2-135m-random model
    (random weights, bf16, CUDA), 256 sequences, prompts of uniform-random token ids with lengths
    uniform in [64, 512], 256 output tokens each (ignore_eos), block_size 16, sampling parameters
    mixed as in config 1. Every prompt is prefilled first; then `steps_ours` decode steps run with
    one batched launch per step (pagedbatch_b200.engine_hook) and `steps_ref` with the reference's
    own per-row sample_token (sampling.py:10-27), each step timed between device synchronisations.
    The sampling share is sampling time / step time (the step includes the model forward)."""
    path = os.path.join(REPO, "baseline", "_ref")
    if not os.path.isdir(os.path.join(path, "pagedbatch")):
        return {"unavailable": "reference package not installed in baseline/_ref"}
    if path not in sys.path:
        sys.path.insert(0, path)
    import pagedbatch.engine as em
    from pagedbatch.config import EngineConfig
    from pagedbatch.config import SamplingParams as RefSP
    from pagedbatch.loader import load_model

    from pagedbatch_b200 import engine_hook

    B, P_LO, P_HI = 256, 64, 512
    model, mcfg, tok = load_model("smollm2-135m-random", device=str(dev), dtype="bfloat16", seed=0)
    ecfg = EngineConfig(block_size=16, num_blocks=B * (P_HI + 256 + 16) // 16 + 64, max_num_seqs=B,
                        max_num_batched_tokens=16384, max_model_len=1024, device=str(dev), dtype="bfloat16",
                        seed=0)
    eng = em.LLMEngine(model, mcfg, tok, ecfg)
    rng = np.random.default_rng(0)
    for i in range(B):
        n = int(rng.integers(P_LO, P_HI + 1))
        eng.add_request(prompt_token_ids=rng.integers(0, mcfg.vocab_size, n).tolist(),
                        sampling=_cfg4_params(RefSP, i, B), request_id=f"r{i}")
    engine_hook.install(eng)
    t0 = time.perf_counter()
    prefill_steps = 0
    while any(not st.seq.output_token_ids for st in eng._requests.values()):
        eng.step()
        prefill_steps += 1
    torch.cuda.synchronize(dev)
    prefill_s = time.perf_counter() - t0

    for _ in range(2):  # warm-up decode steps
        eng.step()
    st_o, sp_o = [], []
    for _ in range(steps_ours):
        before = engine_hook.stats.seconds
        torch.cuda.synchronize(dev)
        a = time.perf_counter()
        eng.step()
        torch.cuda.synchronize(dev)
        st_o.append(time.perf_counter() - a)
        sp_o.append(engine_hook.stats.seconds - before)
    rows_step = len(eng._requests)
    # the reference's per-row sampler on the same engine (its own sample_token, timed per call)
    engine_hook.uninstall(eng)
    engine_hook.restore_module(em)
    ref_fn = em.sample_token
    acc = [0.0]

    def ref_timed(logits, params, generator):
        # the reference's request generators are CPU generators (engine.py:58,84), which
        # torch.multinomial refuses for CUDA probabilities (sampling.py:27): the row is copied to the
        # host first, inside the timed call, as a CUDA engine running this sampler has to
        a = time.perf_counter()
        t = ref_fn(logits.cpu(), params, generator)
        acc[0] += time.perf_counter() - a
        return t

    em.sample_token = ref_timed
    try:
        st_r, sp_r = [], []
        for _ in range(steps_ref):
            acc[0] = 0.0
            torch.cuda.synchronize(dev)
            a = time.perf_counter()
            eng.step()
            torch.cuda.synchronize(dev)
            st_r.append(time.perf_counter() - a)
            sp_r.append(acc[0])
    finally:
        em.sample_token = ref_fn
    med = statistics.median
    out = {
        "workload": "cfg4_smollm2-135m-random_bf16_256seq_decode",
        "model": "smollm2-135m-random (30 layers, hidden 576, 9 heads, 3 KV heads, vocab 49152), bf16, random weights",
        "sequences": B, "prompt_len": f"uniform [{P_LO}, {P_HI}]", "output_tokens": 256, "block_size": 16,
        "sampling": "config 1 mix (64 greedy, 64 temperature-only, 64 top-k, 64 top-p), per-request seeds",
        "prefill": {"steps": prefill_steps, "s": prefill_s},
        "rows_per_decode_step": rows_step,
        "ours": {"decode_steps": steps_ours, "step_ms": 1e3 * med(st_o), "sampling_ms": 1e3 * med(sp_o),
                 "sampling_share": med(sp_o) / med(st_o),
                 "api": "pagedbatch_b200.engine_hook.install (one sample_tokens launch per step)"},
        "reference": {"decode_steps": steps_ref, "step_ms": 1e3 * med(st_r), "sampling_ms": 1e3 * med(sp_r),
                      "sampling_share": med(sp_r) / med(st_r),
                      "api": "pagedbatch.sampling.sample_token per row (engine.py:139) on the row copied to "
                             "the host (its CPU request generators cannot drive torch.multinomial on CUDA)"},
        "timing": "host clock around each engine.step() between torch.cuda.synchronize() calls; medians",
    }
    del eng, model
    torch.cuda.empty_cache()
    return out


# ---- our arm ----------------------------------------------------------------------------------

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
    L = _lib.load()
    w = make_workload(args.workload, rank)
    B, V = w.logits.shape
    elem = w.logits.element_size()
    rec = sampling.pack_rows(w.params, np.array(w.uniforms()))
    params = ops.params_tensor(rec, dev)
    bufs = [w.logits.to(dev) for _ in range(NROT)]
    stream = torch.cuda.Stream(dev)

    # warm-up (also sets the kernels' shared-memory attributes before capture)
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

    med_ms, reps, launches, clocks = timed_graph(lambda b: ops.sample_op(b, params), bufs, args.steps, stream, dev,
                                                 dist=dist)
    t = torch.tensor([med_ms], device=dev, dtype=torch.float64)
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
    # pb_sample_ws (the default path): the balanced streaming kernel, then the cluster kernel over the
    # rows it leaves; pb_sample: 1 or 2 launches by shape
    per_step_launches = launches_per_step(L, bufs[0], params)
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "us_per_step": step_ms * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": {4: "f32", 2: "bf16"}[elem], "data": "synthetic",
        "config": workload_config(w),
        "method": {"parallelism": f"rows sharded over {world} GPU(s), no collective",
                   "l2": f"{NROT} rotating input copies ({NROT * alg_bytes / 1e6:.0f} MB > 126 MB L2)",
                   "timing": f"CUDA graph of {args.steps} steps replayed {len(reps)} times (>= {MIN_TIMED_MS:.0f} ms), "
                             "each replay between CUDA events; median replay, max over ranks"},
        "timing_stats": {"replays": len(reps), "replay_ms": {"median": med_ms, "min": min(reps), "max": max(reps)},
                         "replay_us_per_step": {"median": 1e3 * med_ms / args.steps,
                                                "p99": 1e3 * pct(reps, 99) / args.steps},
                         "per_launch_us_rank0": {"p50": pct(launches, 50), "p99": pct(launches, 99),
                                                 "min": min(launches), "max": max(launches), "n": len(launches),
                                                 "note": "from a second graph with a timing event between "
                                                         "launches (the event nodes add a little time)"}},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} hbm_gbs", "traffic": load_traffic(w.name),
                     "alg_bytes_per_launch": alg_bytes},
        "e2e": {"value": world * B / e2e_s, "unit": "rows/s", "ms_per_step": e2e_s * 1e3,
                "h2d_bytes_per_step": alg_bytes + rec.nbytes, "d2h_bytes_per_step": 8 * B,
                "api": "pagedbatch_b200.sample_tokens(pinned host logits)"},
        # pb_sample_launches: 1 (the cluster kernel) or 2 (the streaming kernel, then the cluster
        # kernel on the rows it leaves), per step of this shape
        "gpu_launches": args.steps * per_step_launches,
        "clocks": clocks,
    }
    del bufs
    torch.cuda.empty_cache()
    if world > 1:
        line["vocab_parallel"] = measure_vocab_parallel(world, rank, local, dist, args.steps, args.warmup)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(w)
    if rank == 0 and world == 1 and not args.no_extra:
        extra = {}
        for name in ("cfg0", "cfg1", "cfg2flat", "cfg3"):
            ew = make_workload(name, 0)
            extra[name] = device_config_measure(ew, dev, stream, args.steps)
            if not args.no_cpu_baseline:
                extra[name]["cpu_baseline"] = cpu_baseline(ew, budget_s=3.0, min_rows=2)
        try:
            extra["cfg4"] = engine_decode_config4(dev)
        except Exception as e:  # the line must still print; the reason is reported
            extra["cfg4"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
        line["extra_configs"] = extra
    if rank == 0:
        print(json.dumps(line), flush=True)
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
    """Plain torch reductions over the same logits, timed like the sampler: what one read-once pass
    over this tensor costs at this size on this GPU, beside the sampler itself. One JSON line, 1 GPU."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    w = make_workload(args.workload, 0)
    rec = sampling.pack_rows(w.params, np.array(w.uniforms()))
    params = ops.params_tensor(rec, dev)
    bufs = [w.logits.to(dev) for _ in range(NROT)]
    nbytes = w.logits.numel() * w.logits.element_size()
    stream = torch.cuda.Stream(dev)

    def graph_us(f):
        med, _, launches, _ = timed_graph(f, bufs, args.steps, stream, dev, min_ms=100.0, soak_ms=100.0)
        us = med * 1e3 / args.steps
        return {"us_per_launch": us, "read_GBps": nbytes / (us * 1e-6) / 1e9, "p99_launch_us": pct(launches, 99)}

    line = {
        "calibration": w.name,
        "bytes_per_launch": nbytes,
        "timing": f"CUDA graph of K launches, median replay; {NROT} rotating input copies",
        "torch_sum": graph_us(lambda a: a.sum()),
        "torch_amax_rows": graph_us(lambda a: torch.amax(a, dim=1)),
        "torch_max_argmax_rows": graph_us(lambda a: torch.max(a, dim=1)),
        "pb_sample": graph_us(lambda a: ops.sample_op(a, params)),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="cfg2", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the extra configurations (N=1)")
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
