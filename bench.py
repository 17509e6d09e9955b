#!/usr/bin/env python
"""Benchmark of the B200 token sampler (verbo's Sampler::pick, src/sampler.cpp:50-109).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

The default configuration is C4: 4096 sampled rows at V = 151936 (flat
N(0, 0.5^2) logits, temp 1.5, top_p 0.99, no top-k), the full-vocabulary
nucleus that the metric's "sampled rows/s ... 1/2/4/8 B200" is quoted on,
sharded by rows over the GPUs.  C1-C3 and C5 are selectable with --config and
are parity cases of the test suite.

Under torchrun (N > 1) every rank runs the same per-rank workload (weak
scaling: rows are independent, no collective on the data path) and rank 0
prints ONE JSON line.  A "step" is one pass of the sampler over one batch of
synthetic logits rows.

  value     sampled rows/s of the whole job, inputs resident in HBM, timed with
            CUDA events around K steps (barrier + synchronize on both sides,
            max over ranks);
  e2e       the same metric through the public call with HOST buffers: each
            step copies its rows (and histories) from pinned host memory,
            samples, and reads the ids back;
  roofline  the sampling kernel's algorithmic bytes per launch (4*V + 4*H + 4
            per row) over its average CUDA-event launch time, against the
            measured HBM copy bandwidth;
  cpu_baseline  the reference's own Sampler (compiled from its sources,
            oracle/_ref) on this host's cores, on a bounded sample of rows.

--impl reference times only that CPU reference (rank 0; other ranks exit).
The c5 configuration measures the vocab-sharded form instead: per-rank
column shard -> shard_topk -> NCCL all-gather of candidates -> merge_sample.

--config tail measures the logits producer tail instead (final RMSNorm + LM
head, src/session.cpp:163-169) on a Qwen2-0.5B-shaped Q8 head (151936 x 896,
--head q8|q4|f32), --rows hidden rows per step (default 1: one decode step);
its roofline is HBM bytes (the head, read once per call, plus the rows in and
the logits out) over the step's CUDA-event time, and its CPU baseline and
--impl reference arm are the reference's own rmsnorm + quant_act + matmul
(AVX2 build, all host threads).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from verbo_b200 import workloads as wl  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", default="c4", choices=sorted(wl.WORKLOADS) + ["tail", "decode"])
    p.add_argument("--head", default="q8", choices=["q8", "q4", "f32"], help="head dtype of --config tail")
    p.add_argument("--shard-head", action="store_true",
                   help="--config tail: tensor-parallel head (vocab rows split over the ranks), each step "
                        "tail shard -> shard top-k -> NCCL all-gather -> merge (greedy pick)")
    p.add_argument("--rows", type=int, default=0, help="rows per GPU (default: the configuration's)")
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--e2e-steps", type=int, default=0, help="steps of the host-buffer measurement (default min(K, 10))")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="budget of the CPU baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-soak", action="store_true", help="skip the 1 s load window kept for the clock record")
    p.add_argument("--no-e2e", action="store_true", help="skip the host-buffer measurement")
    p.add_argument("--no-graph", action="store_true", help="launch each timed step from the host instead of a CUDA graph")
    a = p.parse_args()
    if a.warmup < 3:
        p.error("--warmup must be >= 3")
    return a


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def measured_peak():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.is_file():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def traffic_per_row(workload: str):
    """DRAM bytes per row of the step's kernels from a committed ncu capture
    (profiles/traffic.json: {workload: {"bytes_per_row": B, "rows_captured":
    R, "source": ...}}): (bytes per row, a label saying where it comes from),
    or (None, None)."""
    f = ROOT / "profiles" / "traffic.json"
    if not f.is_file():
        return None, None
    d = json.loads(f.read_text()).get(workload)
    if d is None:
        return None, None
    return float(d["bytes_per_row"]), (f"scaled by rows from one ncu capture of {d['rows_captured']} rows "
                                       f"({d['source']})")


class Clocks:
    """nvidia-smi sampling (200 ms) of SM clocks and throttle reasons."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def rotating_copies(batch_bytes: int) -> int:
    """Input copies the timed steps rotate through, so that consecutive steps
    never find their rows in L2: at least twice L2 in total."""
    return max(1, -(-2 * L2_BYTES // batch_bytes))


def algorithmic_bytes_per_row(w: wl.Workload, cols: int | None = None) -> int:
    cols = w.vocab if cols is None else cols
    return 4 * cols + 4 * w.hist_len + 4


# ----------------------------------------------------------- CPU reference ----
# The bench line's cpu_baseline and the --impl reference arm time the CPU
# reference the same way: the same sample of rows (host_rows_for_budget), one
# untimed pass, then whole timed passes over that sample, on all host threads.
def cpu_reference_pass(w: wl.Workload, x: np.ndarray, h, off, threads: int):
    """One pass of the reference's compiled Sampler (oracle/_ref, else the C
    restatement on one thread) over the host rows `x`.  Returns (kind, threads used)."""
    from oracle import pyoracle as po

    o = po.sampling(**w.sampling_kwargs())
    seeds = w.sampler_seeds(0, x.shape[0])
    if po.ref_available():
        po.ref_sample_rows(x, o, seeds, h, off, steps=1, threads=threads)
        return "reference", threads
    po.sample_rows(x, o, po.seed_states(seeds), h, off)
    return "port", 1


def cpu_reference_rate(w: wl.Workload, x: np.ndarray, h, off, seconds: float, threads: int):
    """Rows/s of the CPU reference over the host rows `x`: one untimed pass,
    then timed passes until `seconds` elapse."""
    kind, used = cpu_reference_pass(w, x, h, off, threads)
    t0 = time.perf_counter()
    n = 0
    while True:
        cpu_reference_pass(w, x, h, off, threads)
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds or n >= 1000:
            break
    return n * x.shape[0] / dt, kind, used, n


def host_rows_for_budget(w: wl.Workload, seconds: float, threads: int, cap: int):
    """Picks a sample size for the CPU leg from a one-row calibration."""
    from oracle import pyoracle as po

    x = wl.make_rows_np(w, 1)
    h, off = wl.make_hist_np(w, 1)
    o = po.sampling(**w.sampling_kwargs())
    t0 = time.perf_counter()
    if po.ref_available():
        po.ref_sample_rows(x, o, w.sampler_seeds(0, 1), h, off, steps=1, threads=1)
    else:
        po.sample_rows(x, o, po.seed_states(w.sampler_seeds(0, 1)), h, off)
    per_row = max(time.perf_counter() - t0, 1e-5)
    eff = threads if po.ref_available() else 1
    return int(max(eff, min(cap, seconds * eff / per_row / 2)))


# ------------------------------------------------------ row-batched configs ----
def bench_rows(a, w: wl.Workload, rank: int, world: int, dev):
    import torch
    import torch.distributed as dist

    import verbo_b200 as vb

    R = a.rows or w.rows
    V = w.vocab
    opts = vb.Sampling(**w.sampling_kwargs())
    batch_bytes = R * V * 4
    copies = rotating_copies(batch_bytes)
    xs = [wl.make_rows_torch(w, R, dev, seed_offset=rank * 1000 + c) for c in range(copies)]
    h, off = wl.make_hist_torch(w, R, dev, seed_offset=rank)
    seeds = w.sampler_seeds(rank * R, R)
    st = np.array(vb.seed_states(seeds.tolist()), dtype=np.uint64)
    rng = torch.from_numpy(st.view(np.int64).copy()).to(dev)
    out = torch.empty(R, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step(i):
        vb.sample(xs[i % copies], opts, rng=rng, hist=h, hist_off=off, out=out, stream=stream)

    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(a.warmup):
            step(i)
        vb.check(stream)
        # Device-resident timing replays each step from a CUDA graph (one per
        # input copy), so host launch overhead does not gap the device work;
        # the library's scratch for this stream exists after the warm-up.
        graphs = []
        if not a.no_graph:
            for c in range(copies):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    step(c)
                graphs.append(g)
        run = (lambda i: graphs[i % copies].replay()) if graphs else step
        clocks = Clocks(torch.cuda.current_device()) if rank == 0 else None
        if clocks:
            clocks.start()
        if clocks and not a.no_soak:
            t_soak = time.perf_counter()
            i = 0
            while time.perf_counter() - t_soak < 1.0:   # >= 1 s of load around the timed region for the clock record
                run(i)
                i += 1
                if i % 64 == 0:
                    torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0.record(stream)
        for i in range(a.steps):
            ev[i][0].record(stream)
            run(i)
            ev[i][1].record(stream)
        t1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        if clocks:
            clocks.stop()
        vb.check(stream)
    elapsed = t0.elapsed_time(t1)
    launch_ms = sum(s_.elapsed_time(e_) for s_, e_ in ev) / a.steps
    red = torch.tensor([elapsed, launch_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(red, op=dist.ReduceOp.MAX)
    elapsed, launch_ms = red.tolist()
    del graphs

    res = dict(R=R, elapsed_ms=elapsed, launch_ms=launch_ms, copies=copies, batch_bytes=batch_bytes,
               launches=a.steps * kernels_per_step(w, R), clocks=clocks.summary() if clocks else None,
               graph=not a.no_graph)
    if not a.no_e2e:
        with torch.cuda.stream(stream):  # copies and sampling on one stream
            res.update(e2e_rows(a, w, R, V, xs[0], h, off, opts, rng, out, stream, world, dev))
    host_sample = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        from oracle import pyoracle as po

        thr = po.host_threads()
        n = min(R, host_rows_for_budget(w, a.cpu_seconds, thr, R))
        host_sample = (xs[0][:n].cpu().numpy(), None if h is None else h[: n * w.hist_len].cpu().numpy(),
                       None if off is None else off[: n + 1].cpu().numpy())
    return res, host_sample


def e2e_rows(a, w, R, V, x0, h, off, opts, rng, out, stream, world, dev):
    """The same metric through the public call with host buffers."""
    import torch
    import torch.distributed as dist

    import verbo_b200 as vb

    e2e_steps = a.e2e_steps or min(a.steps, 10)
    hx = torch.empty((R, V), dtype=torch.float32, pin_memory=True)
    hx.copy_(x0)
    hh = None if h is None else torch.empty(h.shape, dtype=h.dtype, pin_memory=True).copy_(h)
    ho = None if off is None else torch.empty(off.shape, dtype=off.dtype, pin_memory=True).copy_(off)
    ids_host = torch.empty(R, dtype=torch.int32, pin_memory=True)
    dx = torch.empty((R, V), dtype=torch.float32, device=dev)
    dh = None if h is None else torch.empty_like(h)
    do = None if off is None else torch.empty_like(off)
    h2d = R * V * 4 + (0 if h is None else h.numel() * 4 + off.numel() * 8)
    d2h = R * 4

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        if hh is not None:
            dh.copy_(hh, non_blocking=True)
            do.copy_(ho, non_blocking=True)
        vb.sample(dx, opts, rng=rng, hist=dh, hist_off=do, out=out, stream=stream)
        ids_host.copy_(out, non_blocking=True)

    for _ in range(2):
        e2e_step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())
    return dict(e2e_ms=e2e_ms, e2e_steps=e2e_steps, h2d=h2d, d2h=d2h)


# -------------------------------------------------- vocab-sharded config (c5) ----
def bench_sharded(a, w: wl.Workload, rank: int, world: int, dev):
    """Each rank holds V/N contiguous columns of all R rows; a step is one
    verbo_cuda_sharded_sample on the library's communicator: the shard's
    top-64 (split_kernel<emit> + merge_slices_kernel), ONE NCCL all-gather of
    the packed (value, id) candidates, merge_kernel on every rank.  Events
    between the three steps (Comm.mark_next) split every timed step into shard
    kernel / all-gather / merge; each part is the max over ranks of its mean."""
    import torch
    import torch.distributed as dist

    import verbo_b200 as vb
    from verbo_b200 import sharded

    R = a.rows or w.rows
    V = w.vocab
    if V % world:
        raise SystemExit(f"vocab {V} is not divisible by {world} ranks")
    cols = V // world
    k = 64
    opts = vb.Sampling(**w.sampling_kwargs())
    shard_w = wl.Workload(w.name, R, cols, w.dist, w.scale, w.data_seed, w.temp, w.top_k, w.top_p, w.min_p,
                          w.repeat, w.hist_len)
    batch_bytes = R * cols * 4
    copies = rotating_copies(batch_bytes)
    xs = [wl.make_rows_torch(shard_w, R, dev, seed_offset=rank * 1000 + c) for c in range(copies)]
    h, off = wl.make_hist_torch(w, R, dev, seed_offset=0)        # the same histories on every rank
    st = np.array(vb.seed_states(w.sampler_seeds(0, R).tolist()), dtype=np.uint64)
    rng = torch.from_numpy(st.view(np.int64).copy()).to(dev)
    out = torch.empty(R, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    comm = sharded.make_comm(dev.index)
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(a.steps)]
    for m in marks:
        for e in m:
            e.record(stream)   # creates the events before their handles are passed on

    def step(i, m=None):
        if m is not None:
            m[0].record(stream)
            comm.mark_next(m[1], m[2])
        comm.sample(xs[i % copies], rank * cols, V, opts, k, rng, h, off, out=out, stream=stream)
        if m is not None:
            m[3].record(stream)

    try:
        for i in range(a.warmup):
            step(i)
        comm.wait(stream, timeout_ms=60000)
        vb.check(stream)
        clocks = Clocks(torch.cuda.current_device()) if rank == 0 else None
        if clocks:
            clocks.start()
        t_soak = time.perf_counter()
        i = 0
        while not a.no_soak:   # the same number of soak steps on every rank (collectives must match)
            step(i)
            i += 1
            done = torch.tensor([1.0 if time.perf_counter() - t_soak >= 1.0 else 0.0], device=dev)
            if world > 1:
                dist.all_reduce(done, op=dist.ReduceOp.MIN)
            if done.item() > 0:
                break
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0.record(stream)
        for i in range(a.steps):
            step(i, marks[i])
        t1.record(stream)
        comm.wait(stream, timeout_ms=60000)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        if clocks:
            clocks.stop()
        vb.check(stream)
        parts = [sum(m[j].elapsed_time(m[j + 1]) for m in marks) / a.steps for j in range(3)]
        red = torch.tensor([t0.elapsed_time(t1)] + parts, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(red, op=dist.ReduceOp.MAX)
        elapsed, shard_ms, gather_ms, merge_ms = red.tolist()
        e2e = e2e_sharded(a, w, comm, xs[0], h, off, rng, opts, k, rank, cols, world, dev, stream)
    finally:
        torch.cuda.synchronize()
        comm.close()
    return dict(R=R, cols=cols, elapsed_ms=elapsed, launch_ms=shard_ms, copies=copies, batch_bytes=batch_bytes,
                launches=kernels_per_step(w, R) * a.steps, clocks=clocks.summary() if clocks else None, graph=False,
                split={"shard_kernel_ms": shard_ms, "all_gather_ms": gather_ms, "merge_ms": merge_ms,
                       "step_ms": elapsed / a.steps}, **e2e)


def e2e_sharded(a, w, comm, x, h, off, rng, opts, k, rank, cols, world, dev, stream):
    """The same step through the public API with host buffers: every rank
    copies its shard and the histories from pinned host memory, calls
    Comm.sample and reads the ids back, inside the timed region."""
    import torch
    import torch.distributed as dist

    steps = a.e2e_steps or min(a.steps, 10)
    hx = x.cpu().pin_memory()
    hh = None if h is None else h.cpu().pin_memory()
    ho = None if off is None else off.cpu().pin_memory()
    dx = torch.empty_like(x)
    ids_host = torch.empty(x.shape[0], dtype=torch.int32, pin_memory=True)
    out = torch.empty(x.shape[0], dtype=torch.int32, device=dev)
    dh = None if h is None else torch.empty_like(h)
    do = None if off is None else torch.empty_like(off)
    h2d = x.numel() * 4 + (0 if h is None else h.numel() * 4 + off.numel() * 8)
    d2h = x.shape[0] * 4

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        if hh is not None:
            dh.copy_(hh, non_blocking=True)
            do.copy_(ho, non_blocking=True)
        comm.sample(dx, rank * cols, w.vocab, opts, k, rng, dh, do, out=out, stream=stream)
        ids_host.copy_(out, non_blocking=True)

    for _ in range(2):
        e2e_step()
    comm.wait(stream, timeout_ms=60000)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        e2e_step()
    e1.record(stream)
    comm.wait(stream, timeout_ms=60000)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return dict(e2e_ms=float(ms.item()), e2e_steps=steps, h2d=h2d, d2h=d2h)


# ------------------------------------------------------------ reference arm ----
def bench_reference(a, w: wl.Workload, world: int):
    """The CPU reference as the reference arm: --warmup untimed and --steps
    timed passes over a sample of the configuration's rows, timed as the bench
    line's cpu_baseline is (cpu_reference_pass)."""
    from oracle import pyoracle as po

    threads = po.host_threads()
    per_step = min(2.0, 150.0 / (a.steps + a.warmup))
    n = min(w.rows, host_rows_for_budget(w, per_step, threads, w.rows))
    x = wl.make_rows_np(w, n)
    h, off = wl.make_hist_np(w, n)
    kind, used = "port", 1
    for _ in range(a.warmup):
        kind, used = cpu_reference_pass(w, x, h, off, threads)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        cpu_reference_pass(w, x, h, off, threads)
    dt = time.perf_counter() - t0
    value = a.steps * n / dt
    sample = f"{n} of the {w.rows} rows of {w.name}, the same rows every step"
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": dt * 1000.0 / a.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": workload_config(w, n, 1),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": used, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


METRIC = "sampled rows/s at V=151936, 1/2/4/8 B200; HBM GB/s vs ~8 TB/s peak"


def workload_config(w: wl.Workload, rows_per_gpu: int, world: int, ranks=None, **extra):
    """world: rank count the rows multiply by (1 for vocab shards, which share
    rows); ranks: GPUs of the job, for the parallelism label (default world)."""
    ranks = world if ranks is None else ranks
    d = {"workload": (f"{w.name}: {w.rows} x {w.vocab} fp32 logits ({w.dist}, scale {w.scale}), temp {w.temp}, "
                      f"top_k {w.top_k}, top_p {w.top_p}, min_p {w.min_p}, repeat {w.repeat} over {w.hist_len} ids"),
         "vocab": w.vocab, "rows_per_gpu": rows_per_gpu, "global_rows": rows_per_gpu * world,
         "history": w.hist_len, "parallelism": f"rows x{ranks}" if w.shards == 1 else f"vocab shards x{ranks}"}
    d.update(extra)
    return d


TAIL_METRIC = "logits rows/s of the final RMSNorm + LM head (V=151936, dim=896); HBM GB/s vs measured peak"


def tail_config(tw, rows_per_gpu: int, world: int) -> dict:
    return {"workload": (f"tail: {rows_per_gpu} hidden rows x {tw.dim} (N(0, {tw.scale}^2)) -> rmsnorm (eps {tw.eps}) "
                         f"-> {tw.dtype} LM head {tw.vocab} x {tw.dim} -> fp32 logits"),
            "vocab": tw.vocab, "dim": tw.dim, "head": tw.dtype, "rows_per_gpu": rows_per_gpu,
            "global_rows": rows_per_gpu * world, "parallelism": f"rows x{world}",
            "l2": f"the head ({tw.head_bytes() >> 20} MiB) is larger than L2 and is read once per step"}


def tail_alg_bytes(tw, R: int) -> int:
    """Algorithmic bytes of one tail call: the head once, the hidden rows in,
    the norm weight, the logits out."""
    return tw.head_bytes() + R * tw.dim * 4 + tw.dim * 4 + R * tw.vocab * 4


def tail_traffic(tw, R: int):
    path = ROOT / "profiles" / "traffic.json"
    if not path.exists():
        return None
    d = json.loads(path.read_text()).get(f"tail_{tw.dtype}", {})
    return d.get(f"bytes_per_call_r{R}")


def head_share(traffic, res, tw):
    """Traffic of a whole-head capture scaled to a rank's vocab rows of the
    head (the head dominates the bytes), for the sharded-head step."""
    if traffic is None or "shard_rows" not in res:
        return traffic
    return traffic * res["shard_rows"] / tw.vocab


def cpu_tail_rate(tw, q, s, norm, x, seconds: float, threads: int):
    """The reference's AVX2 tail on `x`, repeated within the time budget."""
    from oracle import pyoracle as po

    kind = "reference" if po.ref_tail_available("avx2") else "port"

    def run():
        if kind == "reference":
            po.ref_logits_tail(tw.dtype, q, s, norm, tw.eps, x, build="avx2", threads=threads)
        else:
            po.logits_tail(tw.dtype, q, s, norm, tw.eps, x)

    run()
    reps, t0 = 0, time.perf_counter()
    while True:
        run()
        reps += 1
        if time.perf_counter() - t0 > seconds or reps >= 1000:
            break
    dt = time.perf_counter() - t0
    return x.shape[0] * reps / dt, kind, threads if kind == "reference" else 1, reps


def bench_tail_sharded(a, tw, rank: int, world: int, dev):
    """Tensor-parallel head: rank r holds vocab rows shard_bounds(V, N, r) of
    the head and the same hidden rows; a step is the shard's tail, then
    verbo_cuda_sharded_sample on the library's communicator (its top-8
    candidates, one NCCL all-gather, the greedy merge), identical ids on every
    rank.  Host launches per step (the collective stays outside graphs); the
    CUDA-event window of each step covers the tail shard."""
    import torch
    import torch.distributed as dist

    import verbo_b200 as vb
    from verbo_b200 import sharded

    R = tw.rows
    q, s, norm = tw.make_head()
    lo, hi = sharded.shard_bounds(tw.vocab, world, rank)
    t = vb.Tail(tw.dtype, q[lo:hi], None if s is None else s[lo:hi], norm, tw.eps, device=dev.index)
    x = torch.from_numpy(tw.make_hidden_np(R)).to(dev)   # the same rows on every rank
    shard = torch.empty(R, hi - lo, dtype=torch.float32, device=dev)
    k = 8
    opts = vb.Sampling(temp=0.0)
    out = torch.empty(R, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    comm = sharded.make_comm(dev.index)
    ev = []

    def step(timed=False):
        if timed:
            e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            e[0].record(stream)
        t.logits(x, out=shard, stream=stream)
        if timed:
            e[1].record(stream)
            ev.append(e)
        comm.sample(shard, lo, tw.vocab, opts, k, out=out, stream=stream)

    try:
        for _ in range(a.warmup):
            step()
        comm.wait(stream, timeout_ms=60000)
        vb.check(stream)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(a.steps):
            step(timed=True)
        t1.record(stream)
        comm.wait(stream, timeout_ms=60000)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        vb.check(stream)
        red = torch.tensor([t0.elapsed_time(t1), sum(s_.elapsed_time(e_) for s_, e_ in ev) / a.steps],
                           dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(red, op=dist.ReduceOp.MAX)
    finally:
        torch.cuda.synchronize()
        comm.close()
        t.close()
    return dict(R=R, elapsed_ms=red[0].item(), launch_ms=red[1].item(), shard_rows=hi - lo, clocks=None,
                graph=False), None


def bench_tail(a, tw, rank: int, world: int, dev):
    import torch
    import torch.distributed as dist

    import verbo_b200 as vb

    if a.shard_head:
        return bench_tail_sharded(a, tw, rank, world, dev)
    R = tw.rows
    q, s, norm = tw.make_head()
    t = vb.Tail(tw.dtype, q, s, norm, tw.eps, device=dev.index)
    xh = tw.make_hidden_np(R, seed_offset=rank)
    x = torch.from_numpy(xh).to(dev)
    out = torch.empty(R, tw.vocab, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step(i=0):
        t.logits(x, out=out, stream=stream)

    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(a.warmup):
            step()
        vb.check(stream)
        graph = None
        if not a.no_graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step()
        run = (lambda i: graph.replay()) if graph is not None else step
        clocks = Clocks(torch.cuda.current_device()) if rank == 0 else None
        if clocks:
            clocks.start()
        if clocks and not a.no_soak:
            t_soak = time.perf_counter()
            i = 0
            while time.perf_counter() - t_soak < 1.0:
                run(i)
                i += 1
                if i % 64 == 0:
                    torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0.record(stream)
        for i in range(a.steps):
            ev[i][0].record(stream)
            run(i)
            ev[i][1].record(stream)
        t1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        if clocks:
            clocks.stop()
        vb.check(stream)
        del graph
        res = dict(R=R, elapsed_ms=t0.elapsed_time(t1),
                   launch_ms=sum(s_.elapsed_time(e_) for s_, e_ in ev) / a.steps,
                   clocks=clocks.summary() if clocks else None, graph=not a.no_graph)
        if not a.no_e2e:
            # through the public call with host buffers: hidden rows in, logits out
            xp = torch.from_numpy(xh).pin_memory()
            op = torch.empty(R, tw.vocab, dtype=torch.float32).pin_memory()
            n_e2e = a.e2e_steps or min(a.steps, 10)
            for _ in range(2):
                x.copy_(xp, non_blocking=True)
                step()
                op.copy_(out, non_blocking=True)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(n_e2e):
                x.copy_(xp, non_blocking=True)
                step()
                op.copy_(out, non_blocking=True)
            e1.record(stream)
            torch.cuda.synchronize()
            vb.check(stream)
            res.update(e2e_ms=e0.elapsed_time(e1), e2e_steps=n_e2e, h2d=xp.numel() * 4, d2h=op.numel() * 4)
    red = torch.tensor([res["elapsed_ms"], res["launch_ms"]], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(red, op=dist.ReduceOp.MAX)
    res["elapsed_ms"], res["launch_ms"] = red.tolist()
    host = (q, s, norm, xh) if rank == 0 and world == 1 and not a.no_cpu_baseline else None
    t.close()
    return res, host


def bench_reference_tail(a, tw, world: int):
    from oracle import pyoracle as po

    threads = po.host_threads()
    q, s, norm = tw.make_head()
    x = tw.make_hidden_np(tw.rows)
    kind = "reference" if po.ref_tail_available("avx2") else "port"

    def step():
        if kind == "reference":
            po.ref_logits_tail(tw.dtype, q, s, norm, tw.eps, x, build="avx2", threads=threads)
        else:
            po.logits_tail(tw.dtype, q, s, norm, tw.eps, x)

    for _ in range(a.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        step()
    dt = time.perf_counter() - t0
    value = a.steps * tw.rows / dt
    line = {
        "metric": TAIL_METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": dt * 1000.0 / a.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "i8/f32", "data": "synthetic", "impl": "reference",
        "config": tail_config(tw, tw.rows, 1),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads if kind == "reference" else 1,
                         "kind": kind, "sample": f"all {tw.rows} rows of the step, the same rows every step"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------- decode step (B rows) ----
DECODE_METRIC = "decoded rows/s of B concurrent generations: hidden rows (host) -> Q8 LM head -> pick + accept -> ids (host)"
DECODE_OPTS = dict(temp=0.7, top_k=40, top_p=0.9, min_p=0.0, repeat=1.1, repeat_last=64)  # the reference's defaults + a penalty
DECODE_PROMPT = 64


def decode_config(tw, rows: int, world: int) -> dict:
    return {"workload": (f"decode: {rows} generations x one step: {tw.dim}-dim hidden rows (N(0, {tw.scale}^2), host) "
                         f"-> rmsnorm -> q8 LM head {tw.vocab} x {tw.dim} -> temp 0.7, top_k 40, top_p 0.9, "
                         f"repeat 1.1 over the last 64 ids -> ids (host)"),
            "vocab": tw.vocab, "dim": tw.dim, "rows_per_gpu": rows, "global_rows": rows * world,
            "parallelism": f"rows x{world}", "entry": "verbo_cuda_batch_decode"}


def cpu_decode_rate(tw, q, s, norm, x, hist, seconds: float, threads: int):
    """The reference's decode step on the host for the same rows: its AVX2
    tail (rmsnorm, quant_act, matmul on a Pool) and its Sampler per row
    (history fed through accept), repeated within the time budget."""
    from oracle import pyoracle as po

    ref = po.ref_tail_available("avx2") and po.ref_available()
    rows = x.shape[0]
    off = np.arange(rows + 1, dtype=np.int64) * hist.shape[1]
    seeds = np.arange(1, rows + 1, dtype=np.uint64)
    o = po.sampling(**DECODE_OPTS)

    def run():
        if ref:
            lg, _, _ = po.ref_logits_tail(tw.dtype, q, s, norm, tw.eps, x, build="avx2", threads=threads)
            po.ref_sample_rows(lg, o, seeds, hist.ravel(), off, threads=threads)
        else:
            lg, _, _ = po.logits_tail(tw.dtype, q, s, norm, tw.eps, x)
            po.sample_rows(lg, o, po.seed_states(seeds), hist.ravel(), off)

    run()
    reps, t0 = 0, time.perf_counter()
    while True:
        run()
        reps += 1
        if time.perf_counter() - t0 > seconds or reps >= 1000:
            break
    dt = time.perf_counter() - t0
    return rows * reps / dt, ("reference" if ref else "port"), (threads if ref else 1), reps


def main_decode(a, rank: int, local_rank: int, world: int):
    """One decode step of B generations through verbo_cuda_batch_decode: the
    sessions' final hidden rows in host memory, the Q8 head's logits on the
    device, the pick + accept of every generation, the ids back in host
    memory - the whole call timed, per step."""
    tw = wl.TAIL.with_dtype("q8")
    B = a.rows or 64
    q, s, norm = tw.make_head()
    g = np.random.default_rng(11)
    hist = g.integers(0, tw.vocab, size=(B, DECODE_PROMPT)).astype(np.int32)
    if a.impl == "reference":
        if rank == 0:
            from oracle import pyoracle as po

            x = tw.make_hidden_np(B)
            per_step = min(2.0, 150.0 / (a.steps + a.warmup))
            rate, kind, cores, reps = cpu_decode_rate(tw, q, s, norm, x, hist, per_step * a.steps, po.host_threads())
            line = {"metric": DECODE_METRIC, "value": rate, "unit": "rows/s", "n_gpus": world, "steps": a.steps,
                    "warmup": a.warmup, "ms_per_step": B / rate * 1000.0, "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None, "dtype": "i8/f32", "data": "synthetic", "impl": "reference",
                    "config": decode_config(tw, B, 1),
                    "cpu_baseline": {"value": rate, "unit": "rows/s", "cores": cores, "kind": kind,
                                     "sample": f"the {B} rows of one step x {reps} passes"},
                    "e2e": {"value": rate, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist

    import verbo_b200 as vb

    vb.load_library()  # fails loudly if the CUDA library is missing
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    try:
        tail = vb.Tail("q8", q, s, norm, tw.eps, device=local_rank)
        batch = vb.Batch(vb.Sampling(**DECODE_OPTS), B, device=local_rank)
        for i in range(B):
            batch.reset(i, 1 + i + rank * B)
            batch.accept(i, hist[i])
        copies = 4
        xs = [torch.from_numpy(tw.make_hidden_np(B, seed_offset=rank * 16 + c)).pin_memory() for c in range(copies)]
        ids = np.empty(B, dtype=np.int32)
        stream = torch.cuda.current_stream()
        for i in range(a.warmup):
            batch.decode(tail, xs[i % copies], out=ids, cuda_stream=stream)
        vb.check(stream)
        clocks = Clocks(torch.cuda.current_device()) if rank == 0 else None
        if clocks:
            clocks.start()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(a.steps):
            batch.decode(tail, xs[i % copies], out=ids, cuda_stream=stream)  # host ids: the call waits for them
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        if clocks:
            clocks.stop()
        vb.check(stream)
        red = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(red, op=dist.ReduceOp.MAX)
        elapsed = float(red.item())
        tail.close()
        batch.close()
    finally:
        if world > 1:
            dist.destroy_process_group()
    if rank != 0:
        return
    from oracle import pyoracle as po

    peak, peak_kind = measured_peak()
    value = B * world * a.steps / (elapsed / 1000.0)
    ms = elapsed / a.steps
    # per step: the head once, the hidden rows in, the logits written by the tail and read by the pick
    alg = tw.head_bytes() + B * tw.dim * 4 + 2 * B * tw.vocab * 4
    achieved = alg / (ms / 1000.0) / 1e9
    x0 = xs[0].numpy()
    rate, kind, cores, reps = cpu_decode_rate(tw, q, s, norm, x0, hist, a.cpu_seconds, po.host_threads())
    line = {
        "metric": DECODE_METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "i8/f32", "data": "synthetic", "config": decode_config(tw, B, world),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, "traffic": None,
                     "kernel": "tail_norm_kernel + tail head kernel + the pick's kernels (whole step)",
                     "alg_bytes_per_launch": alg, "launch_ms": ms},
        "clocks": clocks.summary() if clocks else None,
        "timing": "host call per step (host hidden rows in, host ids out)",
        # per step: the tail (norm + head kernel, one fused kernel up to 8 rows), split_kernel + merge_slices_kernel
        "gpu_launches": ((1 if B <= 8 else 2) + 2) * a.steps * world,
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": B * tw.dim * 4 * world,
                "d2h_bytes_per_step": B * 4 * world},
        "cpu_baseline": {"value": rate, "unit": "rows/s", "cores": cores, "kind": kind,
                         "sample": f"the {B} rows of one step x {reps} passes"},
    }
    print(json.dumps(line), flush=True)


def main_tail(a, rank: int, local_rank: int, world: int):
    tw = wl.TAIL.with_dtype(a.head)
    if a.rows:
        tw = tw.with_rows(a.rows)
    if a.impl == "reference":
        if rank == 0:
            bench_reference_tail(a, tw, world)
        return

    import torch
    import torch.distributed as dist

    import verbo_b200 as vb

    vb.load_library()  # fails loudly if the CUDA library is missing
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    try:
        res, host = bench_tail(a, tw, rank, world, dev)
    finally:
        if world > 1:
            dist.destroy_process_group()
    if rank != 0:
        return
    peak, peak_kind = measured_peak()
    R = res["R"]
    sharded_head = "shard_rows" in res
    value = R * (1 if sharded_head else world) * a.steps / (res["elapsed_ms"] / 1000.0)
    if sharded_head:  # one rank's share: its head rows, the rows in, its logits out
        alg = (tw.head_bytes() * res["shard_rows"]) // tw.vocab + R * tw.dim * 4 + tw.dim * 4 + R * res["shard_rows"] * 4
    else:
        alg = tail_alg_bytes(tw, R)
    achieved = alg / (res["launch_ms"] / 1000.0) / 1e9
    head_kernel = "tail_head_f32_kernel" if tw.dtype == "f32" else "tail_head_q_kernel"
    cfg = tail_config(tw, R, 1 if sharded_head else world)
    if sharded_head:
        cfg.update(parallelism=f"head vocab shards x{world}", head_rows_per_gpu=res["shard_rows"],
                   step="tail shard -> verbo_cuda_sharded_sample (k 8, one NCCL all-gather, greedy merge)")
    line = {
        "metric": TAIL_METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": res["elapsed_ms"] / a.steps, "higher_is_better": True,
        "scaling": "strong" if sharded_head else "weak", "vs_baseline": None,
        "dtype": "f32" if tw.dtype == "f32" else "i8/f32", "data": "synthetic", "config": cfg,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, "traffic": head_share(tail_traffic(tw, R), res, tw),
                     "kernel": "tail_norm_kernel + " + head_kernel, "alg_bytes_per_launch": alg,
                     "launch_ms": res["launch_ms"]},
        "clocks": res["clocks"],
        "timing": "CUDA graph replay per step" if res.get("graph") else "host launch per step",
        "gpu_launches": (5 if sharded_head else 2) * a.steps * world,
    }
    if "e2e_ms" in res:
        line["e2e"] = {"value": R * world * res["e2e_steps"] / (res["e2e_ms"] / 1000.0), "unit": "rows/s",
                       "h2d_bytes_per_step": res["h2d"] * world, "d2h_bytes_per_step": res["d2h"] * world}
    else:
        line["e2e"] = None
    if host is not None:
        from oracle import pyoracle as po

        q, s, norm, xh = host
        rate, kind, cores, reps = cpu_tail_rate(tw, q, s, norm, xh, a.cpu_seconds, po.host_threads())
        line["cpu_baseline"] = {"value": rate, "unit": "rows/s", "cores": cores, "kind": kind,
                                "sample": f"the {xh.shape[0]} rows of the timed step x {reps} passes"}
    print(json.dumps(line), flush=True)


def main():
    a = parse_args()
    rank, local_rank, world = dist_env()
    if a.config == "tail":
        main_tail(a, rank, local_rank, world)
        return
    if a.config == "decode":
        main_decode(a, rank, local_rank, world)
        return
    w = wl.WORKLOADS[a.config]
    if a.rows:
        w = w.with_rows(a.rows)
    if a.impl == "reference":
        if rank == 0:
            bench_reference(a, w, world)
        return

    import torch
    import torch.distributed as dist

    import verbo_b200 as vb

    vb.load_library()  # fails loudly if the CUDA library is missing
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    try:
        if w.shards > 1:
            res = bench_sharded(a, w, rank, world, dev)
            host_sample = None
        else:
            res, host_sample = bench_rows(a, w, rank, world, dev)
    finally:
        if world > 1:
            dist.destroy_process_group()
    if rank != 0:
        return

    peak, peak_kind = measured_peak()
    R = res["R"]
    sharded = w.shards > 1
    cols = res.get("cols", w.vocab)
    rows_job = R if sharded else R * world
    value = rows_job * a.steps / (res["elapsed_ms"] / 1000.0)
    alg_launch = R * (algorithmic_bytes_per_row(w, cols) + (8 * 64 if sharded else 0))
    achieved = alg_launch / (res["launch_ms"] / 1000.0) / 1e9
    tr, tr_src = traffic_per_row(w.name)
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": res["elapsed_ms"] / a.steps, "higher_is_better": True,
        "scaling": "strong" if sharded else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(
            w, R, 1 if sharded else world, ranks=world,
            l2=("inputs larger than L2" if res["copies"] == 1 else
                f"{res['copies']} rotating input copies ({res['copies'] * res['batch_bytes'] >> 20} MiB) > L2"),
            **({"columns_per_gpu": cols} if sharded else {})),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind,
                     # per-row traffic was captured on all columns: a rank's shard reads its share
                     "traffic": None if tr is None else tr * R * cols / w.vocab,
                     "traffic_source": tr_src,
                     "kernel": (("window_kernel + " if uses_window(w) else "") + "split_kernel<emit> + merge")
                     if sharded else kernel_name(w),
                     "alg_bytes_per_launch": alg_launch, "launch_ms": res["launch_ms"]},
        "clocks": res["clocks"],
        "timing": "CUDA graph replay per step" if res.get("graph") else "host launch per step",
        "gpu_launches": res["launches"] * world,
    }
    if "split" in res:
        line["step_split"] = res["split"]
        line["config"]["step"] = ("verbo_cuda_sharded_sample: shard top-64 -> one NCCL all-gather of packed "
                                  "(value, id) candidates -> merge")
    if "e2e_ms" in res:
        line["e2e"] = {"value": rows_job * res["e2e_steps"] / (res["e2e_ms"] / 1000.0), "unit": "rows/s",
                       "h2d_bytes_per_step": res["h2d"] * world, "d2h_bytes_per_step": res["d2h"] * world}
    else:
        line["e2e"] = None
    if host_sample is not None:
        x, h, off = host_sample
        from oracle import pyoracle as po

        rate, kind, cores, reps = cpu_reference_rate(w, x, h, off, a.cpu_seconds, po.host_threads())
        line["cpu_baseline"] = {"value": rate, "unit": "rows/s", "cores": cores, "kind": kind,
                                "sample": f"{x.shape[0]} rows of the timed batch x {reps} passes"}
    print(json.dumps(line), flush=True)


def uses_window(w: wl.Workload) -> bool:
    """The split kernels' penalty windows come from window_kernel when the
    window is 1..2048 ids long (verbo_b200/csrc/kernels.cu, split_window_width)."""
    return w.repeat != 1.0 and w.hist_len > 0 and 0 < w.repeat_last <= 2048


NUC_CHUNK_ROWS = 2048  # rows per chunk of the streaming full-vocabulary path (nucleus.cu, kChunkRows)


def streaming_full_vocab(w: wl.Workload) -> bool:
    """The options the streaming full-vocabulary kernel takes (nucleus.cu,
    nucleus_eligible): top_k 0 or >= vocab, no min-p, no penalty."""
    return (w.temp > 0 and not (0 < w.top_k < w.vocab) and not (w.min_p > 0)
            and (w.repeat == 1.0 or w.hist_len == 0) and w.vocab >= 4096)


def kernels_per_step(w: wl.Workload, rows: int) -> int:
    """Kernels of this library launched by one sampling step."""
    win = 1 if uses_window(w) else 0
    if w.shards > 1:
        return 3 + win   # [window_kernel] + split_kernel<emit> + merge_slices_kernel + merge_kernel
    if streaming_full_vocab(w):
        return 4 * -(-rows // NUC_CHUNK_ROWS) + 1   # nuc_a/b/c/r_kernel per chunk + general_list_kernel
    return 1 if kernel_name(w) == "general_kernel" else 2 + win


def kernel_name(w: wl.Workload) -> str:
    win = "window_kernel + " if uses_window(w) else ""
    if w.temp <= 0:
        return win + "split_kernel<greedy> + merge_slices_kernel"
    if 0 < w.top_k < w.vocab and w.top_k <= 256:
        return win + "split_kernel<sample> + merge_slices_kernel"
    if streaming_full_vocab(w):
        return "nuc_a_kernel + nuc_b_kernel + nuc_c_kernel + nuc_r_kernel (per chunk) + general_list_kernel"
    return "general_kernel"


if __name__ == "__main__":
    main()
