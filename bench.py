#!/usr/bin/env python
"""Benchmark: DiskLLM's sampler chain on batched logits, B200.

Workload (the one the headline metric is quoted on): per GPU, a
batch of 1024 rows x vocab 256000 fp32 logits drawn flat N(0, 0.5^2), repetition penalty 1.05
over a 256-id uniform history, temperature 1.0, top-k off, top-p 0.99 (the reference's
index-order prefix), one seeded uniform per row.  A step samples the whole batch: one launch
of the fused kernel.  Inputs are 1.05 GB per GPU, larger than the 126 MB L2, so no flush is
needed between steps.  Multi-GPU: one process per GPU, rows sharded (each rank samples its
own 1024-row batch; no collective on the data path) -> weak scaling.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-extra]
    python bench.py --workload cfg1|cfg2|cfg3|cfg5 [--gpus N] ...   # one configuration alone

After the headline, the same run measures the other BASELINE configurations and adds them to the
line under "configs": 1 (one sequence, 1000 dependent decode steps in a CUDA graph), 2 (64 x
151936 with penalties, top-k 50), 3 (256 x 151936 JSON mask, index-order top-p), each with its
roofline fraction and, at N = 1, the reference's own sampler timed on the host cores; and 5,
vocabulary-sharded over the N ranks with the NCCL all-gather (strong scaling), with its step
split into candidates, all-gather and merge.  Inputs that would fit twice in L2 are preceded by
a 256 MB L2 flush outside each step's events.

Config 5 (--workload cfg5): 512 rows x vocab 262144 bf16 N(0, 2^2), 10 % of ids allowed by the
mask, repetition 1.1 over 128 ids, temperature 0.9, top-k 64, top-p 0.9; every GPU holds 1/N of
the columns of all rows.  A step: shard candidates, NCCL all-gather, merge and draw.

Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
# keep stdout to the one JSON line (NCCL prints its version banner otherwise)
os.environ.setdefault("NCCL_DEBUG", "WARN")

METRIC = "sampled rows/sec and achieved HBM GB/s vs ~8 TB/s at 1/2/4/8 B200"
ROWS, VOCAB, HIST = 1024, 256000, 256
PARAMS = dict(temperature=1.0, top_k=0, top_p=0.99, repetition=1.05)
KERNEL = "sample_rows_kernel"


def algo_bytes_per_row():
    return VOCAB * 4 + HIST * 4  # logits + history ids (no mask in this configuration)


def config_block(n):
    return {
        "workload": "cfg4_nucleus_b1024_v256000_fp32 (BASELINE config 4)",
        "rows_per_gpu": ROWS, "global_batch": ROWS * n, "vocab": VOCAB, "history": HIST,
        "params": PARAMS, "parallelism": f"row-sharded x{n} (no collective)",
        "l2_policy": "inputs larger than L2 (1.05 GB per GPU vs 126 MB L2); no flush",
    }


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic():
    """dram bytes per launch from the committed ncu summary (or None)."""
    p = os.path.join(ROOT, "profiles", f"{KERNEL}_cfg4.md")
    try:
        txt = open(p).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_launch\s*[:=]\s*([0-9.eE+]+)", txt)
    return float(m.group(1)) if m else None


# ----------------------------------------------------------------------------------------------
# clocks during the timed region (NVML polled every 20 ms)

class ClockSampler:
    def __init__(self, dev_index):
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.ok = False
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(dev_index).uuid)
            h = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                hh = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(hh)
                u = u.decode() if isinstance(u, bytes) else u
                if uuid in u:
                    h = hh
                    break
            if h is None:
                h = pynvml.nvmlDeviceGetHandleByIndex(dev_index)
            self.h, self.nv = h, pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # reported in the JSON
            self.err = str(e)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(0.02)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self._t:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok:
            return {"error": getattr(self, "err", "nvml unavailable")}
        names = {"gpu_idle": 0x1, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
                 "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
                 "hw_power_brake_slowdown": 0x80}
        seen = set()
        for _, r in self.samples:
            for k, bit in names.items():
                if r & bit:
                    seen.add(k)
        mhz = [m for m, _ in self.samples]
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": self.max_mhz,
                "samples": len(mhz), "reasons": sorted(seen)}


# ----------------------------------------------------------------------------------------------
# timing helpers for the per-configuration legs

L2_FLUSH_BYTES = 256 << 20  # twice the 126 MB L2


class L2Flush:
    """Writes a buffer twice the size of L2 between timed steps whose inputs would fit in it."""

    def __init__(self, dev):
        import torch

        self.buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.v = 0

    def __call__(self):
        self.v ^= 1
        self.buf.fill_(self.v)


def max_over_ranks(x, dev, world):
    if world == 1:
        return x
    import torch

    t = torch.tensor([x], device=dev, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def timed_steps(step, steps, dev, world, flush=None, kernel=False):
    """CUDA events around each step (an L2 flush, when given, runs before the step and outside its
    events).  Returns (mean ms per step, mean ms of the library's cluster kernel or None), each the
    max over ranks."""
    import torch

    from diskllm_b200 import capi

    stream = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in ev + kev:
        a.record(stream)
        b.record(stream)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    for i in range(steps):
        if flush is not None:
            flush()
        if kernel:
            capi.set_timing_events(*kev[i])
        ev[i][0].record(stream)
        step()
        ev[i][1].record(stream)
    if kernel:
        capi.set_timing_events(None, None)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    ms = sum(a.elapsed_time(b) for a, b in ev) / steps
    kms = sum(a.elapsed_time(b) for a, b in kev) / steps if kernel else None
    ms = max_over_ranks(ms, dev, world)
    if kernel:
        kms = max_over_ranks(kms, dev, world)
    return ms, kms


# ----------------------------------------------------------------------------------------------
# CPU baseline: DiskLLM's own sampler.c (oracle/_ref, as built) or the restated port

def host_rows(n, seed=404):
    import numpy as np

    rng = np.random.default_rng(seed)
    lg = (rng.standard_normal((n, VOCAB), dtype=np.float32) * 0.5).astype(np.float32)
    hist = [rng.integers(0, VOCAB, HIST) for _ in range(n)]
    return lg, hist


def cpu_run(lg, hist, threads):
    """one pass of the CPU implementation over the rows; returns (seconds, kind)"""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np

    import oracle as O

    if O.have_reference():
        _, secs = O.sample_reference(lg, PARAMS, hist=hist, threads=threads, stream=True)
        return secs, "reference"
    t0 = time.perf_counter()
    O.sample_restated(lg, PARAMS, np.full(lg.shape[0], 0.5, np.float32), hist=hist, threads=threads)
    return time.perf_counter() - t0, "port"


def cpu_baseline(seconds=10.0):
    threads = os.cpu_count() or 1
    lg, hist = host_rows(64)
    done, tot, kind = 0, 0.0, "port"
    while tot < seconds:
        s, kind = cpu_run(lg, hist, threads)
        done += lg.shape[0]
        tot += s
    return {"value": done / tot, "unit": "rows/s", "cores": threads, "kind": kind,
            "sample": f"{lg.shape[0]} rows of config 4 (V={VOCAB}, history {HIST}) repeated for "
                      f"{tot:.1f} s on {threads} threads (one reference sampler per thread)"}


def run_reference(args, rank, world):
    """DiskLLM's own sampler.c (oracle/_ref, as built) on the host cores, over the same
    1024-row config-4 batch the GPU arm samples per step, one reference sampler per thread."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    lg, hist = host_rows(ROWS)
    kind = "port"
    for _ in range(args.warmup):
        cpu_run(lg, hist, threads)
    tot = 0.0
    for _ in range(args.steps):
        s, kind = cpu_run(lg, hist, threads)
        tot += s
    value = ROWS * args.steps / tot
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * tot / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,0.5^2) rows)",
        "config": config_block(args.gpus),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": kind,
                         "sample": f"the full {ROWS}-row config-4 batch per step, {threads} threads"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, dev):
    line = headline_result(args, rank, world, dev)
    if not args.no_extra:
        import torch

        torch.cuda.empty_cache()
        extra = extra_configs(args, rank, world, dev)
        if rank == 0:
            line["configs"] = extra
    if rank == 0:
        print(json.dumps(line), flush=True)


def headline_result(args, rank, world, dev):
    import torch

    from diskllm_b200 import capi
    from diskllm_b200 import workloads as W

    capi.load_library()
    w = W.config4(device=dev, seed=404 + rank, rows=ROWS)
    stream = torch.cuda.current_stream(dev)
    tok = torch.empty(ROWS, dtype=torch.int32, device=dev)

    def step():
        capi.sample_batch(w.logits, w.uniforms, PARAMS, hist_ids=w.hist_ids, hist_off=w.hist_off,
                          hist_max=HIST, token=tok)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    # per-step events around the cluster kernel alone (recorded by the library on the launching
    # stream), for the roofline of the dominant kernel
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for a, b in kev:  # creates the events
        a.record(stream)
        b.record(stream)
    clocks = ClockSampler(dev.index)
    barrier()
    clocks.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        capi.set_timing_events(*kev[i])
        step()
    e1.record(stream)
    barrier()
    clocks.stop()
    capi.set_timing_events(None, None)
    ms = e0.elapsed_time(e1)
    ms_kernel = sum(a.elapsed_time(b) for a, b in kev) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps

    # end to end through the public API with host buffers: pinned host -> device copy of the
    # step's inputs, the sampler, device -> host copy of the sampled ids
    h_logits = w.logits.cpu().pin_memory()
    h_hid = w.hist_ids.cpu().pin_memory()
    h_hoff = w.hist_off.cpu().pin_memory()
    h_u = w.uniforms.cpu().pin_memory()
    h_tok = torch.empty(ROWS, dtype=torch.int32).pin_memory()
    d_logits = torch.empty_like(w.logits)
    d_hid = torch.empty_like(w.hist_ids)
    d_hoff = torch.empty_like(w.hist_off)
    d_u = torch.empty_like(w.uniforms)
    h2d = h_logits.numel() * 4 + h_hid.numel() * 4 + h_hoff.numel() * 8 + h_u.numel() * 4
    d2h = ROWS * 4

    def e2e_step():
        d_logits.copy_(h_logits, non_blocking=True)
        d_hid.copy_(h_hid, non_blocking=True)
        d_hoff.copy_(h_hoff, non_blocking=True)
        d_u.copy_(h_u, non_blocking=True)
        capi.sample_batch(d_logits, d_u, PARAMS, hist_ids=d_hid, hist_off=d_hoff, hist_max=HIST,
                          token=tok)
        h_tok.copy_(tok, non_blocking=True)

    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        e2e_step()
    barrier()
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    barrier()
    ms_e2e = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms_e2e], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms_e2e = float(t.item())
    e2e_rows_s = ROWS * world / (ms_e2e / e2e_steps / 1e3)

    del d_logits, h_logits
    w.logits = None
    if rank != 0:
        return None
    value = ROWS * world / (ms_step / 1e3)
    peak, peak_kind = measured_peak()
    achieved = ROWS * algo_bytes_per_row() / (ms_kernel / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.5^2) rows, uniform histories, Philox uniforms)",
        "config": config_block(world),
        "achieved_hbm_gbs_step": ROWS * algo_bytes_per_row() / (ms_step / 1e3) / 1e9,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak,
                     "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6650 GB/s",
                     "traffic": profiled_traffic(),
                     "algorithmic_bytes_per_launch": ROWS * algo_bytes_per_row(),
                     "kernel": KERNEL, "kernel_ms": ms_kernel},
        "e2e": {"value": e2e_rows_s, "unit": "rows/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": 2 * args.steps,  # the cluster kernel and the walk kernel per step
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(seconds=args.cpu_seconds)
    return line


CFG1_VOCAB, CFG1_STEPS, CFG1_RING = 128256, 1000, 8


def run_cfg1(args, rank, world, dev):
    line = cfg1_result(args, rank, world, dev)
    if rank == 0:
        print(json.dumps(line), flush=True)


def cfg1_result(args, rank, world, dev):
    """Config 1: one sequence, 1000 dependent steps (sample, append the id to the history the
    next step penalises), replayed as one CUDA graph.  Reported as steps (rows) per second,
    aggregated over the ranks (each rank decodes its own sequence)."""
    import numpy as np
    import torch

    from diskllm_b200 import workloads as W
    from diskllm_b200.decode import DecodeLoop

    w = W.config1(device=dev, seed=101 + rank)
    g = torch.Generator(device=dev)
    g.manual_seed(11 + rank)
    ring = w.logits.repeat(CFG1_RING, 1) + 0.05 * torch.randn(CFG1_RING, CFG1_VOCAB, generator=g, device=dev)
    u = torch.from_numpy(W.philox_uniforms(101 + rank, CFG1_STEPS)).to(dev)
    loop = DecodeLoop(ring, u, dict(w.params), w.hist_ids, cap=64 + CFG1_STEPS)
    loop.capture()
    for _ in range(args.warmup):
        loop.replay()
    stream = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    reps = max(1, args.steps // 10)
    clocks = ClockSampler(dev.index)
    torch.cuda.synchronize(dev)
    clocks.start()
    e0.record(stream)
    for _ in range(reps):
        loop.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    clocks.stop()
    us_step = max_over_ranks(e0.elapsed_time(e1) * 1e3 / (reps * CFG1_STEPS), dev, world)
    # the same steps launched one by one from the host
    e0.record(stream)
    loop.run_eager()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    us_eager = e0.elapsed_time(e1) * 1e3 / CFG1_STEPS
    # end to end: each step's logits row from pinned host memory, the id back to the host
    h_ring = ring.cpu().pin_memory()
    h_tok = torch.empty(1, dtype=torch.int32).pin_memory()
    n_e2e = 200
    loop._reset()
    e0.record(stream)
    for i in range(n_e2e):
        loop.ring[i % CFG1_RING].copy_(h_ring[i % CFG1_RING], non_blocking=True)
        loop._step(i)
        h_tok.copy_(loop.tokens[i:i + 1], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    us_e2e = max_over_ranks(e0.elapsed_time(e1) * 1e3 / n_e2e, dev, world)
    if rank != 0:
        return None
    bytes_step = CFG1_VOCAB * 4 + 64 * 4
    peak, peak_kind = measured_peak()
    line = {
        "metric": METRIC, "value": world * 1e6 / us_step, "unit": "rows/s", "n_gpus": world,
        "steps": reps * CFG1_STEPS,
        "warmup": args.warmup, "ms_per_step": us_step / 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,2.5^2) row + 20 boosted ids, ring of 8 perturbed rows, Philox uniforms)",
        "config": {"workload": "cfg1_single_row_v128256 (BASELINE config 1, latency)", "rows_per_gpu": 1,
                   "vocab": CFG1_VOCAB, "history": "64 ids, appended each step", "params": dict(w.params),
                   "parallelism": "one sequence per GPU", "us_per_step_graph": us_step,
                   "us_per_step_eager": us_eager,
                   "l2_policy": "8-row ring (4.1 MB) stays in L2: latency, not bandwidth, is measured"},
        "roofline": {"bound": "latency", "achieved": bytes_step / (us_step * 1e-6) / 1e9, "peak": peak,
                     "unit": "GB/s", "frac": bytes_step / (us_step * 1e-6) / 1e9 / peak,
                     "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6650 GB/s", "traffic": None, "kernel": "one decode step (graph replay)"},
        "e2e": {"value": world * 1e6 / us_e2e, "unit": "rows/s", "h2d_bytes_per_step": CFG1_VOCAB * 4,
                "d2h_bytes_per_step": 4},
        "gpu_launches": reps * CFG1_STEPS * 3,
        "clocks": clocks.summary(),
    }
    if not args.no_cpu and world == 1:
        # the reference's step on one host core, the same row and history
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O

        lg = w.logits.cpu().numpy()
        hist = [w.hist_ids.cpu().numpy()]
        reps_cpu, tot, kind = 0, 0.0, "port"
        while tot < args.cpu_seconds / 3:
            if O.have_reference():
                _, secs = O.sample_reference(lg, dict(w.params), hist=hist, threads=1, stream=True)
                kind = "reference"
            else:
                t0 = time.perf_counter()
                O.sample_restated(lg, dict(w.params), np.full(1, 0.5, np.float32), hist=hist, threads=1)
                secs = time.perf_counter() - t0
            tot += secs
            reps_cpu += 1
        line["cpu_baseline"] = {"value": reps_cpu / tot, "unit": "rows/s", "cores": 1, "kind": kind,
                                "sample": f"{reps_cpu} single-row config 1 steps on one core"}
    return line


CFG5_ROWS, CFG5_VOCAB, CFG5_HIST, CFG5_K = 512, 262144, 128, 64


def run_cfg5(args, rank, world, dev):
    line = cfg5_result(args, rank, world, dev)
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)


def cfg5_result(args, rank, world, dev):
    """Config 5, vocabulary-sharded over the ranks: every GPU holds 1/N of the columns of all 512
    rows; a step is the shard candidate kernel, the NCCL all-gather of the candidates and the
    merge kernel (sharded.sample_vocab_sharded).  Strong scaling."""
    import torch

    from diskllm_b200 import capi, sharded
    from diskllm_b200 import workloads as W

    capi.load_library()
    w = W.config5(device=dev, seed=505, rows=CFG5_ROWS)  # the same rows on every rank
    # --emulate-shards N on one GPU: this GPU takes shard 0 of N (candidates and merge only)
    nsh = world if world > 1 or args.emulate_shards <= 1 else args.emulate_shards
    s, e = sharded.shard_range(CFG5_VOCAB, rank, nsh)
    x = w.logits[:, s:e].contiguous()
    m = w.mask[:, s // 32:(e + 31) // 32].contiguous()
    params = dict(w.params)
    w.logits = None  # the rank keeps only its shard

    # N > 1: the NVLink peer exchange (the candidate kernel stores into every rank's buffer) unless
    # --gather nccl asks for the all-gather
    px = sharded.PeerExchange(CFG5_ROWS, CFG5_K, dev) if world > 1 and args.gather == "peer" else None

    def step():
        if px is not None:
            return px.sample(x, s, CFG5_VOCAB, w.uniforms, params, mask_shard=m, hist_ids=w.hist_ids,
                             hist_off=w.hist_off, hist_max=CFG5_HIST)
        return sharded.sample_vocab_sharded(x, s, CFG5_VOCAB, w.uniforms, params, k=CFG5_K, mask_shard=m,
                                            hist_ids=w.hist_ids, hist_off=w.hist_off, hist_max=CFG5_HIST)

    for _ in range(args.warmup):
        step()
    if args.profile_only:
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize(dev)
        return None
    shard_bytes = x.numel() * 2 + m.numel() * 4
    flush = L2Flush(dev) if shard_bytes < 2 * 126e6 else None
    steps = min(args.steps, 50)
    clocks = ClockSampler(dev.index)
    clocks.start()
    ms_step, _ = timed_steps(step, steps, dev, world, flush)
    clocks.stop()

    # the parts of a step, each timed with its own events: candidates, all-gather, merge (with the
    # peer exchange: candidates with their stores to every rank, then the merge with its wait)
    stream = torch.cuda.current_stream(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    parts = [0.0, 0.0, 0.0]
    if px is not None:
        for _ in range(steps):
            if flush is not None:
                flush()
            torch.distributed.barrier()
            px.epoch += 1
            ev[0].record(stream)
            capi.shard_candidates_peer(x, s, CFG5_VOCAB, CFG5_K, params, px.peers, px.rank, px.world, px.epoch,
                                       mask=m, hist_ids=w.hist_ids, hist_off=w.hist_off, hist_max=CFG5_HIST)
            ev[1].record(stream)
            ev[2].record(stream)
            capi.merge_sample_peer(CFG5_ROWS, px.world, CFG5_K, px.local, px.epoch, w.uniforms, params)
            ev[3].record(stream)
            torch.cuda.synchronize(dev)
            for j in range(3):
                parts[j] += ev[j].elapsed_time(ev[j + 1]) / steps
        steps_parts = 0
    else:
        steps_parts = steps
    buf, vals, ids = sharded.candidate_buffer(CFG5_ROWS, CFG5_K, dev)
    for _ in range(steps_parts):
        if flush is not None:
            flush()
        if world > 1:
            torch.distributed.barrier()
        ev[0].record(stream)
        capi.shard_candidates(x, s, CFG5_VOCAB, CFG5_K, params, mask=m, hist_ids=w.hist_ids,
                              hist_off=w.hist_off, hist_max=CFG5_HIST, out=(vals, ids))
        ev[1].record(stream)
        if world > 1:
            all_v, all_i = sharded.gather_packed(buf, CFG5_ROWS, CFG5_K)
        else:
            all_v, all_i = vals.unsqueeze(0), ids.unsqueeze(0)
        ev[2].record(stream)
        capi.merge_sample(all_v, all_i, w.uniforms, params)
        ev[3].record(stream)
        torch.cuda.synchronize(dev)
        for j in range(3):
            parts[j] += ev[j].elapsed_time(ev[j + 1]) / steps
    parts = [max_over_ranks(v, dev, world) for v in parts]

    # end to end: this GPU's shard of the logits from pinned host memory, tokens back to the host
    h_x = x.cpu().pin_memory()
    d_x = torch.empty_like(x)
    h_tok = torch.empty(CFG5_ROWS, dtype=torch.int32).pin_memory()

    def e2e_step():
        d_x.copy_(h_x, non_blocking=True)
        if px is not None:
            tok = px.sample(d_x, s, CFG5_VOCAB, w.uniforms, params, mask_shard=m, hist_ids=w.hist_ids,
                            hist_off=w.hist_off, hist_max=CFG5_HIST)
        else:
            tok = sharded.sample_vocab_sharded(d_x, s, CFG5_VOCAB, w.uniforms, params, k=CFG5_K, mask_shard=m,
                                               hist_ids=w.hist_ids, hist_off=w.hist_off, hist_max=CFG5_HIST)
        h_tok.copy_(tok, non_blocking=True)

    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        e2e_step()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms_e2e = max_over_ranks(e0.elapsed_time(e1), dev, world)
    if px is not None:
        px.close()
    if rank != 0:
        return None
    cols = e - s
    bytes_per_gpu = CFG5_ROWS * (2 * cols + (cols + 7) // 8 + CFG5_HIST * 4)
    peak, peak_kind = measured_peak()
    achieved = bytes_per_gpu / (ms_step / 1e3) / 1e9
    return {
        "metric": METRIC, "value": CFG5_ROWS / (ms_step / 1e3), "unit": "rows/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16 in, f32 arithmetic",
        "data": "synthetic (seeded N(0,2^2) bf16 rows, 10% mask, uniform histories, Philox uniforms)",
        "config": {"workload": "cfg5_vocab_parallel_b512_v262144_bf16 (BASELINE config 5)",
                   "global_batch": CFG5_ROWS, "vocab": CFG5_VOCAB, "columns_per_gpu": cols, "top_k_per_shard": CFG5_K,
                   "params": params, "parallelism": f"vocab-sharded x{world}",
                   "l2_policy": ("L2 flushed (256 MB write) before each timed step: the shard is "
                                 f"{shard_bytes / 1e6:.0f} MB") if flush is not None else
                                f"shard ({shard_bytes / 1e6:.0f} MB) larger than twice the L2; no flush"},
        "parts_ms": ({"candidates_with_peer_stores": parts[0], "merge_with_arrival_wait": parts[2]}
                     if px is not None else {"candidates": parts[0], "all_gather": parts[1], "merge": parts[2]}),
        "exchange": "NVLink peer stores from the candidate kernel" if px is not None else
                    ("NCCL all-gather" if world > 1 else "none (one GPU)"),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6650 GB/s",
                     "traffic": None, "algorithmic_bytes_per_gpu_step": bytes_per_gpu,
                     "kernel": "shard_stream_kernel + exchange + merge_sample_kernel (whole step)"},
        "e2e": {"value": CFG5_ROWS / (ms_e2e / e2e_steps / 1e3), "unit": "rows/s",
                "h2d_bytes_per_step": h_x.numel() * 2, "d2h_bytes_per_step": CFG5_ROWS * 4},
        "gpu_launches": 2 * steps,
        "clocks": clocks.summary(),
    }


def run_profile_workload(args, dev):
    """Small launches of the kernels that have no bench leg of their own, for ncu captures:
    --workload sorted: the sorted-nucleus passes (DLLM_MODE_TOPP_SORTED) on config 4's rows;
    --workload lmhead: the LM-head tail, 8 rows x hidden 4096 x vocab 128256, bf16 weights.
    Runs warm-up plus `steps` launches and prints the mean CUDA-event time per launch."""
    import torch

    from diskllm_b200 import capi
    from diskllm_b200 import workloads as W

    if args.workload == "sorted":
        w = W.config4(device=dev, rows=args.rows)

        def step():
            capi.sample_batch(w.logits, w.uniforms, w.params, hist_ids=w.hist_ids, hist_off=w.hist_off,
                              hist_max=HIST, flags=capi.MODE_TOPP_SORTED)

        desc = f"sorted-nucleus passes, {args.rows} x {VOCAB} fp32 (config 4 rows)"
    else:
        g = torch.Generator(device=dev)
        g.manual_seed(7)
        rows, hidden, vocab = 8, 4096, 128256
        h = torch.randn(rows, hidden, generator=g, device=dev)
        wt = (torch.randn(vocab, hidden, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        nw = torch.rand(hidden, generator=g, device=dev) + 0.5
        out = torch.empty(rows, vocab, device=dev)

        def step():
            capi.lmhead_logits(h, wt, norm_w=nw, logits=out)

        desc = f"LM-head tail, {rows} x {hidden} x {vocab} bf16 weights"
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    ms, _ = timed_steps(step, args.steps, dev, 1)
    print(json.dumps({"workload": desc, "ms_per_launch": ms, "steps": args.steps}), flush=True)


BATCH_SEEDS = {2: 202, 3: 303}


def batch_config_result(cfg, args, rank, world, dev):
    """Configs 2 and 3: one batch per GPU (rows sharded, no collective), a step samples it."""
    import numpy as np
    import torch

    from diskllm_b200 import capi
    from diskllm_b200 import workloads as W

    w = W.CONFIGS[cfg](device=dev, seed=BATCH_SEEDS[cfg] + rank)
    kw = {}
    if w.hist_ids is not None:
        kw.update(hist_ids=w.hist_ids, hist_off=w.hist_off, hist_max=w.hist_max)
    if w.mask is not None:
        kw["mask"] = w.mask
    tok = torch.empty(w.rows, dtype=torch.int32, device=dev)

    def step():
        capi.sample_batch(w.logits, w.uniforms, w.params, token=tok, **kw)

    for _ in range(args.warmup):
        step()
    in_bytes = w.logits.numel() * w.logits.element_size() + (0 if w.mask is None else w.mask.numel() * 4)
    flush = L2Flush(dev) if in_bytes < 2 * 126e6 else None
    steps = min(args.steps, 50)
    ms, kms = timed_steps(step, steps, dev, world, flush, kernel=True)
    if rank != 0:
        return None
    algo = w.algo_bytes_per_row * w.rows
    peak, peak_kind = measured_peak()
    res = {"workload": f"{w.name} (BASELINE config {cfg})", "rows_per_gpu": w.rows, "vocab": w.vocab,
           "params": dict(w.params), "steps": steps, "ms_per_step": ms, "value": w.rows * world / (ms / 1e3),
           "unit": "rows/s", "scaling": "weak", "algorithmic_bytes_per_step": algo,
           "achieved_gbs_step": algo / (ms / 1e3) / 1e9,
           "roofline": {"bound": "hbm", "kernel": "sample_rows_kernel", "kernel_ms": kms,
                        "achieved": algo / (kms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                        "frac": algo / (kms / 1e3) / 1e9 / peak,
                        "peak_source": "measured" if peak_kind == "measured" else "fallback"},
           "l2_policy": (f"inputs {in_bytes / 1e6:.0f} MB: L2 flushed (256 MB write) before each timed step"
                         if flush is not None else f"inputs {in_bytes / 1e6:.0f} MB, over twice the L2; no flush")}
    if world == 1 and not args.no_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O

        threads = os.cpu_count() or 1
        lg = w.logits.float().cpu().numpy()
        mask = None if w.mask is None else w.mask.cpu().numpy().view(np.uint32)
        hist = W.hist_lists(w)
        u = w.uniforms.cpu().numpy()
        done, tot, kind = 0, 0.0, "port"
        while tot < args.cpu_seconds / 3:
            if O.have_reference():
                _, secs = O.sample_reference(lg, dict(w.params), u, mask=mask, hist=hist, threads=threads)
                kind = "reference"
            else:
                t0 = time.perf_counter()
                O.sample_restated(lg, dict(w.params), u, mask=mask, hist=hist, threads=threads)
                secs = time.perf_counter() - t0
            done += w.rows
            tot += secs
        res["cpu_baseline"] = {
            "value": done / tot, "unit": "rows/s", "cores": threads, "kind": kind,
            "sample": f"the config {cfg} batch ({w.rows} rows) repeated for {tot:.1f} s on {threads} threads"
                      + ("; the reference has no frequency penalty, so its rows skip that subtraction"
                         if w.params.get("frequency", 0) else "")}
    return res


def extra_configs(args, rank, world, dev):
    """The other BASELINE configurations, run after the headline: 1 (decode latency), 2 and 3
    (row batches) and 5 (vocabulary-sharded over the ranks).  Every rank runs them in the same
    order (config 5's all-gather needs all ranks)."""
    import torch

    out = {}
    for name, fn in (("cfg1", lambda: cfg1_result(args, rank, world, dev)),
                     ("cfg2", lambda: batch_config_result(2, args, rank, world, dev)),
                     ("cfg3", lambda: batch_config_result(3, args, rank, world, dev)),
                     ("cfg5", lambda: cfg5_result(args, rank, world, dev))):
        r = fn()
        torch.cuda.empty_cache()
        if rank == 0:
            if name in ("cfg1", "cfg5"):
                keep = ("value", "unit", "ms_per_step", "scaling", "config", "roofline", "e2e", "cpu_baseline",
                        "parts_ms", "n_gpus")
                r = {k: r[k] for k in keep if k in r}
            out[name] = r
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-extra", action="store_true",
                    help="headline only: skip the configuration 1, 2, 3 and 5 legs")
    ap.add_argument("--emulate-shards", type=int, default=1,
                    help="cfg5 on one GPU: take 1 of N column shards (no all-gather)")
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                    help="cfg5 with N > 1: NVLink peer stores from the candidate kernel, or the NCCL all-gather")
    ap.add_argument("--profile-only", action="store_true",
                    help="cfg5: only warm-up and `steps` plain steps, no timing legs (for ncu captures)")
    ap.add_argument("--workload", choices=["cfg4", "cfg5", "cfg1", "cfg2", "cfg3", "sorted", "lmhead"],
                    default="cfg4",
                    help="cfg4: the headline row-sharded batch; cfg5: vocabulary-sharded config 5; "
                         "cfg1: one-sequence decode latency (CUDA graph)")
    ap.add_argument("--rows", type=int, default=ROWS,
                    help="rows per GPU (default: config 4's 1024; smaller only for profiling captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.rows != ROWS:
        globals()["ROWS"] = args.rows
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        torch.distributed.init_process_group("nccl", device_id=dev)
    try:
        if args.workload in ("sorted", "lmhead"):
            run_profile_workload(args, dev)
        elif args.workload == "cfg5":
            run_cfg5(args, rank, world, dev)
        elif args.workload == "cfg1":
            run_cfg1(args, rank, world, dev)
        elif args.workload in ("cfg2", "cfg3"):
            r = batch_config_result(int(args.workload[-1]), args, rank, world, dev)
            if rank == 0:
                print(json.dumps(r), flush=True)
        else:
            run_ours(args, rank, world, dev)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
