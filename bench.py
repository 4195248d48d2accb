#!/usr/bin/env python3
"""Benchmark of the B200 LoRA-linear hot path (one JSON line on rank 0).

Workload (default, config C5): the six LoRA-adapted projections of a Wan-style
video DiT block -- q, k, v, o (5120->5120), FFN up (5120->13824) and FFN down
(13824->5120) -- over a batch of M = 32760 tokens, each projection carrying a
weighted stack of three LoRAs (r = 32, 64, 128 with weights 1.0, 0.7, 0.4)
stacked into one rank-224 sidecar exactly as attach_fused_lora does.  bf16,
seeded Gaussian inputs generated on the device.  A step is one pass over all
six projections.

scaling strong (default): the 32760 tokens are split into contiguous shards,
        one per GPU (4095 each at N = 8), with W and the adapters replicated;
        no data-path collective.  The optional NCCL all-gather of the outputs
        into full [32760, N] tensors on every rank is timed separately
        (``allgather``), and with N > 1 a weak-scaling figure (every rank its
        own 32760 tokens) is reported beside the headline (``weak``).
value   whole-job TFLOP/s: algorithmic FLOPs of the step / max-over-ranks
        device time, inputs resident in HBM.  Every input tensor is larger
        than the 126 MB L2 at N = 1 (x >= 335 MB per projection), and each
        step streams 5.2 GB of activations, so no flush is needed.
parity  the last timed step's six outputs, sampled rows against the float64
        oracle (the bf16 bars), reported per run.
e2e     the same FLOPs through the public module API (three attach_fused_lora
        calls per projection, then FusedLoRALinear.forward) from pinned HOST
        buffers: each step copies every projection's activations in on one
        stream and its outputs out on another, so H2D(i+1), compute(i) and
        D2H(i-1) overlap; reported beside the measured bidirectional copy
        bound of the same bytes.
configs (N = 1) C1-C4 measured against their own rooflines, with parity.

--impl reference times the reference's CPU path (F.linear + two mm in fp32,
fused_linear.py:376-378, restated in oracle/) on the host cores instead.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fused LoRA-linear TFLOP/s & tokens/s per B200 (1/2/4/8 GPU), % of roofline"
WORKLOAD = ("C5 Wan DiT block projections (q,k,v,o 5120->5120; ffn 5120->13824->5120) with 3-LoRA stack "
            "r=32/64/128 (w 1.0/0.7/0.4) -> r224")
M_TOKENS = 32760
CPU_SAMPLE_TOKENS = 4096
# DRAM read + write of one fused-GEMM launch (C5 q projection), from the full
# ncu capture at M = 16384 committed under profiles/, scaled linearly to M:
# 822.1 MB read + 151.3 MB write per launch at M = 16384 (CTA-pair kernel, 256x512 tiles).
NCU_TRAFFIC_Q_16384 = 973.4e6
L2_BYTES = 126e6


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--scaling", default="strong", choices=["weak", "strong"])
    p.add_argument("--tokens", type=int, default=M_TOKENS)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-parity", action="store_true")
    p.add_argument("--no-configs", action="store_true", help="skip the C1-C4 entries of the N=1 line")
    p.add_argument("--workload", default="c5", choices=["c1", "c2", "c3", "c4", "c5", "gate"],
                   help="c5 is the headline; c1-c4 (and gate: plain GEMM vs cuBLAS) alone print one line each")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def _peaks():
    try:
        return json.load(open(ROOT / "MEASURED_PEAKS.json"))
    except (OSError, ValueError):
        return {}


# ------------------------------------------------------------------ CPU baseline
def cpu_baseline(steps: int = 1, tokens: int = CPU_SAMPLE_TOKENS, warmup: int = 1):
    """Reference CPU path on a bounded sample: `tokens` rows of each C5 projection, fp32;
    `warmup` untimed passes over the six projections, then `steps` timed ones."""
    import torch

    from oracle import lora_oracle as orc
    from probe_b200 import workloads

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    projs = workloads.c5(device="cpu", dtype=torch.float32, m=tokens)
    flops = sum(p.flops() for p in projs)
    for _ in range(max(warmup, 1)):  # untimed passes
        for p in projs:
            orc.naive_linear_torch(p.x, p.w, None, p.a, p.b, p.scale)
    times = []
    for _ in range(max(steps, 1)):
        t0 = time.perf_counter()
        for p in projs:
            orc.naive_linear_torch(p.x, p.w, None, p.a, p.b, p.scale)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    cpu_model = ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                cpu_model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {
        "value": flops / t / 1e12,
        "unit": "TFLOP/s",
        "cores": cores,
        "kind": "port",
        "sample": f"{tokens} of {M_TOKENS} tokens of each of the 6 C5 projections, fp32, "
                  f"torch F.linear + 2 mm (the reference's _torch_naive CPU path); median of {len(times)}",
        "seconds_per_sample": t,
        "cpu_model": cpu_model,
    }


# ---------------------------------------------------------------------- clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.skip = 0
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"lora_b200_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def _rows(self):
        rows = []
        try:
            for line in open(self.path):
                parts = [s.strip() for s in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except OSError:
            pass
        return rows

    def wait_first(self, timeout: float = 5.0):
        """Block until nvidia-smi has written its first sample (it can take
        longer to start than a short timed region lasts); samples taken before
        this point are left out of the statistics."""
        self.skip = 0
        if self.proc is None:
            return
        t0 = time.time()
        while time.time() - t0 < timeout:
            n = len(self._rows())
            if n:
                self.skip = n
                return
            time.sleep(0.02)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = self._rows()
        try:
            self.path.unlink()
        except OSError:
            pass
        if len(rows) > self.skip:
            rows = rows[self.skip:]  # the samples taken during the timed region
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ C5 (headline)
def _c5_runners(projs):
    from probe_b200.fused_linear import _KConcat

    return [_KConcat(p.w, p.bias, p.a, p.b, p.scale) for p in projs]


def _time_c5(projs, runners, outs, steps, warmup, world, dist, sample_clocks=None):
    """Device time of ``steps`` C5 steps (max over ranks) and of the fused-GEMM launches in them."""
    import torch

    from probe_b200 import kernels

    def step(events=None):
        for i, (p, run) in enumerate(zip(projs, runners)):
            # r = 224 > 128: the shrink is itself a tcgen05 GEMM writing [hi | lo] of s.z
            z = run.shrink(p.x)
            if events is not None:
                events[i][0].record()
            # the fused GEMM: x.W^T with the LoRA expand as an extra K-slice
            kernels.gemm(p.x, run.weight, z, run.b_dup, rank=run.tail, bias=run.bias, out=outs[i])
            if events is not None:
                events[i][1].record()

    for _ in range(max(warmup, 3)):
        step()
    torch.cuda.synchronize()
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in projs]
          for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sample_clocks is not None:
        sample_clocks.start()
        sample_clocks.wait_first()
    start.record()
    for s in range(steps):
        step(ev[s])
    end.record()
    torch.cuda.synchronize()
    clock_info = sample_clocks.stop() if sample_clocks is not None else None
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    gemm_ms = sum(a.elapsed_time(b) for row in ev for a, b in row)
    dev = projs[0].x.device
    t = torch.tensor([ms, gemm_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0]) / steps, float(t[1]) / steps, clock_info


def _c5_parity(projs, outs, world, dist):
    """Sampled rows of the last step's outputs against the oracle (max over ranks)."""
    import torch

    from oracle import checks
    from oracle import lora_oracle as orc

    worst = {"max_abs_excess": 0.0, "rel_fro": 0.0, "rows_checked": 0, "failed": 0}
    for i, (p, o) in enumerate(zip(projs, outs)):
        if p.m == 0:
            continue
        a64, b64, scale = orc.stack_adapters(
            [(checks.np64(d), checks.np64(u), al) for d, u, al in p.adapters], dtype="bf16")
        rep = checks.linear_report(o, p.x, p.w, None, a64, b64, scale, n_random=24, seed=i, full_checks=False)
        worst["max_abs_excess"] = max(worst["max_abs_excess"], rep["max_abs_excess"])
        worst["rel_fro"] = max(worst["rel_fro"], rep["rel_fro"])
        worst["rows_checked"] += rep["rows_checked"]
        worst["failed"] += 0 if rep["ok"] else 1
    dev = projs[0].x.device
    t = torch.tensor([worst["max_abs_excess"], worst["rel_fro"], worst["failed"]], device=dev, dtype=torch.float64)
    n = torch.tensor([worst["rows_checked"]], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(n, op=dist.ReduceOp.SUM)
    return {"what": "sampled rows (first, last, tile edges, 24 random) of each of the six outputs of the last "
                    "timed step against the float64 oracle on the same bf16 inputs and stacked factors",
            "rows_checked": int(n[0]), "max_abs_excess": float(t[0]), "rel_fro": float(t[1]),
            "bars": {"max_abs_excess": 2e-2, "rel_fro": 5e-3}, "ok": bool(t[2] == 0 and t[0] <= 2e-2 and t[1] <= 5e-3)}


def _time_allgather(outs, total, world, dist):
    """All-gather every projection's output shard into a full [total, N] tensor on
    every rank (sharding.gather_rows: all_gather_into_tensor, NCCL over NVLink)."""
    import torch

    from probe_b200.sharding import gather_rows

    full = [gather_rows(o, total) for o in outs]  # warm-up (and the buffers' first allocation)
    nbytes = sum(f.numel() * f.element_size() for f in full)
    del full
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    a.record()
    for _ in range(reps):
        full = [gather_rows(o, total) for o in outs]
        del full
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / reps], device=outs[0].device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    return {"ms_per_step": round(ms, 4), "bytes_per_rank": nbytes,
            "algbw_gbs": round(nbytes / ms / 1e6, 1), "busbw_gbs": round(nbytes * (world - 1) / world / ms / 1e6, 1),
            "note": "all_gather_into_tensor of the six [tokens/N, N] bf16 outputs into full outputs on every rank; "
                    "outside the headline timing"}


def _copy_bound(host_x, host_out, dev_x, dev_out, dev, world=1, dist=None):
    """Device time of copying the step's inputs in and outputs out at the same
    time (two streams, pinned host memory): the e2e step's lower bound."""
    import torch

    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    main = torch.cuda.current_stream(dev)
    times = []
    for _ in range(3):
        if world > 1:  # every rank copies at once, as in the e2e steps
            torch.cuda.synchronize()
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(main)
        h2d_s.wait_stream(main)
        d2h_s.wait_stream(main)
        with torch.cuda.stream(h2d_s):
            for hx, dx in zip(host_x, dev_x):
                dx.copy_(hx, non_blocking=True)
        with torch.cuda.stream(d2h_s):
            for ho, do in zip(host_out, dev_out):
                ho.copy_(do, non_blocking=True)
        main.wait_stream(h2d_s)
        main.wait_stream(d2h_s)
        b.record(main)
        b.synchronize()
        times.append(a.elapsed_time(b))
    return min(times)


def _e2e(projs, steps, world, dist, dev):
    """The C5 step through the public module API from pinned host buffers."""
    import torch

    from probe_b200.runtime_lora import attach_fused_lora

    holder = torch.nn.Module()
    for i, p in enumerate(projs):
        lin = torch.nn.Linear(p.k, p.n, bias=False, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(p.w)
        holder.add_module(f"p{i}", lin)
        for down, up, alpha in p.adapters:  # three adapters stacked by the public API
            attach_fused_lora(holder, f"p{i}", down, up, alpha=alpha)
    mods = [getattr(holder, f"p{i}") for i in range(len(projs))]
    host_x = [p.x.cpu().pin_memory() for p in projs]
    host_out = [torch.empty((p.m, p.n), dtype=torch.bfloat16, pin_memory=True) for p in projs]
    dev_x = [[torch.empty_like(p.x) for p in projs] for _ in range(2)]  # double-buffered inputs
    h2d_bytes = sum(x.numel() * x.element_size() for x in host_x)
    d2h_bytes = sum(o.numel() * o.element_size() for o in host_out)
    compute = torch.cuda.current_stream(dev)
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    consumed = [[None] * len(projs) for _ in range(2)]

    def e2e_step(s):
        buf = dev_x[s % 2]
        ready = []
        with torch.cuda.stream(h2d_s):
            for i in range(len(projs)):
                if consumed[s % 2][i] is not None:  # the step two back has finished reading this buffer
                    h2d_s.wait_event(consumed[s % 2][i])
                buf[i].copy_(host_x[i], non_blocking=True)
                e = torch.cuda.Event()
                e.record(h2d_s)
                ready.append(e)
        for i, mod in enumerate(mods):
            compute.wait_event(ready[i])
            y = mod(buf[i])
            done = torch.cuda.Event()
            done.record(compute)
            consumed[s % 2][i] = done
            d2h_s.wait_event(done)
            with torch.cuda.stream(d2h_s):
                host_out[i].copy_(y, non_blocking=True)
            y.record_stream(d2h_s)

    with torch.no_grad():
        for s in range(2):
            e2e_step(s)
        torch.cuda.synchronize()
        bound_ms = _copy_bound(host_x, host_out, dev_x[0], [torch.empty((p.m, p.n), device=dev,
                                                                       dtype=torch.bfloat16) for p in projs], dev,
                               world, dist)
        if world > 1:
            dist.barrier()
        e_steps = max(1, min(steps, 5))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(compute)
        h2d_s.wait_stream(compute)
        for s in range(e_steps):
            e2e_step(s)
        compute.wait_stream(d2h_s)
        compute.wait_stream(h2d_s)
        e1.record(compute)
        torch.cuda.synchronize()
        tt = torch.tensor([e0.elapsed_time(e1) / e_steps, bound_ms], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    return {"ms_per_step": float(tt[0]), "copy_bound_ms": float(tt[1]), "h2d": h2d_bytes, "d2h": d2h_bytes,
            "steps": e_steps}


def run_gpu(args):
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from probe_b200 import _lib, workloads
    from probe_b200.sharding import shard_rows

    _lib.load()
    total = args.tokens
    if args.scaling == "strong":
        lo, hi = shard_rows(total, world, rank)
    else:
        lo, hi = 0, total
    m = hi - lo
    projs = workloads.c5(device=dev, dtype=torch.bfloat16, m=total, rows=(lo, hi))
    runners = _c5_runners(projs)
    outs = [torch.empty((p.m, p.n), device=dev, dtype=torch.bfloat16) for p in projs]
    flops_local = sum(p.flops() for p in projs)
    gemm_flops = sum(2.0 * p.m * p.k * p.n + 2.0 * p.m * p.r * p.n for p in projs)  # algorithmic (rank r)
    launches_per_step = 2 * len(projs)  # shrink GEMM + fused GEMM per projection
    x_min_mb = min(p.m * p.k * 2 for p in projs) / 1e6
    stream_gb = sum(p.m * (p.k + p.n) * 2 for p in projs) / 1e9  # activations read + written per step

    clocks = ClockSampler(local)
    ms_step, gemm_ms_step, clock_info = _time_c5(projs, runners, outs, args.steps, args.warmup, world, dist, clocks)
    err = _lib.device_error(local)
    parity = None if args.no_parity else _c5_parity(projs, outs, world, dist)

    allgather = None
    if world > 1 and args.scaling == "strong":
        allgather = _time_allgather(outs, total, world, dist)

    e2e = None
    if not args.no_e2e:
        e = _e2e(projs, args.steps, world, dist, dev)
        job_flops = workloads.c5_flops(total) if args.scaling == "strong" else flops_local * world
        e2e = {"value": round(job_flops / (e["ms_per_step"] * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
               "h2d_bytes_per_step": e["h2d"], "d2h_bytes_per_step": e["d2h"],
               "ms_per_step": round(e["ms_per_step"], 3), "steps": e["steps"],
               "copy_bound_ms": round(e["copy_bound_ms"], 3),
               "frac_of_copy_bound": round(e["copy_bound_ms"] / e["ms_per_step"], 4),
               "path": "3x attach_fused_lora -> FusedLoRALinear.forward per projection; pinned host in/out; "
                       "H2D on one stream, D2H on another, double-buffered inputs",
               "copy_bound_note": "device time of copying the same H2D and D2H bytes concurrently, no compute"}
        del e

    weak = None
    if world > 1 and args.scaling == "strong":
        del runners, outs
        projs = workloads.c5(device=dev, dtype=torch.bfloat16, m=total)
        runners = _c5_runners(projs)
        outs = [torch.empty((p.m, p.n), device=dev, dtype=torch.bfloat16) for p in projs]
        w_ms, _, _ = _time_c5(projs, runners, outs, max(5, args.steps // 2), 3, world, dist)
        weak = {"value": round(workloads.c5_flops(total) * world / (w_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "ms_per_step": round(w_ms, 4), "tokens_per_gpu": total,
                "note": "every rank its own 32760-token batch (weights replicated), same kernels"}
        del runners, outs, projs

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    job_flops = workloads.c5_flops(total) if args.scaling == "strong" else flops_local * world
    job_tokens = total if args.scaling == "strong" else total * world
    value = job_flops / (ms_step * 1e-3) / 1e12
    peaks = _peaks()
    peak = peaks.get("bf16_tflops_sustained")
    peak_src = "measured sustained (MEASURED_PEAKS.json)"
    if peak is None:
        peak, peak_src = 1400.0, "fallback sustained"
    gemm_achieved = gemm_flops / (gemm_ms_step * 1e-3) / 1e12
    traffic = round(NCU_TRAFFIC_Q_16384 * m / 16384)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "tokens_per_s": round(job_tokens / (ms_step * 1e-3), 1),
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded Gaussian, generated on device; no public dataset)",
        "config": {"workload": WORKLOAD, "tokens_per_gpu": m, "global_tokens": job_tokens, "lora_rank": 224,
                   "parallelism": (f"token-sharded x{world} (contiguous shards of the {total}-token batch)"
                                   if args.scaling == "strong" else f"x{world} replicas of the {total}-token batch")
                   + ", weights+adapters replicated, no data-path collective",
                   "l2": (f"x >= {x_min_mb:.0f} MB per projection, {stream_gb:.2f} GB of activations streamed "
                          f"per step (> 126 MB L2 between reuses of any input); no flush")},
        "roofline": {"bound": "tensor",
                     "kernel": "gemm_tc2_kernel (CTA pair, tcgen05 cta_group::2) fused base + LoRA K-slice",
                     "achieved": round(gemm_achieved, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(gemm_achieved / peak, 4), "peak_source": peak_src, "traffic": traffic,
                     "traffic_note": "bytes per q-projection launch (ncu capture at M=16384, scaled to M); "
                                     "algorithmic bytes of that launch: "
                                     f"{round(2 * (m * 5120 * 2 + 5120 * 5120 + 448 * (m + 5120)))}",
                     "flops_per_step_per_gpu": gemm_flops, "gemm_ms_per_step": round(gemm_ms_step, 4)},
        "gpu_launches": launches_per_step * args.steps,
        "device_error": err,
    }
    if parity is not None:
        line["parity"] = parity
    if clock_info is not None:
        line["clocks"] = clock_info
    if e2e is not None:
        line["e2e"] = e2e
    if allgather is not None:
        line["allgather"] = allgather
    if weak is not None:
        line["weak"] = weak
    if world == 1 and not args.no_configs:
        line["configs"] = measure_configs(steps=10)
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(steps=5)
    print(json.dumps(line), flush=True)


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    cb = cpu_baseline(steps=max(args.steps, 1), warmup=max(args.warmup, 1))
    line = {
        "metric": METRIC,
        "impl": "reference",
        "value": round(cb["value"], 4),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": max(args.steps, 1),
        "warmup": max(args.warmup, 1),
        "ms_per_step": round(cb["seconds_per_sample"] * 1e3, 2),
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded Gaussian)",
        "config": {"workload": WORKLOAD, "tokens_per_gpu": CPU_SAMPLE_TOKENS,
                   "parallelism": "host CPU, all cores (rank 0 only)"},
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": round(cb["value"], 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------- other configs (C1-C4)
def _time_flushed(fn, iters, dev):
    """Median device time (ms) of fn, each run from a cold L2 (a 512 MB write in between).

    fn is captured once in a CUDA graph, so the time is the kernels' own, not
    the host's launch overhead."""
    import torch

    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    side = torch.cuda.Stream(dev)  # warm up on the capture stream: per-stream workspaces exist before capture
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        fn()
    times = []
    for _ in range(iters):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    del g
    return statistics.median(times)


def _time_chain(fns, iters, dev, launches=20):
    """Device time (ms) per call inside a CUDA graph of ``launches`` chained calls.

    ``fns`` are the same call over distinct copies of the inputs; the chain
    cycles through them, so each call's inputs were last touched
    ``len(fns) - 1`` calls earlier.  With the copies together well above the
    126 MB L2 every call reads its operands from HBM, and the graph-launch
    floor (about 6 us per replay) is spread over the whole chain.  Median over
    ``iters`` replays."""
    return _time_chains([fns], iters, dev, launches)[0]


def _time_chains(fn_lists, iters, dev, launches=20):
    """``_time_chain`` for several calls compared with one another: one graph per
    entry of ``fn_lists``, their replays interleaved (A B A B ...), so that the
    clock and power state of the part (which drifts after a heavy shape under the
    power cap) is shared by every arm instead of favouring whichever ran last."""
    import torch

    side = torch.cuda.Stream(dev)  # warm up on the capture stream: per-stream workspaces exist before capture
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for fns in fn_lists:
            for f in fns:
                f()
    torch.cuda.synchronize()
    graphs = []
    for fns in fn_lists:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for i in range(launches):
                fns[i % len(fns)]()
        graphs.append(g)
    for _ in range(3):
        for g in graphs:
            g.replay()
    torch.cuda.synchronize()
    times = [[] for _ in graphs]
    for _ in range(iters):
        for g, ts in zip(graphs, times):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b) / launches)
    del graphs
    return [statistics.median(ts) for ts in times]


def _copies_for(nbytes, floor=3, l2_multiple=3.0):
    """Copies of a working set of ``nbytes`` needed to exceed ``l2_multiple`` x L2."""
    return max(floor, int(math.ceil(l2_multiple * L2_BYTES / max(nbytes, 1))) + 1)


CHAIN_NOTE = ("ms: median per call of a 20-call CUDA-graph chain cycling through input copies (> 3x L2 "
              "between reuses, so operands come from HBM); ms_single: one call per replay after a 512 MB flush "
              "(includes the ~6 us replay floor)")


def _config_c1_c2(name, steps):
    import torch

    from oracle import checks
    from probe_b200 import workloads
    from probe_b200.fused_linear import fused_lora_linear

    dev = torch.device("cuda", 0)
    peaks = _peaks()
    hbm, tc = peaks.get("hbm_gbs", 6650.0), peaks.get("bf16_tflops", 1590.0)
    bf = torch.bfloat16
    cases = [workloads.c1(device="cpu")] if name == "c1" else [workloads.c2(m, device="cpu") for m in (1, 4, 16, 64)]
    rows = []
    for p in cases:
        flops, nbytes = p.flops(), p.bytes()
        copies = []
        for _ in range(_copies_for(nbytes)):
            copies.append(tuple(t.to(dev, bf) for t in (p.x, p.w, p.a, p.b)))
        fns = [lambda c=c: fused_lora_linear(c[0], c[1], None, c[2], c[3], p.scale) for c in copies]
        ms = _time_chain(fns, max(steps, 10), dev)
        ms1 = _time_flushed(fns[0], max(steps, 20), dev)
        x, w, a, b = copies[0]
        rep = checks.linear_report(fused_lora_linear(x, w, None, a, b, p.scale), x, w, None, a, b, p.scale,
                                   full_checks=False)
        gbs = nbytes / ms / 1e6
        rows.append({"m": p.m, "ms": round(ms, 5), "ms_single": round(ms1, 5), "tflops": round(flops / ms / 1e9, 2),
                     "gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4),
                     "t_star_us": round(max(flops / tc / 1e12, nbytes / hbm / 1e9) * 1e6, 2), "copies": len(fns),
                     "parity": {k: rep[k] for k in ("rows_checked", "max_abs_excess", "rel_fro", "ok")}})
        del fns, copies
        torch.cuda.empty_cache()
    return {"workload": "C1 single fused LoRA linear 256x4096x4096 r16" if name == "c1"
            else "C2 decode LoRA linear M in {1,4,16,64}, W 11008x4096, r16",
            "path": "fused_lora_linear (public API)", "bound": "hbm", "unit": "GB/s", "peak": hbm,
            "cases": rows, "timing": CHAIN_NOTE}


def _config_c3(steps):
    import torch

    from oracle import checks
    from probe_b200 import kernels, segmented_branch, workloads

    dev = torch.device("cuda", 0)
    peaks = _peaks()
    hbm = peaks.get("hbm_gbs", 6650.0)
    bf = torch.bfloat16
    c = workloads.c3(device="cpu", dtype=bf)
    flops, nbytes = c.branch_flops(), c.branch_bytes()
    w = c.w.to(dev)
    copies = []
    for _ in range(_copies_for(nbytes)):
        x = c.x.to(dev)
        y = kernels.gemm(x, w)
        tabs = [t.to(dev) for t in (c.a_flat, c.b_flat, c.offsets, c.ranks, c.seg_start, c.seg_adapter)]
        copies.append((x, y, tabs))
    fns = [lambda x=x, y=y, tabs=tabs: segmented_branch.segmented_branch_varlen(x, y, *tabs, c.r_max)
           for x, y, tabs in copies]
    ms = _time_chain(fns, max(steps, 10), dev)
    ms1 = _time_flushed(fns[0], max(steps, 20), dev)
    x, y, tabs = copies[0]
    out = fns[0]()
    rep = checks.branch_report(out, x, y, tabs[0], tabs[1], c.offsets, c.ranks, c.token_ids())
    gbs = nbytes / ms / 1e6
    # The same batch with its base linear: base GEMM then the branch, against the
    # fused kernel (base and adapters in one GEMM).
    unfused = [lambda x=x, tabs=tabs: segmented_branch.segmented_branch_varlen(x, kernels.gemm(x, w), *tabs, c.r_max)
               for x, _, tabs in copies]
    fused = [lambda x=x, tabs=tabs: segmented_branch.segmented_linear_varlen(x, w, None, *tabs, c.r_max)
             for x, _, tabs in copies]
    ms_unfused, ms_fused = _time_chains([unfused, fused], max(steps, 10), dev)
    got = fused[0]()
    rep_f = checks.seg_linear_report(got, x, w, None, tabs[0], tabs[1], c.offsets, c.ranks, c.token_ids())
    flops_f = flops + 2.0 * c.x.shape[0] * c.x.shape[1] * c.w.shape[0]
    sus = peaks.get("bf16_tflops_sustained", 1400.0)
    del fns, copies, unfused, fused
    torch.cuda.empty_cache()
    return {"workload": "C3 segmented multi-LoRA branch: 4096 tokens, 128 Zipf(1.1) segments, 64 adapters "
                        "r in {4..64}, K=N=4096",
            "path": "segmented_branch_varlen (schedule + shrink + expand)", "bound": "hbm", "unit": "GB/s",
            "value": round(gbs, 1), "ms": round(ms, 5), "ms_single": round(ms1, 5), "bytes": nbytes,
            "tflops": round(flops / ms / 1e9, 3), "peak": hbm, "hbm_frac": round(gbs / hbm, 4),
            "parity": {k: rep[k] for k in ("rows_checked", "max_abs_excess", "rel_fro", "ok")},
            "with_base": {"what": "C3 batch with its base linear y = x W^T (W 4096x4096): base GEMM + branch "
                                  "vs segmented_linear_varlen (one GEMM, adapters as per-tile K tail)",
                          "ms_unfused": round(ms_unfused, 5), "ms_fused": round(ms_fused, 5),
                          "speedup": round(ms_unfused / ms_fused, 3),
                          "tflops_fused": round(flops_f / ms_fused / 1e9, 1),
                          "frac_of_sustained": round(flops_f / ms_fused / 1e9 / sus, 4),
                          "parity": {k: rep_f[k] for k in ("rows_checked", "max_abs_excess", "rel_fro", "ok")}},
            "timing": CHAIN_NOTE}


def _config_c4(steps):
    import torch

    from oracle import checks
    from probe_b200 import workloads

    dev = torch.device("cuda", 0)
    peaks = _peaks()
    sus = peaks.get("bf16_tflops_sustained", 1400.0)
    bf = torch.bfloat16
    projs = workloads.c4(device=dev, dtype=bf)
    runners = _c5_runners(projs)
    outs = [torch.empty((p.m, p.n), device=dev, dtype=bf) for p in projs]

    def step():
        for p, run, o in zip(projs, runners, outs):
            run(p.x, out=o)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        step()
    b.record()
    b.synchronize()
    ms = a.elapsed_time(b) / steps
    flops = sum(p.flops() for p in projs)
    tf = flops / ms / 1e9
    worst = {"rows_checked": 0, "max_abs_excess": 0.0, "rel_fro": 0.0, "ok": True}
    for i, (p, o) in enumerate(zip(projs, outs)):
        rep = checks.linear_report(o, p.x, p.w, None, p.a, p.b, p.scale, seed=i, full_checks=False)
        worst["rows_checked"] += rep["rows_checked"]
        worst["max_abs_excess"] = max(worst["max_abs_excess"], rep["max_abs_excess"])
        worst["rel_fro"] = max(worst["rel_fro"], rep["rel_fro"])
        worst["ok"] = worst["ok"] and rep["ok"]
    del projs, runners, outs
    torch.cuda.empty_cache()
    return {"workload": "C4 Llama-7B layer prefill, M=8192, r16 on q,k,v,o,gate,up,down",
            "path": "kconcat plan (shrink + fused GEMM) per projection", "bound": "tensor", "unit": "TFLOP/s",
            "value": round(tf, 2), "ms": round(ms, 4), "tokens_per_s": round(8192 / ms * 1e3, 1), "peak": sus,
            "frac": round(tf / sus, 4), "parity": worst,
            "timing": f"{steps} back-to-back steps of the seven projections, CUDA events; inputs >= 67 MB per "
                      "projection, 7 projections per step"}


GATE_SHAPES = (  # (name, M, K, N): the layer shapes the reference's CUTLASS-vs-cuBLAS gate runs
    ("wan/attn-1536", 32760, 1536, 1536),
    ("wan/ffn-up-8960", 32760, 1536, 8960),
    ("wan/ffn-down-1536", 32760, 8960, 1536),
    ("llm/prefill-4096", 4096, 4096, 4096),
)


def _config_gate(steps):
    """Plain GEMM (no LoRA) of this library against cuBLAS (torch's linear) on
    the gate shapes of loraforge_kernels/bench_cutlass_gate.py:21-26: fusing
    the LoRA expand into the GEMM only pays if the GEMM itself is cuBLAS-class."""
    import torch

    from probe_b200 import kernels

    dev = torch.device("cuda", 0)
    sus = _peaks().get("bf16_tflops_sustained", 1400.0)
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(7)
    rows = []
    for name, m, k, n in GATE_SHAPES:
        flops = 2.0 * m * k * n
        nbytes = 2 * (m * k + k * n + m * n)
        copies = [(torch.randn((m, k), generator=g, device=dev, dtype=bf),
                   torch.randn((n, k), generator=g, device=dev, dtype=bf) / math.sqrt(k),
                   torch.empty((m, n), device=dev, dtype=bf)) for _ in range(_copies_for(nbytes))]
        ours = [lambda c=c: kernels.gemm(c[0], c[1], out=c[2]) for c in copies]
        ref = [lambda c=c: torch.matmul(c[0], c[1].t(), out=c[2]) for c in copies]
        ms_ours, ms_ref = _time_chains([ours, ref], max(steps, 10), dev)
        x, w, o = copies[0]
        got = kernels.gemm(x, w)
        want = torch.matmul(x, w.t())
        rel = float((got.float() - want.float()).norm() / want.float().norm())
        rows.append({"shape": name, "m": m, "k": k, "n": n, "ms": round(ms_ours, 5), "ms_cublas": round(ms_ref, 5),
                     "tflops": round(flops / ms_ours / 1e9, 1), "tflops_cublas": round(flops / ms_ref / 1e9, 1),
                     "ratio_vs_cublas": round(ms_ref / ms_ours, 3), "rel_fro_vs_cublas": rel,
                     "copies": len(copies)})
        del copies, ours, ref, got, want
        torch.cuda.empty_cache()
    geo = math.exp(sum(math.log(r["ratio_vs_cublas"]) for r in rows) / len(rows))
    return {"workload": "GEMM gate: plain bf16 GEMM vs cuBLAS on the reference's gate shapes (no LoRA)",
            "path": "kernels.gemm (lora_gemm_ex, rank 0) vs torch.matmul (cuBLAS)", "bound": "tensor",
            "unit": "TFLOP/s", "value": round(sum(r["tflops"] for r in rows) / len(rows), 1),
            "ms": round(sum(r["ms"] for r in rows), 5), "peak": sus,
            "frac": round(sum(r["tflops"] for r in rows) / len(rows) / sus, 4),
            "geomean_speedup_vs_cublas": round(geo, 3), "cases": rows, "timing": CHAIN_NOTE.split(";")[0]}


def measure_configs(steps=10):
    """C1-C4 against their own rooflines (each entry carries its parity)."""
    out = {}
    for name, fn in (("c1", lambda: _config_c1_c2("c1", steps)), ("c2", lambda: _config_c1_c2("c2", steps)),
                     ("c3", lambda: _config_c3(steps)), ("c4", lambda: _config_c4(steps))):
        try:
            out[name] = fn()
        except Exception as exc:  # noqa: BLE001 -- a failed config is reported, not hidden
            out[name] = {"error": f"{type(exc).__name__}: {exc}"}
    for name in ("c1", "c2"):
        e = out.get(name, {})
        if "cases" in e:
            main = e["cases"][-1]
            e.update({"value": main["gbs"], "ms": main["ms"], "hbm_frac": main["hbm_frac"]})
    return out


def run_config(args):
    """One JSON line for a single config c1-c4, against the roofline that bounds it."""
    import torch

    from probe_b200 import _lib

    _lib.load()
    torch.cuda.set_device(0)
    res = {"c1": lambda: _config_c1_c2("c1", args.steps), "c2": lambda: _config_c1_c2("c2", args.steps),
           "c3": lambda: _config_c3(args.steps), "c4": lambda: _config_c4(args.steps),
           "gate": lambda: _config_gate(args.steps)}[args.workload]()
    if "cases" in res and args.workload != "gate":
        main = res["cases"][-1]
        value, ms, frac = main["gbs"], main["ms"], main["hbm_frac"]
        tokens = main["m"]
    else:
        value, ms = res["value"], res["ms"]
        frac = res.get("hbm_frac", res.get("frac"))
        tokens = {"c3": 4096, "c4": 8192}.get(args.workload, 0)
    line = {"metric": METRIC, "value": value, "unit": res["unit"], "n_gpus": 1, "steps": args.steps, "warmup": 3,
            "ms_per_step": ms, "tokens_per_s": round(tokens / ms * 1e3, 1) if tokens else None, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded Gaussian; no public dataset)",
            "config": {k: v for k, v in res.items() if k not in ("value", "unit")},
            "roofline": {"bound": res["bound"], "achieved": value, "peak": res["peak"], "unit": res["unit"],
                         "frac": frac, "peak_source": "measured (MEASURED_PEAKS.json)"},
            "workload_id": args.workload, "device_error": _lib.device_error(0)}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload != "c5":
        run_config(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
