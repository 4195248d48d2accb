#!/usr/bin/env python3
"""Benchmark of the B200 LoRA-linear hot path (one JSON line on rank 0).

Workload (default, config C5): the six LoRA-adapted projections of a Wan-style
video DiT block -- q, k, v, o (5120->5120), FFN up (5120->13824) and FFN down
(13824->5120) -- at M = 32760 tokens, each carrying a weighted stack of three
LoRAs (r = 32, 64, 128 with weights 1.0, 0.7, 0.4) stacked into one rank-224
sidecar exactly as attach_fused_lora does.  bf16, seeded Gaussian inputs
generated on the device.  A step is one pass over all six projections.

value   whole-job TFLOP/s (algorithmic FLOPs / max-over-ranks device time), inputs
        resident in HBM.  Every input tensor is larger than the 126 MB L2, so no
        flush is needed between iterations.
e2e     the same FLOPs through the public module API (FusedLoRALinear via
        attach_fused_lora) from pinned HOST buffers: each step copies every
        projection's activations in and its outputs back.
scaling weak: every rank processes its own 32760-token batch (token / request
        sharding with W and the adapters replicated; no data-path collective).
        --scaling strong splits the 32760 tokens across the ranks instead.

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
WORKLOAD = "C5 Wan DiT block projections (q,k,v,o 5120->5120; ffn 5120->13824->5120) with 3-LoRA stack r=32/64/128 (w 1.0/0.7/0.4) -> r224"
M_TOKENS = 32760
CPU_SAMPLE_TOKENS = 4096
# DRAM read + write of one fused-GEMM launch (C5 q projection), from the full
# ncu capture at M = 16384 committed under profiles/, scaled linearly to M:
# 820.2 MB read + 152.6 MB write per launch at M = 16384 (CTA-pair kernel, 256x512 tiles).
NCU_TRAFFIC_Q_16384 = 972.8e6


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--scaling", default="weak", choices=["weak", "strong"])
    p.add_argument("--tokens", type=int, default=M_TOKENS)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--workload", default="c5", choices=["c1", "c2", "c3", "c4", "c5"],
                   help="c5 is the headline; c1-c4 measure the other configs against their own rooflines")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


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
        skip = getattr(self, "skip", 0)
        if len(rows) > skip:
            rows = rows[skip:]  # the samples taken during the timed region
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------- GPU bench
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
    from probe_b200.fused_linear import _KConcat
    from probe_b200.runtime_lora import attach_fused_lora

    _lib.load()
    m = args.tokens if args.scaling == "weak" else -(-args.tokens // world)
    if args.scaling == "strong":
        lo = min(rank * m, args.tokens)
        m = max(0, min(args.tokens, lo + m) - lo)
    torch.manual_seed(1234 + rank)
    projs = workloads.c5(device=dev, dtype=torch.bfloat16, m=m)
    runners = [_KConcat(p.w, p.bias, p.a, p.b, p.scale) for p in projs]
    outs = [torch.empty((p.m, p.n), device=dev, dtype=torch.bfloat16) for p in projs]
    flops = sum(p.flops() for p in projs)
    gemm_flops = sum(2.0 * p.m * p.k * p.n + 2.0 * p.m * p.r * p.n for p in projs)  # algorithmic (rank r, not 2 r16)
    launches_per_step = 2 * len(projs)  # shrink GEMM + fused GEMM per projection

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

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()

    # ---- timed region (device-resident inputs)
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in projs]
          for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    clocks.wait_first()
    start.record()
    for s in range(args.steps):
        step(ev[s])
    end.record()
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    gemm_ms = sum(a.elapsed_time(b) for row in ev for a, b in row)
    t = torch.tensor([ms, gemm_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, gemm_ms = float(t[0]), float(t[1])
    err = _lib.device_error(local)

    # ---- e2e through the public module API with pinned host buffers
    e2e = None
    if not args.no_e2e:
        holder = torch.nn.Module()
        for i, p in enumerate(projs):
            lin = torch.nn.Linear(p.k, p.n, bias=False, device=dev, dtype=torch.bfloat16)
            with torch.no_grad():
                lin.weight.copy_(p.w)
            holder.add_module(f"p{i}", lin)
            attach_fused_lora(holder, f"p{i}", p.a, p.b, alpha=p.scale)
        host_x = [p.x.cpu().pin_memory() for p in projs]
        host_out = [torch.empty((p.m, p.n), dtype=torch.bfloat16, pin_memory=True) for p in projs]
        dev_x = [torch.empty_like(p.x) for p in projs]
        copy_in = torch.cuda.Stream(dev)
        compute = torch.cuda.current_stream(dev)
        h2d = sum(x.numel() * x.element_size() for x in host_x)
        d2h = sum(o.numel() * o.element_size() for o in host_out)

        def e2e_step():
            ready = []
            with torch.cuda.stream(copy_in):
                for i in range(len(projs)):
                    dev_x[i].copy_(host_x[i], non_blocking=True)
                    e = torch.cuda.Event()
                    e.record(copy_in)
                    ready.append(e)
            for i in range(len(projs)):
                compute.wait_event(ready[i])
                y = getattr(holder, f"p{i}")(dev_x[i])
                host_out[i].copy_(y, non_blocking=True)
            copy_in.wait_stream(compute)

        with torch.no_grad():
            for _ in range(2):
                e2e_step()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e_steps = max(1, min(args.steps, 5))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(e_steps):
                e2e_step()
            e1.record()
            torch.cuda.synchronize()
            tt = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
            if world > 1:
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e_ms = float(tt[0]) / e_steps
        e2e = {"value": flops * world / (e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e_ms, "steps": e_steps,
               "path": "attach_fused_lora -> FusedLoRALinear.forward, pinned host in/out, copy-in stream overlap"}
        del host_x, host_out

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    total_flops = flops * world if args.scaling == "weak" else workloads.c5_flops(args.tokens)
    total_tokens = (m * world) if args.scaling == "weak" else args.tokens
    ms_step = ms / args.steps
    value = total_flops / (ms_step * 1e-3) / 1e12
    peaks = {}
    try:
        peaks = json.load(open(ROOT / "MEASURED_PEAKS.json"))
    except (OSError, ValueError):
        pass
    peak = peaks.get("bf16_tflops_sustained")
    peak_src = "measured sustained (MEASURED_PEAKS.json)"
    if peak is None:
        peak, peak_src = 1400.0, "fallback sustained"
    gemm_achieved = gemm_flops / (gemm_ms / args.steps * 1e-3) / 1e12
    traffic = round(NCU_TRAFFIC_Q_16384 * m / 16384)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "tokens_per_s": round(total_tokens / (ms_step * 1e-3), 1),
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded Gaussian, generated on device; no public dataset)",
        "config": {"workload": WORKLOAD, "tokens_per_gpu": m, "global_tokens": total_tokens, "lora_rank": 224,
                   "parallelism": f"token-sharded x{world}, weights+adapters replicated, no collective",
                   "l2": "every input > 126 MB L2 (x >= 335 MB per projection); no flush needed"},
        "roofline": {"bound": "tensor", "kernel": ("gemm_tc_kernel<256,4,bf16>" if os.environ.get("LORA_B200_GEMM") == "1sm"
                                else "gemm_tc2_kernel<4,2,bf16> (CTA pair, 256x512 tiles)")
                               + " fused base + LoRA K-slice",
                     "achieved": round(gemm_achieved, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(gemm_achieved / peak, 4), "peak_source": peak_src, "traffic": traffic,
                     "traffic_note": "bytes per q-projection launch (ncu capture at M=16384, scaled to M); "
                                     "algorithmic bytes of that launch: "
                                     f"{round(2 * (m * 5120 * 2 + 5120 * 5120 + 448 * (m + 5120)))}",
                     "flops_per_step": gemm_flops, "gemm_ms_per_step": round(gemm_ms / args.steps, 4)},
        "gpu_launches": launches_per_step * args.steps,
        "device_error": err,
    }
    if clock_info is not None:
        line["clocks"] = clock_info
    if e2e is not None:
        line["e2e"] = e2e
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
def _peaks():
    try:
        return json.load(open(ROOT / "MEASURED_PEAKS.json"))
    except (OSError, ValueError):
        return {}


def _time_flushed(fn, iters, dev):
    """Median device time (ms) of fn, each run from a cold L2 (a 512 MB write in between).

    fn is captured once in a CUDA graph, so the time is the kernels' own, not
    the host's launch overhead."""
    import torch

    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
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
    import torch

    for f in fns:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(launches):
            fns[i % len(fns)]()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b) / launches)
    del g
    return statistics.median(times)


def _copies_for(nbytes, floor=3, l2_multiple=3.0):
    """Copies of a working set of ``nbytes`` needed to exceed ``l2_multiple`` x L2."""
    return max(floor, int(math.ceil(l2_multiple * 126e6 / max(nbytes, 1))) + 1)


def run_config(args):
    """One JSON line for config c1-c4, each against the roofline that bounds it.

    C1-C3 are timed two ways: ``ms`` per call inside a 20-call CUDA-graph chain
    over rotating input copies (cold L2 for every call, graph floor amortised),
    and ``ms_single`` for one call per graph replay after a 512 MB L2 flush
    (includes the ~6 us replay floor)."""
    import torch

    from probe_b200 import _lib, kernels, segmented_branch, workloads
    from probe_b200.fused_linear import _KConcat, build_plan

    _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks = _peaks()
    hbm = peaks.get("hbm_gbs", 6650.0)
    tc = peaks.get("bf16_tflops", 1590.0)
    line = {"metric": METRIC, "n_gpus": 1, "steps": args.steps, "warmup": 3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded Gaussian; no public dataset)"}
    bf = torch.bfloat16
    if args.workload in ("c1", "c2"):
        cases = [workloads.c1(device="cpu")] if args.workload == "c1" else \
            [workloads.c2(m, device="cpu") for m in (1, 4, 16, 64)]
        rows = []
        for p in cases:
            flops, nbytes = p.flops(), p.bytes()
            ncopy = _copies_for(nbytes)
            fns = []
            for _ in range(ncopy):
                x, w, a, b = (t.to(dev, bf) for t in (p.x, p.w, p.a, p.b))
                plan = build_plan(x, w, None, a, b, p.scale)
                fns.append(lambda plan=plan, x=x: plan(x))
            ms = _time_chain(fns, max(args.steps, 10), dev)
            ms1 = _time_flushed(fns[0], max(args.steps, 20), dev)
            rows.append({"m": p.m, "ms": round(ms, 5), "ms_single": round(ms1, 5),
                         "tflops": round(flops / ms / 1e9, 2),
                         "gbs": round(nbytes / ms / 1e6, 1), "hbm_frac": round(nbytes / ms / 1e6 / hbm, 4),
                         "t_star_us": round(max(flops / tc / 1e12, nbytes / hbm / 1e9) * 1e6, 2),
                         "copies": ncopy})
            del fns
            torch.cuda.empty_cache()
        main = rows[-1]
        line.update({"value": main["gbs"], "unit": "GB/s", "ms_per_step": main["ms"],
                     "tokens_per_s": round(main["m"] / main["ms"] * 1e3, 1),
                     "config": {"workload": "C1 single fused LoRA linear 256x4096x4096 r16" if args.workload == "c1"
                                else "C2 decode LoRA linear M in {1,4,16,64}, W 11008x4096, r16",
                                "cases": rows,
                                "l2": "ms: 20-call CUDA-graph chain over rotating input copies (> 3x L2 between "
                                      "reuses); ms_single: one call per replay after a 512 MB flush"},
                     "roofline": {"bound": "hbm", "achieved": main["gbs"], "peak": hbm, "unit": "GB/s",
                                  "frac": main["hbm_frac"], "peak_source": "measured (MEASURED_PEAKS.json)"}})
    elif args.workload == "c3":
        c = workloads.c3(device="cpu", dtype=bf)
        flops, nbytes = c.branch_flops(), c.branch_bytes()
        w = c.w.to(dev)
        fns = []
        for _ in range(_copies_for(nbytes)):
            x = c.x.to(dev)
            y = kernels.gemm(x, w)
            tabs = [t.to(dev) for t in (c.a_flat, c.b_flat, c.offsets, c.ranks, c.seg_start, c.seg_adapter)]
            fns.append(lambda x=x, y=y, tabs=tabs: segmented_branch.segmented_branch_varlen(x, y, *tabs, c.r_max))
        ms = _time_chain(fns, max(args.steps, 10), dev)
        ms1 = _time_flushed(fns[0], max(args.steps, 20), dev)
        gbs = nbytes / ms / 1e6
        line.update({"value": round(gbs, 1), "unit": "GB/s", "ms_per_step": round(ms, 5),
                     "tokens_per_s": round(4096 / ms * 1e3, 1),
                     "config": {"workload": "C3 segmented multi-LoRA branch: 4096 tokens, 128 Zipf(1.1) segments, "
                                            "64 adapters r in {4..64}, K=N=4096",
                                "tflops": round(flops / ms / 1e9, 3), "bytes": nbytes,
                                "ms_single": round(ms1, 5), "copies": len(fns),
                                "l2": "ms: 20-call CUDA-graph chain over rotating input copies (> 3x L2 between "
                                      "reuses); ms_single: one call per replay after a 512 MB flush"},
                     "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                                  "frac": round(gbs / hbm, 4), "peak_source": "measured (MEASURED_PEAKS.json)"}})
    else:  # c4
        projs = workloads.c4(device=dev, dtype=bf)
        runners = [_KConcat(p.w, p.bias, p.a, p.b, p.scale) for p in projs]
        outs = [torch.empty((p.m, p.n), device=dev, dtype=bf) for p in projs]

        def step():
            for p, run, o in zip(projs, runners, outs):
                run(p.x, out=o)

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            step()
        b.record()
        b.synchronize()
        ms = a.elapsed_time(b) / args.steps
        flops = sum(p.flops() for p in projs)
        tf = flops / ms / 1e9
        sus = peaks.get("bf16_tflops_sustained", 1400.0)
        line.update({"value": round(tf, 2), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
                     "tokens_per_s": round(8192 / ms * 1e3, 1),
                     "config": {"workload": "C4 Llama-7B layer prefill, M=8192, r16 on q,k,v,o,gate,up,down",
                                "l2": "inputs >= 67 MB per projection, 7 projections per step"},
                     "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": sus, "unit": "TFLOP/s",
                                  "frac": round(tf / sus, 4),
                                  "peak_source": "measured sustained (MEASURED_PEAKS.json)"}})
    line["workload_id"] = args.workload
    line["device_error"] = _lib.device_error(0)
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
