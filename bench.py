"""Benchmark of the B200 hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

Workloads (seeded synthetic data, see telmo_b200/synthetic.py):
  linear   config 1: one int8-weight linear, A f32 [1500, 1024] x W int8 [4096, 1024] + bias,
           f32 out. A step is one telmo_linear call (activation quantization + tensor-core GEMM).

`--impl reference` times the reference's CPU path for the same workload -- the oracle's C
restatement of telmo's CPU kernels (the reference is Rust and cannot be built here), on all
host cores -- and prints the same JSON line with "impl": "reference". Under torchrun only rank 0
runs it.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def peaks():
    try:
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------------
# the config-1 linear workload

class LinearWorkload:
    name = "config1-linear"
    metric = "int8 linear TOPS (config 1: A f32 [1500,1024] x W int8 [4096,1024] + bias, f32 out)"
    unit = "TOPS"

    def __init__(self):
        from telmo_b200 import synthetic
        self.a, (self.values, self.scales, self.n, self.k), self.bias = synthetic.config1()
        self.m = self.a.shape[0]
        self.ops = 2.0 * self.m * self.n * self.k

    def config(self):
        return {"workload": self.name, "m": self.m, "k": self.k, "n": self.n,
                "activations": "split int8 (2 levels), i32 accumulate", "l2": "flushed"}

    # -- GPU ------------------------------------------------------------------------------
    def setup_gpu(self, ctx):
        import torch
        from telmo_b200 import Kernels, PackedWeights, Precision
        self.torch = torch
        self.kern = Kernels(ctx)
        self.w = PackedWeights(self.n, self.k, Precision.INT8, self.values, self.scales).upload(ctx)
        self.da = torch.from_numpy(self.a).cuda()
        self.dbias = torch.from_numpy(self.bias).cuda()
        self.dc = torch.empty((self.m, self.n), dtype=torch.float32, device="cuda")
        ldq = (self.k + 15) // 16 * 16
        self.ldq = ldq
        self.hi = torch.empty((self.m, ldq), dtype=torch.int8, device="cuda")
        self.lo = torch.empty_like(self.hi)
        self.rs = torch.empty(self.m, dtype=torch.float32, device="cuda")
        self.ha = torch.from_numpy(self.a).pin_memory()
        self.hc = torch.empty((self.m, self.n), dtype=torch.float32).pin_memory()

    def step_gpu(self, ev=None):
        """One step; ev = (e_before_gemm, e_after_gemm) to time the dominant kernel."""
        from telmo_b200 import Epilogue
        self.kern.quantize_x2(self.da, self.k, self.m, self.k, self.hi, self.lo, self.ldq, self.rs)
        if ev:
            ev[0].record()
        self.kern.linear_q(self.hi, self.lo, self.ldq, self.rs, self.m, self.w, self.dc, self.n,
                           Epilogue(bias=self.dbias))
        if ev:
            ev[1].record()

    launches_per_step = 2

    def step_e2e(self):
        """Through the public call with host buffers: H2D of A, telmo_linear, D2H of C."""
        from telmo_b200 import Epilogue
        self.da.copy_(self.ha, non_blocking=True)
        self.kern.linear(self.da, self.m, self.w, self.dc, Epilogue(bias=self.dbias))
        self.hc.copy_(self.dc, non_blocking=True)

    def e2e_bytes(self):
        return self.a.nbytes, self.m * self.n * 4

    def units_per_step(self):
        return self.ops / 1e12  # tera-ops

    def kernel_roofline(self, hbm_gbs, bf16_tflops, peak_kind):
        # The GEMM's algorithmic HBM bytes: both int8 levels of A, W, the f32 output, scales.
        traffic = 2 * self.m * self.k + self.n * self.k + 4 * self.m * self.n + 4 * (self.m + 2 * self.n)
        return {"bound": "hbm", "bytes": traffic, "peak": hbm_gbs, "unit": "GB/s",
                "peak_kind": peak_kind}

    # -- CPU reference -------------------------------------------------------------------------
    def cpu_step(self, threads, rows):
        from oracle import oracle
        oracle.linear_int8(self.a[:rows], self.values, self.scales, self.n, self.k, self.bias,
                           threads=threads)

    def cpu_sample(self, threads):
        """Times the reference's CPU path (oracle port) on a bounded sample: the full config-1
        product, best of 5 (benches/matmul.rs:59-60)."""
        rows = self.m
        best = float("inf")
        t_end = time.time() + 20
        for _ in range(5):
            t0 = time.perf_counter()
            self.cpu_step(threads, rows)
            best = min(best, time.perf_counter() - t0)
            if time.time() > t_end:
                break
        ops = 2.0 * rows * self.n * self.k
        return ops / best / 1e12, f"config-1 product ({rows}x{self.k}x{self.n}), best of 5"


WORKLOADS = {"linear": LinearWorkload}


def flush_l2(buf):
    buf.zero_()


def run_ours(args, rank, world, local_rank):
    import torch
    import telmo_b200
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist_mod
        import datetime
        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local_rank))
        dist = dist_mod
    ctx = telmo_b200.Context(local_rank)
    wl = WORKLOADS[args.workload]()
    wl.setup_gpu(ctx)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    for _ in range(args.warmup):
        wl.step_gpu()
        flush_l2(flush)
    ctx.check()

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    clocks = Clocks(local_rank)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    barrier()
    clocks.start()
    time.sleep(0.3)
    for i in range(args.steps):
        flush_l2(flush)
        starts[i].record()
        wl.step_gpu(kev[i])
        ends[i].record()
    barrier()
    ctx.check()
    # e2e through the public call with host buffers.
    e_start = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e_end = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush_l2(flush)
        e_start[i].record()
        wl.step_e2e()
        e_end[i].record()
    barrier()
    clk = clocks.stop()
    ctx.check()
    step_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    kern_ms = [a.elapsed_time(b) for a, b in kev]
    e2e_ms = sum(s.elapsed_time(e) for s, e in zip(e_start, e_end))
    t = torch.tensor([step_ms, e2e_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms, e2e_ms = t.tolist()
    if rank == 0:
        hbm, bf16, kind = peaks()
        units = wl.units_per_step() * args.steps * world
        value = units / (step_ms / 1e3)
        rl = wl.kernel_roofline(hbm, bf16, kind)
        avg_kernel_s = statistics.mean(kern_ms) / 1e3
        if rl["bound"] == "hbm":
            achieved = rl["bytes"] / avg_kernel_s / 1e9
        else:
            achieved = rl["flops"] / avg_kernel_s / 1e12
        cpu_value, cpu_sample = wl.cpu_sample(os.cpu_count() or 1)
        bi, bo = wl.e2e_bytes()
        line = {
            "metric": wl.metric, "value": round(value, 3), "unit": wl.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(step_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int8 -> i32 (2 levels)",
            "data": "synthetic (seeded, telmo_b200/synthetic.py)", "config": wl.config(),
            "e2e": {"value": round(wl.units_per_step() * args.steps * world / (e2e_ms / 1e3), 3),
                    "unit": wl.unit, "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo},
            "roofline": {"bound": rl["bound"], "achieved": round(achieved, 1), "peak": rl["peak"],
                         "unit": rl["unit"], "frac": round(achieved / rl["peak"], 4),
                         "traffic": None, "peak_source": rl["peak_kind"],
                         "kernel_us": round(avg_kernel_s * 1e6, 2)},
            "cpu_baseline": {"value": round(cpu_value, 4), "unit": wl.unit,
                             "cores": os.cpu_count(), "kind": "port", "sample": cpu_sample},
            "clocks": clk,
            "gpu_launches": wl.launches_per_step * args.steps,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()


def run_reference(args, rank, world):
    if rank != 0:
        return
    wl = WORKLOADS[args.workload]()
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        wl.cpu_step(threads, wl.m)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        wl.cpu_step(threads, wl.m)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = wl.units_per_step() * args.steps / total
    line = {
        "impl": "reference", "metric": wl.metric, "value": round(value, 4), "unit": wl.unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (int8 weights widened)",
        "data": "synthetic (seeded, telmo_b200/synthetic.py)", "config": wl.config(),
        "cpu_baseline": {"value": round(value, 4), "unit": wl.unit, "cores": threads,
                         "kind": "port",
                         "sample": "the oracle's C restatement of telmo's AVX-512 path "
                                   "(reference Rust not buildable here), full config-1 product"},
        "e2e": {"value": round(value, 4), "unit": wl.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="linear")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus if args.gpus == 1 else 1)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
