"""Benchmark of the B200 hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

Workloads (seeded synthetic data, telmo_b200/synthetic.py):
  granite  (default) config 5: 4096 utterances, lengths log-uniform in 1-30 s (about 34,900 s of
           audio), through the config-2 Granite-shaped int8 CTC model: log-mel front end,
           16-block encoder, CTC head, greedy argmax and collapse. Utterances are sharded across
           ranks by longest-first greedy assignment (no collective; each rank keeps its tokens)
           and processed in length-sorted batches of about equal audio, at most 4500 s each
           (ceil(shard seconds / 4500) of them). A step is
           one pass over the whole set. metric = RTFx (audio seconds / wall second), whole job.
  parakeet config 4: 256 utterances, lengths uniform in 1-30 s (about 4,000 s of audio), through
           the Parakeet-TDT-shaped int8 model: 128-bin log-mel, 8x convolutional subsampling,
           24-layer FastConformer encoder, greedy TDT decoding (token and duration per step),
           sharded and batched as granite.
  linear   config 1: one int8-weight linear, A f32 [1500, 1024] x W int8 [4096, 1024] + bias
           (--shape M,K,N for another product shape with the same distributions).
  load     the config-5 Granite model loaded from a pack in host memory: the median load time
           from the reference's panel layout and from a device-layout pack (no host repack).

`--impl reference` times the reference's CPU path for the same workload: the oracle's C
restatement of telmo's CPU path (the reference is Rust and cannot be built here) on all host
cores, each step a bounded sample of the workload, and prints the same line with "impl":
"reference". Under torchrun only rank 0 runs it.
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
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
SR = 16000


def peaks():
    try:
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        return {k: float(p[k]) for k in FALLBACK}, "measured (MEASURED_PEAKS.json)"
    except Exception:
        return dict(FALLBACK), "fallback (profiling recipe)"


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device, self.proc, self.lines = device, None, []

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
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


# ---------------------------------------------------------------------------------------------
# config 5: the Granite-shaped model over 4096 log-uniform utterances

class GraniteWorkload:
    name = "config5-granite-ctc"
    metric = ("RTFx (audio-s per wall-s, whole job): Granite-shaped int8 CTC model, "
              "16 kHz audio -> log-mel -> 16-block encoder -> CTC greedy tokens")
    unit = "audio-s/s"
    POOL = 64  # distinct 30 s base waveforms; utterance u is a slice of waveform u % 64

    def __init__(self, rank, world, n_utt=4096, batch_seconds=4500.0, precision="int8"):
        from telmo_b200 import sharding, synthetic
        self.synthetic = synthetic
        self.n_utt = n_utt
        self.precision = precision
        secs = synthetic.lengths_log_uniform(n_utt, 1.0, 30.0, seed=0)
        self.samples = np.maximum((secs * SR).astype(np.int64), 2 * 160)
        self.total_seconds = float(self.samples.sum()) / SR
        # Longest-first greedy assignment of utterances to ranks, then length-sorted batches.
        mine = sharding.assign(self.samples, world)[rank]
        self.batches = sharding.batches(mine, self.samples, batch_seconds)
        self.mine = [u for b in self.batches for u in b]
        self.rank_seconds = float(self.samples[self.mine].sum()) / SR
        self.batch_seconds = batch_seconds

    def _entries(self, cfg):
        return self.synthetic.granite_entries(cfg, seed=1, scales="spec", precision=self.precision)

    def utterance(self, u, pool):
        n = int(self.samples[u])
        base = pool[u % self.POOL]
        off = int(self.synthetic.rng(10_000 + u).integers(0, len(base) - n + 1))
        return base[off:off + n]

    def make_pool(self):
        return [self.synthetic.audio(30.0, seed=1000 + i) for i in range(self.POOL)]

    def config(self, world):
        return {"workload": self.name, "utterances": self.n_utt,
                "audio_seconds": round(self.total_seconds, 1),
                "lengths": "log-uniform 1-30 s (seed 0)",
                "model": "Granite-shaped: d 1024, 16 blocks, 8 heads x 128, ff 4096, conv 2048 x k15, "
                         "context 128, vocab 2049, int8 weights (scales U(1e-3,1e-2))",
                "weights": self.precision if self.precision == "int8" else
                "q8_0 (Int8 weights re-quantized per 32 inputs; the relative tables and the "
                "2049-input mid projection stay Int8)",
                "global_batch": self.n_utt, "sharding": f"utterances over {world} GPU(s), "
                                                        "longest-first greedy, no collective",
                "per_rank_batches": len(self.batches), "batch_seconds_max": self.batch_seconds,
                "activations": "split int8 (2 levels) x int8 weights -> i32, f32 elsewhere",
                "l2": "inputs larger than L2 (2.2 GB of audio, ~1 GB of weights+activations "
                      "per batch)"}

    # -- GPU --------------------------------------------------------------------------------
    def setup_gpu(self, ctx):
        import torch
        from telmo_b200.granite import Granite
        cfg = self.synthetic.granite_config()
        entries = self._entries(cfg)
        self.model = Granite.from_entries(ctx, cfg, entries)
        del entries
        pool = self.make_pool()
        audio = [self.utterance(u, pool) for u in self.mine]
        del pool
        packed = np.concatenate(audio) if audio else np.zeros(1, np.float32)
        self.host_audio = torch.from_numpy(packed).pin_memory()
        self.dev_audio = self.host_audio.cuda()
        self.offsets = []
        at = 0
        for b in self.batches:
            n = int(self.samples[b].sum())
            self.offsets.append((at, n))
            at += n
        frames = max((sum(self.model.frames_for_samples(int(self.samples[u])) for u in b)
                      for b in self.batches), default=1)
        self.dev_tokens = torch.empty(3 * frames + 3, dtype=torch.int32, device="cuda")
        self.dev_counts = torch.empty(max(len(b) for b in self.batches) + 1, dtype=torch.int32,
                                      device="cuda")
        self.bi = int(packed.nbytes)
        self.bo = 0
        # End to end: the whole shard in one telmo_granite_transcribe call with host buffers; it
        # transcribes in groups of batch_seconds (the same cut as self.batches, since self.mine is
        # length-sorted) and copies each group's audio up while the previous group runs -- in at
        # least two groups, so that a copy overlaps compute even when the shard fits one batch.
        self.model.set_transcribe_group(min(self.batch_seconds, self.rank_seconds / 2 + 1.0))
        self.mine_lengths = np.ascontiguousarray(self.samples[self.mine], dtype=np.int64)
        all_frames = sum(self.model.frames_for_samples(int(x)) for x in self.mine_lengths)
        self.host_tokens_all = torch.empty(3 * all_frames + 3, dtype=torch.int32).pin_memory()

    def step_gpu(self):
        for b, (at, n) in zip(self.batches, self.offsets):
            self.model.transcribe_device(self.dev_audio[at:at + n], self.samples[b],
                                         self.dev_tokens, self.dev_counts)

    def step_e2e(self):
        """The shard through telmo_granite_transcribe, the host-buffer entry point: pinned host
        audio in, host tokens, counts and frames out, every copy inside the call."""
        if not self.mine:
            return
        _, counts, frames = self.model.transcribe_arrays(self.host_audio, self.mine_lengths,
                                                         tokens_buf=self.host_tokens_all)
        self.bo = 12 * int(frames.sum()) + 4 * int(counts.size)

    def units_per_step(self):
        return self.rank_seconds

    # -- per-kernel-class timing through the model's profiler -----------------------------------
    def profile_start(self):
        from telmo_b200 import _lib
        L = _lib.load()
        getattr(L, self.PROFILE)(self.model.handle, 1)
        getattr(L, self.PROFILE + "_read")(self.model.handle, None, None, None, None)
        self.launches0 = self.model.launches()

    def profile_stop(self):
        import ctypes
        from telmo_b200 import _lib
        L = _lib.load()
        ms = (ctypes.c_double * 4)()
        cnt = (ctypes.c_long * 4)()
        ops, byt = ctypes.c_double(), ctypes.c_double()
        getattr(L, self.PROFILE + "_read")(self.model.handle, ms, cnt, ctypes.byref(ops),
                                           ctypes.byref(byt))
        getattr(L, self.PROFILE)(self.model.handle, 0)
        launches = self.model.launches() - self.launches0
        return launches, {"gemm_ms": ms[0], "gemm_n": cnt[0], "attn_ms": ms[1], "attn_n": cnt[1],
                          "rows_ms": ms[2], "fe_ms": ms[3], "ops": ops.value, "bytes": byt.value}

    PROFILE = "telmo_granite_profile"

    # -- CPU reference ------------------------------------------------------------------------
    CPU_SAMPLE_SECONDS = 240.0

    def cpu_sample_utts(self, target_s=None):
        """A bounded sample of the workload for the CPU path, spread over its length
        distribution: with the set's utterances sorted by length, the ones at evenly spaced
        quantiles (i + 1/2) / n, n chosen so the sample holds about target_s seconds."""
        target_s = target_s or self.CPU_SAMPLE_SECONDS
        order = np.argsort(self.samples, kind="stable")
        mean = float(self.samples.mean()) / SR
        n = int(min(len(order), max(1, round(target_s / mean))))
        chosen = [int(order[int((i + 0.5) * len(order) / n)]) for i in range(n)]
        return chosen, float(self.samples[chosen].sum()) / SR

    def cpu_setup(self):
        from oracle import oracle
        cfg = self.synthetic.granite_config()
        entries = self._entries(cfg)
        self.oracle = oracle
        self.ref = oracle.Granite(cfg, entries)
        del entries
        pool = self.make_pool()
        self.cpu_utts, self.cpu_seconds = self.cpu_sample_utts()
        self.cpu_audio = [self.utterance(u, pool) for u in self.cpu_utts]

    def cpu_step(self, threads):
        for a in self.cpu_audio:
            f = self.oracle.granite_features(a)
            enc = self.ref.encode(f, threads=threads)
            ids, _ = self.ref.frame_ids(enc, threads=threads)
            self.oracle.ctc_tokens(ids)

    def cpu_sample(self, threads):
        self.cpu_setup()
        t0 = time.perf_counter()
        self.cpu_step(threads)
        dt = time.perf_counter() - t0
        return self.cpu_seconds / dt, (f"{len(self.cpu_utts)} utterances at evenly spaced length "
                                       f"quantiles of the set ({self.cpu_seconds:.1f} s of audio), "
                                       f"audio -> tokens")


# ---------------------------------------------------------------------------------------------
# config 4: the Parakeet-TDT-shaped model over 256 uniform utterances

class ParakeetWorkload(GraniteWorkload):
    name = "config4-parakeet-tdt"
    metric = ("RTFx (audio-s per wall-s, whole job): Parakeet-TDT-shaped int8 model, "
              "16 kHz audio -> log-mel -> 8x conv subsampling -> 24-layer FastConformer -> "
              "greedy TDT tokens and durations")
    PROFILE = "telmo_parakeet_profile"
    CPU_SAMPLE_SECONDS = 150.0

    # The whole set (about 4,240 s) fits one batch: every matrix product runs over all frames.
    def __init__(self, rank, world, n_utt=256, batch_seconds=4500.0, precision="int8"):
        from telmo_b200 import sharding, synthetic
        self.synthetic = synthetic
        self.n_utt = n_utt
        self.precision = precision
        secs = synthetic.lengths_uniform(n_utt, 1.0, 30.0, seed=0)
        self.samples = np.maximum((secs * SR).astype(np.int64), 2 * 160)
        self.total_seconds = float(self.samples.sum()) / SR
        mine = sharding.assign(self.samples, world)[rank]
        self.batches = sharding.batches(mine, self.samples, batch_seconds)
        self.mine = [u for b in self.batches for u in b]
        self.rank_seconds = float(self.samples[self.mine].sum()) / SR
        self.batch_seconds = batch_seconds
        self.cfg = synthetic.parakeet_config()

    def config(self, world):
        c = dict(super().config(world))
        c.update({"lengths": "uniform 1-30 s (seed 0)",
                  "model": "Parakeet-TDT-shaped: 128 mels, 3 stride-2 convs x 256 ch, d 1024, "
                           "24 layers, 8 heads x 128, ff 4096, conv k9, Transformer-XL positions; "
                           "2-layer LSTM 640, joint 640 -> 8193 + 5 durations, max 10 symbols "
                           "per frame; int8 weights (scales U(1e-3,1e-2))",
                  "weights": self.precision if self.precision == "int8" else
                  "q8_0 (the Int8 weights re-quantized per 32 inputs; the reference's "
                  "recommended Parakeet precision)",
                  "l2": "inputs larger than L2 (127 MB of audio, ~10 GB of activations per "
                        "batch)"})
        return c

    def _entries(self, cfg=None):
        return self.synthetic.parakeet_entries(self.cfg, seed=3, scales="spec", precision=self.precision)

    def setup_gpu(self, ctx):
        import torch
        from telmo_b200.parakeet import Parakeet, frames_for_samples
        self.model = Parakeet.from_entries(ctx, self.cfg, self._entries())
        pool = self.make_pool()
        audio = [self.utterance(u, pool) for u in self.mine]
        del pool
        packed = np.concatenate(audio) if audio else np.zeros(1, np.float32)
        self.host_audio = torch.from_numpy(packed).pin_memory()
        self.dev_audio = self.host_audio.cuda()
        self.offsets = []
        at = 0
        for b in self.batches:
            n = int(self.samples[b].sum())
            self.offsets.append((at, n))
            at += n
        frames = max((sum(frames_for_samples(int(self.samples[u])) for u in b)
                      for b in self.batches), default=1)
        cap = 3 * self.cfg["max_symbols"] * frames + 3
        self.dev_tokens = torch.empty(cap, dtype=torch.int32, device="cuda")
        self.dev_counts = torch.empty(max(len(b) for b in self.batches) + 1, dtype=torch.int32,
                                      device="cuda")
        self.host_tokens = torch.empty(cap, dtype=torch.int32).pin_memory()
        self.bi = int(packed.nbytes)
        self.bo = 0

    def step_e2e(self):
        bo = 0
        for b, (at, n) in zip(self.batches, self.offsets):
            toks, counts, _ = self.model.transcribe_arrays(self.host_audio[at:at + n], self.samples[b],
                                                           tokens_buf=self.host_tokens)
            bo += 12 * int(counts.sum()) + 4 * len(b)
        self.bo = bo
        return toks

    def cpu_setup(self):
        from oracle import oracle
        self.oracle = oracle
        self.ref = oracle.Parakeet(self.cfg, self._entries())
        pool = self.make_pool()
        self.cpu_utts, self.cpu_seconds = self.cpu_sample_utts()
        self.cpu_audio = [self.utterance(u, pool) for u in self.cpu_utts]

    def cpu_step(self, threads):
        for a in self.cpu_audio:
            f = self.oracle.parakeet_features(a)
            self.ref.decode(self.ref.encode(f, threads=threads), threads=threads)


# ---------------------------------------------------------------------------------------------
# config 1: one linear

class LinearWorkload:
    name = "config1-linear"
    metric = "int8 linear TOPS (config 1: A f32 [1500,1024] x W int8 [4096,1024] + bias, f32 out)"
    unit = "TOPS"

    def __init__(self, rank, world, shape=None, precision="int8"):
        from telmo_b200 import synthetic
        if shape:  # another product shape (M, K, N) with config 1's distributions
            m, k, n = shape
            self.a, (self.values, self.scales, self.n, self.k), self.bias = synthetic.config1(m=m, k=k, n=n)
            self.name = f"linear-{m}x{k}x{n}"
            self.metric = f"int8 linear TOPS (A f32 [{m},{k}] x W int8 [{n},{k}] + bias, f32 out)"
        else:
            self.a, (self.values, self.scales, self.n, self.k), self.bias = synthetic.config1()
        self.precision = precision
        if precision == "q8_0":  # the same weights re-quantized per block of 32 inputs
            self.values, self.scales, _, _, _ = synthetic.as_q8_0((self.values, self.scales, self.n, self.k))
            self.metric = self.metric.replace("W int8", "W Q8_0")
            self.name += "-q8_0"
        self.m = self.a.shape[0]
        self.ops = 2.0 * self.m * self.n * self.k

    def config(self, world):
        return {"workload": self.name, "m": self.m, "k": self.k, "n": self.n, "weights": self.precision,
                "activations": "split int8 (2 levels), i32 accumulate", "l2": "flushed"}

    def setup_gpu(self, ctx):
        import torch
        from telmo_b200 import Kernels, PackedWeights, Precision
        self.kern = Kernels(ctx)
        prec = Precision.Q8_0 if self.precision == "q8_0" else Precision.INT8
        self.w = PackedWeights(self.n, self.k, prec, self.values, self.scales).upload(ctx)
        self.da = torch.from_numpy(self.a).cuda()
        self.dbias = torch.from_numpy(self.bias).cuda()
        self.dc = torch.empty((self.m, self.n), dtype=torch.float32, device="cuda")
        self.ha = torch.from_numpy(self.a).pin_memory()
        self.hc = torch.empty((self.m, self.n), dtype=torch.float32).pin_memory()
        self.flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
        self.bi, self.bo = self.a.nbytes, self.m * self.n * 4

    def step_gpu(self):
        from telmo_b200 import Epilogue
        self.kern.linear(self.da, self.m, self.w, self.dc, Epilogue(bias=self.dbias))

    def step_e2e(self):
        from telmo_b200 import Epilogue
        self.da.copy_(self.ha, non_blocking=True)
        self.kern.linear(self.da, self.m, self.w, self.dc, Epilogue(bias=self.dbias))
        self.hc.copy_(self.dc, non_blocking=True)

    def between_steps(self):
        self.flush.zero_()

    def algorithmic_bytes(self):
        return 4 * self.m * self.k + self.n * self.k + 8 * self.n + 4 * self.m * self.n

    def units_per_step(self):
        return self.ops / 1e12

    def _oracle_linear(self):
        from oracle import oracle
        return oracle.linear_q8_0 if self.precision == "q8_0" else oracle.linear_int8

    def cpu_step(self, threads):
        self._oracle_linear()(self.a, self.values, self.scales, self.n, self.k, self.bias,
                              threads=threads)

    def cpu_sample(self, threads):
        # At most 1500 rows of A per timing (the config-1 product), best of 5.
        from oracle import oracle
        rows = min(self.m, 1500)
        a = self.a[:rows]
        best = float("inf")
        for _ in range(5):
            t0 = time.perf_counter()
            self._oracle_linear()(a, self.values, self.scales, self.n, self.k, self.bias, threads=threads)
            best = min(best, time.perf_counter() - t0)
        return 2.0 * rows * self.n * self.k / best / 1e12, f"{rows} rows of the product, best of 5"


WORKLOADS = {"granite": GraniteWorkload, "parakeet": ParakeetWorkload, "linear": LinearWorkload}
SPEECH = ("granite", "parakeet")


def make_workload(args, rank, world):
    if args.workload == "granite":
        return GraniteWorkload(rank, world, n_utt=args.utterances or 4096, precision=args.precision)
    if args.workload == "parakeet":
        return ParakeetWorkload(rank, world, n_utt=args.utterances or 256, precision=args.precision)
    shape = tuple(int(x) for x in args.shape.split(",")) if args.shape else None
    return LinearWorkload(rank, world, shape=shape, precision=args.precision)


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_ours(args, rank, world, local_rank):
    import torch
    import telmo_b200
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist_mod
        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local_rank))
        dist = dist_mod
    ctx = telmo_b200.Context(local_rank)
    wl = make_workload(args, rank, world)
    wl.setup_gpu(ctx)
    speech = args.workload in SPEECH

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        wl.step_gpu()
        if hasattr(wl, "between_steps"):
            wl.between_steps()
    wl.step_e2e()  # the host-buffer path's own buffers are allocated before timing
    ctx.check()
    if speech:
        wl.profile_start()
    clocks = Clocks(local_rank)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    clocks.start()
    time.sleep(0.3)
    for i in range(args.steps):
        if hasattr(wl, "between_steps"):
            wl.between_steps()
        starts[i].record()
        wl.step_gpu()
        ends[i].record()
    barrier()
    ctx.check()
    step_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    prof = None
    if speech:
        launches, prof = wl.profile_stop()
    else:
        launches = 2 * args.steps
    # e2e through the public call with host buffers.
    e_start = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e_end = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        if hasattr(wl, "between_steps"):
            wl.between_steps()
        e_start[i].record()
        wl.step_e2e()
        e_end[i].record()
    barrier()
    clk = clocks.stop()
    ctx.check()
    e2e_ms = sum(s.elapsed_time(e) for s, e in zip(e_start, e_end))
    # Every rank's own figures (device busy time of the timed steps, its share of the work), then
    # the whole job's: its time is the slowest rank's.
    mine = torch.tensor([step_ms, e2e_ms, wl.units_per_step(),
                         float(len(getattr(wl, "batches", [None])))], dtype=torch.float64, device="cuda")
    if dist:
        every = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
    else:
        every = [mine]
    every = [t.tolist() for t in every]
    step_ms = max(r[0] for r in every)
    e2e_ms = max(r[1] for r in every)
    total_units = sum(r[2] for r in every)
    if rank == 0:
        pk, pk_src = peaks()
        value = total_units * args.steps / (step_ms / 1e3)
        e2e_value = total_units * args.steps / (e2e_ms / 1e3)
        if speech:
            own_ms = every[0][0]  # the profile is rank 0's
            avg = prof["gemm_ms"] / max(prof["gemm_n"], 1) / 1e3
            ops_launch = prof["ops"] / max(prof["gemm_n"], 1)
            achieved = ops_launch / avg / 1e12
            peak = pk["bf16_tflops_sustained"]
            roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                        "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": None,
                        "traffic_note": "null: achieved averages launches of every product shape, "
                        "which no single ncu capture covers; a capture of the feed-forward "
                        "up-projection alone counts DRAM bytes below its algorithmic bytes",
                        "kernel": "gemm_i8x2_kernel (split-int8 tcgen05 linear)",
                        "ops_per_launch": ops_launch, "avg_launch_us": round(avg * 1e6, 2),
                        "peak_source": pk_src + ": bf16_tflops_sustained; the split-int8 "
                        "product issues two int8 MMAs per multiply-add, so its tensor ceiling "
                        "is the bf16 one",
                        "time_share": {"gemm": round(prof["gemm_ms"] / own_ms, 3),
                                       "attention": round(prof["attn_ms"] / own_ms, 3),
                                       "row_kernels_timed": round(prof["rows_ms"] / own_ms, 3),
                                       "front_end": round(prof["fe_ms"] / own_ms, 3)}}
        else:
            # One telmo_linear call (split quantization of A, then the tcgen05 product) against
            # its algorithmic bytes: A f32 read, W int8 read, scales and bias read, C f32 written.
            per_call_s = (every[0][0] / args.steps) / 1e3
            alg = wl.algorithmic_bytes()
            achieved = alg / per_call_s / 1e9
            roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                        "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": None,
                        "algorithmic_bytes": alg, "avg_launch_us": round(per_call_s * 1e6, 2),
                        "kernel": "telmo_linear: quantize_x2_regs_kernel + gemm_i8x2_kernel, timed "
                                  "together as one call",
                        "peak_source": pk_src + ": hbm_gbs"}
        cpu_value, cpu_sample = wl.cpu_sample(os.cpu_count() or 1)
        line = {
            "metric": wl.metric, "value": round(value, 2), "unit": wl.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(step_ms / args.steps, 3), "higher_is_better": True,
            "scaling": "strong" if speech else "weak", "vs_baseline": None,
            "dtype": "int8 x int8 -> i32 (split-int8 activations), f32/f64 elsewhere",
            "data": "synthetic (seeded; telmo_b200/synthetic.py), random-init weights",
            "config": wl.config(world),
            "e2e": {"value": round(e2e_value, 2), "unit": wl.unit,
                    "h2d_bytes_per_step": int(wl.bi), "d2h_bytes_per_step": int(wl.bo)},
            "roofline": roofline,
            "cpu_baseline": {"value": round(cpu_value, 3), "unit": wl.unit,
                             "cores": os.cpu_count(), "cpu_model": cpu_model(), "kind": "port",
                             "sample": cpu_sample},
            "clocks": clk,
            "gpu_launches": int(launches),
            "per_rank": [{"rank": r, "ms_per_step": round(v[0] / args.steps, 3),
                          "e2e_ms_per_step": round(v[1] / args.steps, 3),
                          "units_per_step": round(v[2], 3), "batches": int(v[3])}
                         for r, v in enumerate(every)],
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()


def run_reference(args, rank, world):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    wl = make_workload(args, 0, 1)
    if hasattr(wl, "cpu_setup"):
        wl.cpu_setup()
        per_step = wl.cpu_seconds
        sample = (f"the oracle's C restatement of telmo's CPU path (reference Rust not "
                  f"buildable here): {len(wl.cpu_utts)} utterances at evenly spaced length "
                  f"quantiles of the set ({wl.cpu_seconds:.1f} s of audio) per step, audio -> tokens")
    else:
        per_step = wl.units_per_step()
        sample = "the oracle's C restatement, full config-1 product per step"
    for _ in range(args.warmup):
        wl.cpu_step(threads)
    total = 0.0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        wl.cpu_step(threads)
        total += time.perf_counter() - t0
    value = per_step * args.steps / total
    line = {
        "impl": "reference", "metric": wl.metric, "value": round(value, 3), "unit": wl.unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 2), "higher_is_better": True,
        "scaling": "strong" if args.workload in SPEECH else "weak", "vs_baseline": None,
        "dtype": "f32 (int8 weights widened), f64 statistics",
        "data": "synthetic (seeded; telmo_b200/synthetic.py), random-init weights",
        "config": wl.config(world),
        "cpu_baseline": {"value": round(value, 3), "unit": wl.unit, "cores": threads,
                         "cpu_model": cpu_model(), "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": wl.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_load(args, rank):
    """Model load time: the config-5 Granite model's pack, held in host memory, to a finalized model
    on the device -- once from the reference's panel layout (repacked into rows on the host) and
    once from the device-layout pack (copied as it is). Wall clock around the load call, with the
    device synchronized on both sides; the median of the timed loads."""
    if rank != 0:
        return
    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": "the reference maps its pack and reads the "
                          "panels in place on the CPU; it has no device load to time"}), flush=True)
        return
    import torch
    import telmo_b200
    from telmo_b200 import synthetic
    from telmo_b200.granite import Granite
    from telmo_b200.pack import Pack, granite_config_json, write_pack
    torch.cuda.set_device(0)
    ctx = telmo_b200.Context(0)
    cfg = synthetic.granite_config()
    entries = synthetic.granite_entries(cfg, seed=1, scales="spec", precision=args.precision)
    panel = Pack(data=write_pack("granite-speech-ctc", dict(entries, **{"config.json": granite_config_json(cfg)})))
    del entries
    t0 = time.perf_counter()
    device = panel.to_device()
    convert_s = time.perf_counter() - t0

    def load(pack):
        torch.cuda.synchronize()
        t = time.perf_counter()
        model = Granite.from_pack(ctx, pack)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t
        model.close()
        return dt

    for _ in range(args.warmup):
        load(panel)
        load(device)
    panel_s = statistics.median([load(panel) for _ in range(args.steps)])
    device_s = statistics.median([load(device) for _ in range(args.steps)])
    line = {
        "metric": "model load seconds (pack in host memory -> finalized model on the device)",
        "value": round(device_s, 4), "unit": "s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(device_s * 1e3, 2), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic (random-init weights)",
        "config": {"workload": "load-config5-granite", "weights": args.precision,
                   "layout": "device-layout pack"},
        "panel_pack_s": round(panel_s, 4), "convert_s": round(convert_s, 4), "impl": "ours",
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["load"], default="granite",
                    help="load: model load time from a panel pack and from a device-layout pack")
    ap.add_argument("--shape", default="",
                    help="linear: M,K,N of another product (config 1's distributions), e.g. "
                         "53000,1024,4096 for an encoder's feed-forward up-projection")
    ap.add_argument("--precision", choices=["int8", "q8_0"], default="int8",
                    help="weight precision (the reference's Precision::Int8 or Q8_0)")
    ap.add_argument("--utterances", type=int, default=0,
                    help="utterances in the set (default: 4096 for granite, config 5; 256 for "
                         "parakeet, config 4; fewer for profiling)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload == "load":
        run_load(args, rank)
    elif args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
