"""Benchmark of the B200 gate/up path (quantize -> INT8 gate/up GEMM -> dequant -> SwiGLU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg2]

Prints ONE JSON line on rank 0.  A step is one pass of the hot path over one batch of synthetic input
(the BASELINE config named by ``--workload``; default ``cfg2``: the decode buckets M = 1, 8, 32, 64 at
K = 4096, H = 14336, one quantize + one gate/up launch each).  Under torchrun (N > 1) the intermediate
dimension H is sharded over the ranks: rank r owns gate rows [r*H/N, (r+1)*H/N) and the matching up
rows, every rank quantizes the replicated activations itself, and no collective runs on the path
(the total work is fixed, so the scaling is strong).  The step's public API calls are captured once
per rotating weight copy into CUDA graphs (as the reference runtime captures its decode steps) and
replayed.  Timing: W warm-up steps, then exactly K graph replays between barriers + synchronizes,
CUDA events on the launching stream, max over ranks.  Three copies of
the weights rotate between steps (3 x 117 MB > 126 MB L2), so no step finds its weights in L2.

The one-GPU cfg2 line also carries two records outside ``value``: ``prefill`` (the
INT8-TOPS half of the metric, through the same public API, with the GEMM's TOP/s against a live
``torch._int_mm`` measurement, twice the measured bf16 peak and the 4.5 POP/s datasheet figure) and
``ref_kernel`` (the reference's own GPU implementation, its Triton quantizer and its native_hybrid8
kernel built from source, timed per call on the same buckets and weights, next to ours).

The default workload's line also carries ``cfg4`` at every N: BASELINE config 4 (X [8192, 8192], H = 28672)
sharded the same way, per-rank GEMM TOP/s and the job's tokens/s.

``--impl reference`` times the reference arithmetic of the path on the host cores (the reference
ships no CPU implementation of it; the timed code is the oracle's restatement, ``oracle/``), on
rank 0 only: every bucket, every output column, one pass per step.
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
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "gate/up+SwiGLU tokens/s"

WORKLOADS = {
    # name: (buckets of M, K, H, activation kind, weight scale range, description)
    "cfg1": ((16,), 1024, 2816, "normal", (1e-3, 1e-2), "config 1: X [16, 1024], Wg/Wu int8 [2816, 1024]"),
    "cfg2": ((1, 8, 32, 64), 4096, 14336, "normal", (1e-3, 1e-2),
             "config 2 decode buckets M={1,8,32,64}, K=4096, Wg/Wu int8 [14336, 4096]"),
    "cfg3": ((4096,), 4096, 14336, "normal", (1e-3, 1e-2), "config 3 prefill: X [4096, 4096], Wg/Wu int8 [14336, 4096]"),
    "cfg4": ((8192,), 8192, 28672, "normal", (5e-4, 5e-3), "config 4: X [8192, 8192], Wg/Wu int8 [28672, 8192]"),
    "cfg5a": ((128, 512, 2048), 4096, 14336, "student", (1e-3, 1e-2),
              "config 5a: Student-t X (8 channels x50), buckets M={128,512,2048}, INT8 Wg/Wu [14336, 4096]"),
    "cfg5b": ((128, 512, 2048), 4096, 14336, "student", None,
              "config 5b: Student-t X, buckets M={128,512,2048}, BF16 Wg/Wu ~ N(0,0.02) [14336, 4096]"),
}
DEFAULT_WORKLOAD = "cfg2"
# The rotated INT8 down projection that consumes the gate/up output (reaxv2/assets.py:65-82 ->
# reaxv2/rotation.py): decode buckets, input width K = 9216, N = 2560 output columns, 4 rotated groups of
# 2304 columns, Walsh-Hadamard blocks of 256 (a reference rotation_g2304_b256 shape).
DOWN = dict(buckets=(1, 8, 32, 64), K=9216, N=2560, group=2304, parts=4, block=256)
DOWN_METRIC = "rotated INT8 down projection tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["down"], default=DEFAULT_WORKLOAD)
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffers) leg")
    ap.add_argument("--measure-int8-peak", action="store_true", help="print torch._int_mm int8 throughput and exit")
    ap.add_argument("--lane-sms", choices=("whole", "half", "weighted"), default="weighted",
                    help="SMs each of the two lanes' GEMMs are planned for (reax_set_stream_sms): a larger share "
                         "for the lane holding the largest bucket (weighted), half each, or the whole GPU each")
    ap.add_argument("--emulate-shard", type=int, default=1,
                    help="one GPU runs rank 0's H shard of an N-way job (a diagnostic of per-rank latency)")
    ap.add_argument("--no-side-records", action="store_true",
                    help="skip the prefill and reference-kernel records of the one-GPU cfg2 line")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    return a


# -------------------------------------------------------------------------------------------------- inputs
def make_inputs(name: str, rank: int, world: int, copies: int):
    """Seeded synthetic inputs on the CPU (same on every rank), this rank's H shard on the GPU."""
    buckets, K, H, kind, srange, _ = WORKLOADS[name]
    g = torch.Generator().manual_seed(20261201)
    xs = []
    for M in buckets:
        if kind == "normal":
            x = torch.randn(M, K, generator=g)
        else:
            normal = torch.randn(M, K, generator=g)
            chi2 = torch.randn(M, K, 3, generator=g).square().sum(-1)
            x = normal / torch.sqrt(chi2 / 3.0)
            idx = torch.arange(8) * (K // 8) + 3
            x[:, idx] *= 50.0
        xs.append(x.to(torch.bfloat16))
    h = H // world
    rows = torch.cat([torch.arange(rank * h, (rank + 1) * h), H + torch.arange(rank * h, (rank + 1) * h)])
    dev = torch.device("cuda", torch.cuda.current_device())
    banks = []
    for c in range(copies):
        gc = torch.Generator().manual_seed(1000 + c)
        if srange is None:
            w = (torch.randn(2 * H, K, generator=gc) * 0.02).to(torch.bfloat16)[rows].contiguous()
            banks.append(dict(w=w.to(dev)))
        else:
            w = torch.randint(-127, 128, (2 * H, K), generator=gc, dtype=torch.int8)[rows].contiguous()
            lo, hi = srange
            sw = (lo + (hi - lo) * torch.rand(2 * H, generator=gc))[rows].contiguous()
            from types import SimpleNamespace
            banks.append(SimpleNamespace(width=K, centered=False, low_columns=torch.arange(K, dtype=torch.int32, device=dev),
                                         high_columns=torch.zeros(0, dtype=torch.int32, device=dev),
                                         low_weight=w.to(dev), high_weight=torch.zeros(2 * h, 0, dtype=torch.bfloat16, device=dev),
                                         smoothing=torch.ones(K, device=dev), centers=torch.zeros(K, device=dev),
                                         scales=sw.to(dev), bias=torch.zeros(2 * h, device=dev)))
    return xs, banks, h


def gemm_bytes(M, K, h, int8=True):
    """Algorithmic DRAM bytes of one gate/up GEMM launch: weights + per-channel scale and bias,
    the activation operand, per-row scales, the bf16 output."""
    if int8:
        return 2 * h * K + 2 * h * 8 + M * K + M * 4 + M * h * 2
    return 2 * h * K * 2 + M * K * 2 + M * h * 2


def gemm_ops(M, K, h):
    return 2 * M * (2 * h) * K


# -------------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        for ln in self.lines:
            f = [v.strip() for v in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# -------------------------------------------------------------------------------------------------- helpers
def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def int8_peak():
    """Measured dense INT8 throughput on this pool (torch._int_mm 8192^3, recorded under profiles/)."""
    p = ROOT / "profiles" / "int8_peak.json"
    if p.exists():
        return json.loads(p.read_text())
    return None


def ncu_traffic(workload):
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        return json.loads(p.read_text()).get(workload)
    return None


def deal_lanes(buckets):
    """Two lanes, as the reference runtime replays two lanes' graphs at the same time
    (runtime/bootstrap.py:29, vendor/s1eng/s1eng/kprio.py:1-4): the buckets, largest first, dealt to the
    lanes from both ends (cfg2: M = 64 then 1 on one lane, 32 then 8 on the other).  Returns the lanes
    (lists of bucket indices, empty ones dropped) and each bucket's slot, its place in the interleaved
    call order."""
    order = sorted(range(len(buckets)), key=lambda j: -buckets[j])
    lanes = [[], []]
    for k in range((len(order) + 1) // 2):
        lanes[k % 2] += sorted({order[k], order[len(order) - 1 - k]}, key=lambda j: -buckets[j])
    lanes = [ln for ln in lanes if ln]
    return lanes, {j: 2 * k + l for l, ln in enumerate(lanes) for k, j in enumerate(ln)}


def lane_runner(lanes, dev, side=None):
    """run(work): work(j) for every bucket, lane 0 on the current stream and lane 1 on a side stream
    forked from and joined to it (inside a graph capture too)."""
    side = side if side is not None else torch.cuda.Stream(dev)

    def run(work):
        main = torch.cuda.current_stream(dev)
        outs = []
        if len(lanes) > 1:
            side.wait_stream(main)
        for l, ln in enumerate(lanes):
            with torch.cuda.stream(main if l == 0 else side):
                outs += [work(j) for j in ln]
        if len(lanes) > 1:
            main.wait_stream(side)
        return outs
    return run


# Share of the SMs for the first lane (the one holding the largest bucket, whose GEMM has the longest
# epilogue) under --lane-sms weighted: 78 of 148.  Measured on cfg2 (one B200, 60 steps per point): step
# 92.6-93.0 us at 74/74, 90.2 us at 77/71, 90.6-90.8 at 80/68, 90.4 at 83/65, 92.7 at 86/62.
LANE0_SHARE = 0.527


class LaneShares:
    """With two lanes: each lane's GEMMs are planned for a share of the SMs (reax_set_stream_sms), so the
    two lanes' persistent grids run side by side (``--lane-sms weighted``: LANE0_SHARE for the first lane,
    ``half``: half each); used around the capture of the step graphs, which keep the plans they were
    captured with."""

    def __init__(self, streams, dev, enabled, weighted=False):
        self.streams = streams if enabled and len(streams) > 1 else []
        self.sms = torch.cuda.get_device_properties(dev).multi_processor_count
        first = round(self.sms * LANE0_SHARE) if weighted else self.sms // 2
        self.split = [first, self.sms - first]

    def __enter__(self):
        from reax_engine_runtime_v3_b200 import _native
        for i, st in enumerate(self.streams):
            _native.set_stream_sms(st, self.split[0] if i == 0 else self.split[1])
        return self

    def __exit__(self, *exc):
        from reax_engine_runtime_v3_b200 import _native
        for st in self.streams:
            _native.set_stream_sms(st, 0)
        return False


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()


# -------------------------------------------------------------------------------------------------- CPU legs
class CpuSample:
    """The oracle's restatement of the path (the reference ships no CPU implementation of it) on the
    host cores: every bucket of the workload, all output columns, rows capped at 512 per bucket on the
    prefill buckets.  One pass = one step of that sample."""

    MAX_ROWS = 512

    def __init__(self, name: str):
        from oracle import reax_oracle as ro
        self.ro = ro
        buckets, K, H, kind, srange, _ = WORKLOADS[name]
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        g = np.random.default_rng(7)
        self.int8 = srange is not None
        self.K = K
        if self.int8:
            from types import SimpleNamespace
            w = g.integers(-127, 128, (2 * H, K), dtype=np.int8)
            sw = (1e-3 + 9e-3 * g.random(2 * H)).astype(np.float32)
            self.bank = SimpleNamespace(low_columns=np.arange(K), high_columns=np.zeros(0, np.int64),
                                        smoothing=np.ones(K, np.float32), centers=np.zeros(K, np.float32),
                                        centered=False, low_weight=w, high_weight=np.zeros((2 * H, 0), np.uint16),
                                        scales=sw, bias=np.zeros(2 * H, np.float32))
        else:
            self.wb = ro.f32_to_bf16((g.standard_normal((2 * H, K)) * 0.02).astype(np.float32))
        self.xs = [ro.f32_to_bf16(g.standard_normal((min(M, self.MAX_ROWS), K)).astype(np.float32)) for M in buckets]
        self.tokens = sum(len(x) for x in self.xs)
        self.H = H

    def one_pass(self) -> float:
        t0 = time.perf_counter()
        for x in self.xs:
            if self.int8:
                self.ro.gate_up_project(x, self.bank)
            else:
                self.ro.gate_up_bf16(x, self.wb, 0, dict(parts=1, chunk=self.K), dict(parts=1, chunk=self.K))
        return time.perf_counter() - t0

    def describe(self, passes: int, seconds: float) -> str:
        return (f"{passes} passes over buckets {[len(x) for x in self.xs]} rows x all {self.H} output columns, "
                f"{seconds:.1f} s")


def cpu_run(name: str, budget_s: float = 12.0):
    """Tokens/s of the CPU port over a bounded sample of the workload (CpuSample), as many passes as fit
    in the budget (at most 50)."""
    sample = CpuSample(name)
    sample.one_pass()                      # first-touch of the weights
    passes, total = 0, 0.0
    while total < budget_s and passes < 50:
        total += sample.one_pass()
        passes += 1
    return sample.tokens * passes / total, sample.threads, sample.describe(passes, total)


def run_reference(args, world, rank):
    if rank != 0:
        return 0
    if args.workload == "down":
        return run_down_reference(args)
    buckets, K, H, kind, srange, desc = WORKLOADS[args.workload]
    sample = CpuSample(args.workload)
    for _ in range(args.warmup):
        sample.one_pass()
    times = [sample.one_pass() for _ in range(args.steps)]
    ms = statistics.median(times) * 1e3
    tok_s = sample.tokens / (ms * 1e-3)
    desc_sample = sample.describe(args.steps, sum(times)) + " (median pass is the step)"
    line = {"impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "s8" if srange else "bf16",
            "data": "synthetic", "config": {"workload": desc, "parallelism": "host cores",
                                            "tokens_per_step": sample.tokens},
            "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": sample.threads, "kind": "port",
                             "sample": desc_sample},
            "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------- down projection workload
def down_inputs(copies):
    from types import SimpleNamespace
    g = torch.Generator().manual_seed(20261202)
    K, N, G, P, B = DOWN["K"], DOWN["N"], DOWN["group"], DOWN["parts"], DOWN["block"]
    xs = [torch.randn(M, K, generator=g).to(torch.bfloat16) for M in DOWN["buckets"]]
    dev = torch.device("cuda", torch.cuda.current_device())
    banks = []
    for c in range(copies):
        gc = torch.Generator().manual_seed(2000 + c)
        banks.append(SimpleNamespace(
            width=K, parts=P, group=G, block=B, chunk=K // P, hp=0,
            centers=(torch.randn(K, generator=gc) * 0.05).to(dev),
            low_weight=torch.randint(-127, 128, (N, P * G), generator=gc, dtype=torch.int8).to(dev),
            high_weight=torch.zeros(N, 0, dtype=torch.bfloat16, device=dev),
            scales=(1e-3 + 9e-3 * torch.rand(P, N, generator=gc)).to(dev),
            bias=(torch.randn(P, N, generator=gc) * 0.05).to(dev)))
    return xs, banks


def down_cpu_run(budget_s: float = 12.0):
    """The oracle's rotated projection on the host cores over a bounded sample (all buckets, 256 of the
    N output columns), scaled to full width."""
    from types import SimpleNamespace
    from oracle import reax_oracle as ro
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    K, N, G, P, B = DOWN["K"], DOWN["N"], DOWN["group"], DOWN["parts"], DOWN["block"]
    g = np.random.default_rng(9)
    cols = 256
    bank = SimpleNamespace(parts=P, group=G, block=B, chunk=K // P, centers=(g.standard_normal(K) * 0.05).astype(np.float32),
                           low_weight=g.integers(-127, 128, (cols, P * G), dtype=np.int8),
                           scales=(1e-3 + 9e-3 * g.random((P, cols))).astype(np.float32),
                           bias=(g.standard_normal((P, cols)) * 0.05).astype(np.float32))
    xs = [ro.f32_to_bf16(g.standard_normal((M, K)).astype(np.float32)) for M in DOWN["buckets"]]
    tokens = sum(len(x) for x in xs)
    t0 = time.perf_counter()
    passes = 0
    while True:
        for x in xs:
            ro.rotated_project(x, bank)
        passes += 1
        if time.perf_counter() - t0 > budget_s or passes >= 50:
            break
    dt = time.perf_counter() - t0
    sample = (f"{passes} passes over buckets {list(len(x) for x in xs)} rows x {cols}/{N} output columns "
              f"(scaled to full width), {dt:.1f} s")
    return tokens * passes / dt * (cols / N), threads, sample


def down_desc():
    return (f"rotated INT8 down projection, decode buckets M={{1,8,32,64}}, K={DOWN['K']}, N={DOWN['N']}, "
            f"{DOWN['parts']} groups of {DOWN['group']}, Walsh-Hadamard blocks of {DOWN['block']}")


def run_down_reference(args):
    times = []
    threads, sample = os.cpu_count() or 1, ""
    for i in range(args.warmup + args.steps):
        v, threads, sample = down_cpu_run(budget_s=1.5 if args.steps > 20 else 4.0)
        if i >= args.warmup:
            times.append(v)
    tok_s = statistics.median(times)
    line = {"impl": "reference", "metric": DOWN_METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sum(DOWN["buckets"]) / tok_s * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "s8", "data": "synthetic",
            "config": {"workload": down_desc(), "parallelism": "host cores"},
            "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_down(args, world, rank, local):
    """The rotated down projection (rotated quantizer -> grouped INT8 partials -> ordered fold) through the
    reference's API (reaxv2.rotation.Native.project), timed like the gate/up step."""
    if world > 1:
        if rank == 0:
            print(json.dumps({"error": "the down workload runs on one GPU"}), flush=True)
        torch.distributed.destroy_process_group()
        return 0
    from reax_engine_runtime_v3_b200.reaxv2.rotation import Native as Rotation, quantize_rotated
    from reax_engine_runtime_v3_b200.reaxv2.sliced import Native as Sliced, sliced_i8
    K, N, G, P, B = DOWN["K"], DOWN["N"], DOWN["group"], DOWN["parts"], DOWN["block"]
    buckets = DOWN["buckets"]
    copies = 3
    dev = torch.device("cuda", local)
    xs_cpu, banks = down_inputs(copies)
    xs = [x.to(dev) for x in xs_cpu]
    native = Rotation(Sliced(None), None, 128)

    lanes, slot_of = deal_lanes(buckets)
    side = torch.cuda.Stream(dev)
    run_lanes = lane_runner(lanes, dev, side)

    def bank_of(i, j):
        return banks[(4 * i + slot_of[j]) % copies]

    def step(i):
        return run_lanes(lambda j: native.project(xs[j], bank_of(i, j), "slice_m128n256"))

    cap = torch.cuda.Stream(dev)
    cap.wait_stream(torch.cuda.current_stream(dev))
    # each lane's grouped GEMMs planned for half of the SMs, as in the gate/up step
    shares = LaneShares([cap, side], dev, args.lane_sms != "whole" and len(lanes) > 1, args.lane_sms == "weighted")

    def graphs_of(fn):
        gs = []
        for c in range(copies):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                fn(c)
            gs.append(g)
        return gs

    def timed(gs, n):
        for i in range(args.warmup):
            gs[i % len(gs)].replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cap)
        for i in range(n):
            gs[i % len(gs)].replay()
        e1.record(cap)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    with torch.cuda.stream(cap):
        with shares:
            for i in range(args.warmup):
                step(i)
            torch.cuda.synchronize()
            graphs = graphs_of(step)
        sampler = ClockSampler(local)
        sampler.start()
        ms = timed(graphs, args.steps)
        clocks = sampler.stop()
        # dominant kernel (the grouped INT8 GEMM) and the quantizer, back to back per bucket
        # (the GEMM as the step runs it, weight stream started before its dependency wait, and once more
        # as the plain reax_sliced_i8, which waits first)
        per_gemm, per_gemm_plain, per_quant = [], [], []
        for x in xs:
            M = x.shape[0]
            low, sc = quantize_rotated(x, banks[0].centers, K // P, P, G, B)
            parts_buf = torch.empty(P, M, N, dtype=torch.bfloat16, device=dev)
            reps = 3 * copies
            for static, dst in ((True, per_gemm), (False, per_gemm_plain)):
                gg = graphs_of(lambda c: [sliced_i8(low, banks[r % copies].low_weight, None, None, sc,
                                                    banks[r % copies].scales, banks[r % copies].bias, parts_buf, G, 0,
                                                    P, static_weights=static) for r in range(reps)])
                dst.append((M, timed(gg, max(2, args.steps // reps)) * 1e-3 / reps))
                del gg
            gq = graphs_of(lambda c: [quantize_rotated(x, banks[r % copies].centers, K // P, P, G, B) for r in range(reps)])
            per_quant.append((M, timed(gq, max(2, args.steps // reps)) * 1e-3 / reps))
            del gq
        # end to end with host buffers (inputs from pinned memory, outputs back), copies on side streams
        xs_host = [x.pin_memory() for x in xs_cpu]
        outs_host = [torch.empty((x.shape[0], N), dtype=torch.bfloat16).pin_memory() for x in xs_cpu]
        xs_dev = [torch.empty_like(x, device=dev) for x in xs_cpu]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        order = sorted(range(len(buckets)), key=lambda j: -buckets[j])

        def e2e_step(i):
            main = torch.cuda.current_stream(dev)
            s_in.wait_stream(main)
            s_out.wait_stream(main)
            arrived = []
            with torch.cuda.stream(s_in):
                for j in order:
                    xs_dev[j].copy_(xs_host[j], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(s_in)
                    arrived.append(ev)
            outs = []
            for j, ev in zip(order, arrived):
                main.wait_event(ev)
                o = native.project(xs_dev[j], bank_of(i, j), "slice_m128n256")
                outs.append(o)
                done = torch.cuda.Event()
                done.record(main)
                s_out.wait_event(done)
                with torch.cuda.stream(s_out):
                    outs_host[j].copy_(o, non_blocking=True)
            main.wait_stream(s_in)
            main.wait_stream(s_out)
            return outs
        e2e_step(0)
        torch.cuda.synchronize()
        eg = graphs_of(e2e_step)
        ems = timed(eg, args.steps)
        # the last replay's read-back must equal the device path's outputs for the same weight copies
        last = (args.steps - 1) % copies
        for j, x in enumerate(xs):
            o = native.project(x, bank_of(last, j), "slice_m128n256")
            if not torch.equal(o.cpu(), outs_host[j]):
                raise RuntimeError(f"down e2e read-back of bucket M={x.shape[0]} differs from the device path")
        status = 0
        del eg, graphs
    tokens = sum(buckets)
    peaks, peak_kind = measured_peaks()
    by = sum(N * P * G + P * N * 8 + M * P * G + P * M * 4 + P * M * N * 2 for M, _ in per_gemm)
    dur = sum(d for _, d in per_gemm)
    achieved = by / dur / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "peak_source": f"{peak_kind} hbm_gbs",
                "traffic": ncu_traffic("down"),
                "kernel": "grouped INT8 GEMM (tc_gemm_kernel, plain epilogue, one partial per group)",
                "how": "back-to-back launches on the whole GPU (weight-major tiles of one wave); the two-lane step "
                       "plans each lane for half of the SMs, where the groups' columns need two waves of those "
                       "tiles and the token-major tiles run instead",
                "per_launch_us": {str(M): round(d * 1e6, 2) for M, d in per_gemm},
                "per_launch_us_plain": {str(M): round(d * 1e6, 2) for M, d in per_gemm_plain},
                "quantizer_per_launch_us": {str(M): round(d * 1e6, 2) for M, d in per_quant}}
    cpu = None
    if not args.no_cpu_baseline:
        v, threads, sample = down_cpu_run()
        cpu = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample}
    line = {"metric": DOWN_METRIC, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "s8",
            "data": "synthetic (seeded N(0,1) activations, uniform int8 rotated weights)",
            "config": {"workload": down_desc(), "tokens_per_step": tokens, "parallelism": "1 GPU",
                       "lanes": [[buckets[j] for j in ln] for ln in lanes],
                       "lane_sms": shares.split if shares.streams else "whole GPU",
                       "l2": f"{copies} rotating weight copies, a different copy on consecutive calls"},
            "roofline": roofline, "cpu_baseline": cpu,
            "e2e": {"value": tokens / (ems * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": sum(x.numel() * 2 for x in xs_cpu),
                    "d2h_bytes_per_step": sum(x.shape[0] * N * 2 for x in xs_cpu),
                    "how": "public API calls captured into CUDA graphs; H2D and D2H on side streams"},
            "gpu_launches": args.steps * len(buckets) * 3, "clocks": clocks, "device_status": status,
            "timing": "CUDA-graph replay of the captured step"}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------ side records of the cfg2 line
def graph_time(fn, reps, n_rep, cap):
    """Seconds per call of fn(0), ..., fn(reps - 1) captured back to back in one CUDA graph on stream
    `cap` and replayed n_rep times (CUDA events on `cap`).  Call with `cap` current.  Every call runs
    once eagerly first, so that anything a call prepares on first use (the dense-bank check of
    gate_up.Native.project) is done outside the capture."""
    for r in range(reps):
        fn(r)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=cap):
        for r in range(reps):
            fn(r)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cap)
    for _ in range(n_rep):
        g.replay()
    e1.record(cap)
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e-3 / (n_rep * reps)


def int_mm_tops(n=8192, tries=5):
    """Dense INT8 tensor throughput on this GPU now: torch._int_mm at n^3, best of `tries` (CUDA events)."""
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda").t()
    for _ in range(2):
        torch._int_mm(a, b)
    best = None
    for _ in range(tries):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) * 1e-3
        best = t if best is None else min(best, t)
    del a, b
    return 2 * n ** 3 / best / 1e12


def prefill_record(banks, dev, cap, steps):
    """BASELINE config 3 (the INT8-TOPS half of the metric) through the public API, on the cfg2 weight
    copies (same K, H and weight distribution): X bf16 [4096, 4096] ~ N(0,1).  Per call of
    gate_up.Native.project (quantize + gate/up), per GEMM launch and per quantizer launch, with the GEMM's
    TOP/s against three denominators."""
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import Native, gate_up_i8, project_quantizer
    _, K, H, _, _, desc = WORKLOADS["cfg3"]
    M = 4096
    gx = torch.Generator().manual_seed(20261201)
    x = torch.randn(M, K, generator=gx).to(torch.bfloat16).to(dev)
    nat = Native(None)
    copies = len(banks)
    n_rep = max(3, steps // copies)
    with torch.cuda.stream(cap):
        call = graph_time(lambda r: nat.project(x, banks[r % copies], "hybrid8_b128n256_s64n256"), copies, n_rep, cap)
        low, high, sc = project_quantizer(x, banks[0])
        gemm = graph_time(lambda r: gate_up_i8(low, banks[r % copies].low_weight, high, banks[r % copies].high_weight,
                                               sc, banks[r % copies].scales, banks[r % copies].bias,
                                               static_weights=True), copies, n_rep, cap)
        quant = graph_time(lambda r: project_quantizer(x, banks[r % copies]), copies, n_rep, cap)
    ops = gemm_ops(M, K, H)
    tops = ops / gemm / 1e12
    live = int_mm_tops()
    peaks, kind = measured_peaks()
    return {"workload": desc, "tokens_per_s": M / call, "call_us": call * 1e6, "gemm_us": gemm * 1e6,
            "quant_us": quant * 1e6, "gemm_tops": tops, "call_tops": ops / call / 1e12,
            "frac": {"torch_int_mm_live": tops / live, "twice_bf16_burst": tops / (2 * peaks["bf16_tflops"]),
                     "datasheet_dense_int8": tops / 4500.0},
            "denominators_tops": {"torch_int_mm_live": live, "twice_bf16_burst": 2 * peaks["bf16_tflops"],
                                  "datasheet_dense_int8": 4500.0},
            "how": "CUDA graphs of back-to-back calls over the 3 rotating weight copies; GEMM as "
                   "reax_gate_up_i8_static on pre-quantized codes; torch._int_mm 8192^3 best of 5 measured in this run"}


def cfg4_record(rank, world, dev, cap, steps):
    """BASELINE config 4, the large MLP N-sharded over the ranks: X bf16 [8192, 8192] replicated, this
    rank's H / world gate rows and the matching up rows of Wg/Wu int8 [28672, 8192], per-channel scales
    U(5e-4, 5e-3).  Per rank: one gate_up.Native.project call (the replicated quantizer + this rank's
    GEMM) and the GEMM alone, CUDA graphs over two weight copies, max over ranks.  tokens_per_s is the
    job's (every rank produces its columns of all 8192 rows at once)."""
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import Native, gate_up_i8, project_quantizer
    xs_cpu, banks, h = make_inputs("cfg4", rank, world, 2)
    _, K, H, _, _, desc = WORKLOADS["cfg4"]
    x = xs_cpu[0].to(dev)
    M = x.shape[0]
    nat = Native(None)
    n_rep = max(2, steps // 4)
    with torch.cuda.stream(cap):
        call = graph_time(lambda r: nat.project(x, banks[r % 2], "hybrid8_b128n256_s64n256"), 2, n_rep, cap)
        low, high, sc = project_quantizer(x, banks[0])
        gemm = graph_time(lambda r: gate_up_i8(low, banks[r % 2].low_weight, high, banks[r % 2].high_weight, sc,
                                               banks[r % 2].scales, banks[r % 2].bias, static_weights=True), 2, n_rep,
                          cap)
        quant = graph_time(lambda r: project_quantizer(x, banks[r % 2]), 2, n_rep, cap)
    call, gemm, quant = (max_over_ranks(v, world) for v in (call, gemm, quant))
    del banks, x, low, high, sc
    torch.cuda.empty_cache()
    return {"workload": desc, "H_per_rank": h, "tokens_per_s": M / call, "call_us": call * 1e6,
            "gemm_us": gemm * 1e6, "quant_us": quant * 1e6, "gemm_tops_per_rank": gemm_ops(M, K, h) / gemm / 1e12,
            "how": "per rank: CUDA graphs of back-to-back calls over 2 weight copies, max over ranks; the quantizer "
                   "runs on every rank over the replicated activations; no collective"}


def ref_kernel_record(banks, xs, dev, cap, steps):
    """The reference's own implementation of the path on this GPU, as reaxv2.gate_up.Native.project runs
    it (reaxv2/gate_up.py:29-37): its Triton _prepare, compiled ahead of time from the unmodified source,
    then its native_hybrid8 kernel (kernel-source/legacy-v2/src/native_hybrid8.cu, built from source for
    sm_100a), the best hybrid8_* configuration per bucket, against ours on the same inputs, weights and
    L2 rotation.  Both are timed per call (serially), outside `value`; outputs are compared once."""
    from oracle import ref_gpu
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import Native
    name0 = ref_gpu.TritonQuantizer.prepare_name(4096, 4096, 0, False)
    if not (ref_gpu.available("native_hybrid8.cubin") and ref_gpu.TritonQuantizer.available(name0)):
        return {"unavailable": "reference kernels not built into oracle/_ref (oracle/build_ref.py)"}
    hy, tq = ref_gpu.Hybrid8(), ref_gpu.TritonQuantizer()
    nat = Native(None)
    copies = len(banks)
    n_rep = max(3, steps // copies)

    def ref_project(x, b, name):
        low, high, sc = tq.prepare(x, b.low_columns, b.high_columns, b.smoothing, b.centers, b.centered)
        return hy.product(low, b.low_weight, high, b.high_weight, sc, b.scales, b.bias, name)

    rec = {}
    with torch.cuda.stream(cap):
        for x in xs:
            M = x.shape[0]
            best = None
            for name in ref_gpu.HYBRID:
                t = graph_time(lambda r: ref_project(x, banks[r % copies], name), copies, n_rep, cap)
                if best is None or t < best[0]:
                    best = (t, name)
            ours = graph_time(lambda r: nat.project(x, banks[r % copies], "hybrid8_b128n256_s64n256"), copies, n_rep, cap)
            same = torch.equal(ref_project(x, banks[0], best[1]).view(torch.int16),
                               nat.project(x, banks[0], "hybrid8_b128n256_s64n256").view(torch.int16))
            rec[str(M)] = {"ref_us": round(best[0] * 1e6, 2), "ref_config": best[1], "ours_us": round(ours * 1e6, 2),
                           "speedup": best[0] / ours, "outputs_bit_identical": same}
    return {"per_bucket": rec, "how": "CUDA graphs of back-to-back calls over the 3 rotating weight copies, "
                                      "quantize + gate/up per call, best reference hybrid8_* config per bucket"}


# -------------------------------------------------------------------------------------------------- GPU leg
def main():
    args = parse()
    world, rank, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, world, rank)
    if not torch.cuda.is_available():
        print(json.dumps({"error": "no CUDA device"}))
        return 1
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    if args.measure_int8_peak:
        return measure_int8_peak()
    if args.workload == "down":
        return run_down(args, world, rank, local)

    from reax_engine_runtime_v3_b200 import _native
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import Native
    from reax_engine_runtime_v3_b200.runtime.mixed_origin_bf16 import Native as Bf16Native

    buckets, K, H, kind, srange, desc = WORKLOADS[args.workload]
    int8 = srange is not None
    copies = 3
    shard_world = args.emulate_shard if world == 1 and args.emulate_shard > 1 else world
    xs_cpu, banks, h = make_inputs(args.workload, rank, shard_world, copies)
    dev = torch.device("cuda", local)
    xs = [x.to(dev) for x in xs_cpu]
    gate_up = Native(None)
    bf16 = Bf16Native()
    stream = torch.cuda.current_stream()

    # The step's buckets run on two lanes (deal_lanes).  Consecutive calls on a lane, and calls running
    # at the same time, always read different weight copies.
    order = sorted(range(len(buckets)), key=lambda j: -buckets[j])
    lanes, slot_of = deal_lanes(buckets)
    side = torch.cuda.Stream(dev)
    run_lanes = lane_runner(lanes, dev, side)

    def bank_of(i, j):
        return banks[(4 * i + slot_of[j]) % copies]

    def step(i, inputs=None):
        xs_ = inputs or xs

        def work(j):
            b = bank_of(i, j)
            return gate_up.project(xs_[j], b, "hybrid8_b128n256_s64n256") if int8 else bf16.gate_up(xs_[j], b["w"])
        return run_lanes(work)

    # Every timed loop replays CUDA graphs captured from the public API calls, as the reference runtime
    # replays its captured decode steps (runtime/capture.py); one graph per rotating weight copy.  The
    # capture stream gets its workspace during the eager warm-up, so nothing is allocated or zeroed
    # inside a graph.
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(torch.cuda.current_stream(dev))
    shares = LaneShares([cap, side], dev, args.lane_sms != "whole" and len(lanes) > 1, args.lane_sms == "weighted")
    with torch.cuda.stream(cap), shares:
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        # eager steps, for reference only (host launch overhead included)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cap)
        for i in range(args.warmup):
            step(i)
        e1.record(cap)
        torch.cuda.synchronize()
        eager_ms = e0.elapsed_time(e1) / args.warmup
        graphs = []
        for c in range(copies):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                step(c)
            graphs.append(g)
        for i in range(args.warmup):
            graphs[i % copies].replay()
        _native.clear_status(_native.workspace(dev))
    barrier(world)

    sampler = ClockSampler(local)
    if rank == 0 or world > 1:
        sampler.start()
    barrier(world)
    with torch.cuda.stream(cap):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(cap)
        for i in range(args.steps):
            graphs[i % copies].replay()
        ev1.record(cap)
    barrier(world)
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    ms = max_over_ranks(ms, world)
    with torch.cuda.stream(cap):
        status = _native.read_status(_native.workspace(dev))
    tokens = sum(buckets)
    value = tokens / (ms * 1e-3)
    launches = args.steps * len(buckets) * (2 if int8 else 1)

    # dominant kernel (the GEMM) alone: a graph of back-to-back launches over the rotating weight
    # copies, timed with events on its stream; per launch = replay time / launches (gaps included).  The
    # INT8 GEMM is timed as the step runs it, with its weight stream started before its dependency wait
    # (reax_project_i8 launches it that way behind the quantizer; here through reax_gate_up_i8_static),
    # and once more as the plain reax_gate_up_i8, which waits first (per_launch_us_plain).
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import gate_up_i8, quantize_rows
    per_bucket, per_bucket_plain = [], []
    reps = 3 * copies
    with torch.cuda.stream(cap):
        pre = [quantize_rows(x, banks[0]) for x in xs] if int8 else None
        for bi, x in enumerate(xs):
            M = x.shape[0]
            for static in ((True, False) if int8 else (False,)):
                def gemm(r):
                    b = banks[r % copies]
                    if int8:
                        low, high, sc = pre[bi]
                        gate_up_i8(low, b.low_weight, high, b.high_weight, sc, b.scales, b.bias,
                                   static_weights=static)
                    else:
                        bf16.gate_up(x, b["w"])
                gemm(0)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=cap):
                    for r in range(reps):
                        gemm(r)
                for _ in range(2):
                    g.replay()
                torch.cuda.synchronize()
                n_rep = max(1, args.steps // reps) + 2
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(cap)
                for _ in range(n_rep):
                    g.replay()
                e1.record(cap)
                torch.cuda.synchronize()
                d = e0.elapsed_time(e1) * 1e-3 / (n_rep * reps)
                d = max_over_ranks(d, world)
                (per_bucket if static or not int8 else per_bucket_plain).append((M, d))
                del g
    peaks, peak_kind = measured_peaks()
    # The bound is the roof that dominates the launches' ideal time: each bucket's ideal is the larger of
    # its bytes over the HBM peak and its ops over the tensor peak (decode buckets are HBM-bound, large
    # ones tensor-bound; mixed buckets, as in cfg5, take the roof that most of their ideal time is spent
    # under).  achieved = that roof's quantity summed over the buckets / their summed launch time.
    if int8:
        ip = int8_peak()
        t_peak = ip["tops"] if ip else 4500.0
        t_src = "measured torch._int_mm int8" if ip else "datasheet dense INT8 (no measured int8 peak)"
    else:
        t_peak = peaks["bf16_tflops"]
        t_src = f"{peak_kind} bf16_tflops"
    ideal_hbm = sum(gemm_bytes(M, K, h, int8) / (peaks["hbm_gbs"] * 1e9) for M, _ in per_bucket
                    if gemm_bytes(M, K, h, int8) / (peaks["hbm_gbs"] * 1e9) >= gemm_ops(M, K, h) / (t_peak * 1e12))
    ideal_tc = sum(gemm_ops(M, K, h) / (t_peak * 1e12) for M, _ in per_bucket
                   if gemm_bytes(M, K, h, int8) / (peaks["hbm_gbs"] * 1e9) < gemm_ops(M, K, h) / (t_peak * 1e12))
    dur = sum(d for _, d in per_bucket)
    if ideal_tc > ideal_hbm:
        achieved = sum(gemm_ops(M, K, h) for M, _ in per_bucket) / dur / 1e12
        roofline = {"bound": "tensor", "achieved": achieved, "peak": t_peak, "unit": "TOP/s" if int8 else "TFLOP/s",
                    "frac": achieved / t_peak, "peak_source": t_src}
    else:
        achieved = sum(gemm_bytes(M, K, h, int8) for M, _ in per_bucket) / dur / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": achieved / peaks["hbm_gbs"], "peak_source": f"{peak_kind} hbm_gbs"}
    # the committed capture is of the one-GPU launch; a rank of a sharded job moves 1/N of its bytes
    # ncu DRAM bytes per launch of this rank's GEMM: the unsharded workload's, or the 8-way shard's
    roofline["traffic"] = ncu_traffic(args.workload if shard_world == 1 else f"{args.workload}_shard{shard_world}")
    roofline["per_launch_us"] = {str(M): round(d * 1e6, 2) for M, d in per_bucket}
    if per_bucket_plain:
        roofline["per_launch_us_plain"] = {str(M): round(d * 1e6, 2) for M, d in per_bucket_plain}

    # Side records of the one-GPU default line (outside `value`): the prefill half of the metric (cfg3)
    # and the reference's own GPU implementation on the same buckets.
    prefill = ref_kernel = cfg4 = None
    if shard_world == world and args.workload == DEFAULT_WORKLOAD and int8 and not args.no_side_records:
        cfg4 = cfg4_record(rank, world, dev, cap, args.steps)
    if world == 1 and shard_world == 1 and args.workload == DEFAULT_WORKLOAD and int8 and not args.no_side_records:
        prefill = prefill_record(banks, dev, cap, args.steps)
        gx = torch.Generator().manual_seed(20261201)
        x3 = torch.randn(4096, K, generator=gx).to(torch.bfloat16).to(dev)
        ref_kernel = ref_kernel_record(banks, xs + [x3], dev, cap, args.steps)
        del x3

    # end to end through the public API with host buffers: every step copies each bucket's input from
    # pinned host memory, runs the path and reads every output back to pinned host memory, all inside the
    # replayed graph.  The compute runs on the step's two lanes; the copies run on two more streams, so a
    # bucket's read-back overlaps the compute after it and the inputs arrive ahead of their compute.
    # Inputs go largest first and a bucket of 1024 rows or more runs as four row pieces (the path is per
    # token, so the outputs are the same); what stays exposed is the first piece's input and the last
    # piece's output.
    e2e = None
    if not args.no_e2e:
        xs_host = [x.pin_memory() for x in xs_cpu]
        outs_host = [torch.empty((x.shape[0], h), dtype=torch.bfloat16).pin_memory() for x in xs_cpu]
        xs_dev = [torch.empty_like(x, device=dev) for x in xs_cpu]

        def pieces_of(j):
            M = xs_cpu[j].shape[0]
            rows = -(-M // (4 if M >= 1024 else 1))
            return [(j, r, min(M, r + rows)) for r in range(0, M, rows)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

        def e2e_step(i):
            main = torch.cuda.current_stream(dev)
            s_in.wait_stream(main)
            s_out.wait_stream(main)
            arrived = {}
            with torch.cuda.stream(s_in):
                for j in order:
                    for piece in pieces_of(j):
                        xs_dev[j][piece[1]:piece[2]].copy_(xs_host[j][piece[1]:piece[2]], non_blocking=True)
                        ev = torch.cuda.Event()
                        ev.record(s_in)
                        arrived[piece] = ev

            def work(j):
                lane = torch.cuda.current_stream(dev)
                outs = []   # alive until the step is enqueued, so no output buffer is reused under a read-back
                for piece in pieces_of(j):
                    _, r0, r1 = piece
                    lane.wait_event(arrived[piece])
                    xd = xs_dev[j][r0:r1]
                    b = bank_of(i, j)
                    o = gate_up.project(xd, b, "hybrid8_b128n256_s64n256") if int8 else bf16.gate_up(xd, b["w"])
                    outs.append(o)
                    done = torch.cuda.Event()
                    done.record(lane)
                    s_out.wait_event(done)
                    with torch.cuda.stream(s_out):
                        outs_host[j][r0:r1].copy_(o, non_blocking=True)
                return outs
            outs = run_lanes(work)
            main.wait_stream(s_in)
            main.wait_stream(s_out)
            return outs
        with torch.cuda.stream(cap), shares:
            e2e_step(0)
            torch.cuda.synchronize()
            egraphs = []
            for c in range(copies):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=cap):
                    e2e_step(c)
                egraphs.append(g)
            for i in range(args.warmup):
                egraphs[i % copies].replay()
            torch.cuda.synchronize()
            # the read-back of the last warm-up replay must equal the device step's outputs
            for j, x in enumerate(xs):
                last = bank_of(args.warmup - 1, j)
                o = gate_up.project(x, last, "hybrid8_b128n256_s64n256") if int8 else bf16.gate_up(x, last["w"])
                if not torch.equal(o.cpu(), outs_host[j]):
                    raise RuntimeError(f"e2e read-back of bucket M={x.shape[0]} differs from the device step")
        barrier(world)
        with torch.cuda.stream(cap):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(cap)
            for i in range(args.steps):
                egraphs[i % copies].replay()
            e1.record(cap)
        barrier(world)
        ems = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
        e2e = {"value": tokens / (ems * 1e-3), "unit": "tokens/s",
               "h2d_bytes_per_step": sum(x.numel() * 2 for x in xs_cpu),
               "d2h_bytes_per_step": sum(x.shape[0] * h * 2 for x in xs_cpu),
               "how": "public API calls captured once per weight copy into CUDA graphs, replayed per step; "
                      "compute on two lanes, H2D and D2H on side streams overlapping it, inputs largest first, "
                      "buckets of >= 1024 rows in four row pieces"}
        del egraphs
    del graphs

    # The optional collective: the all-gather of the largest bucket's output into the concatenated
    # [M, H] (sharding.gather_output, NCCL), timed on its own; it is not part of `value`.
    allgather = None
    if world > 1:
        from reax_engine_runtime_v3_b200.sharding import gather_output
        jmax = max(range(len(buckets)), key=lambda j: buckets[j])
        with torch.cuda.stream(cap):
            local = gate_up.project(xs[jmax], banks[0], "hybrid8_b128n256_s64n256") if int8 else \
                bf16.gate_up(xs[jmax], banks[0]["w"])
            full = gather_output(local, world)
            torch.cuda.synchronize()
            if not torch.equal(full[:, rank * h:(rank + 1) * h], local):
                raise RuntimeError("all-gather: this rank's columns of the gathered output differ from its shard")
            for _ in range(3):
                gather_output(local, world)
            barrier(world)
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n_gather = max(3, args.steps // 5)
            g0.record(cap)
            for _ in range(n_gather):
                gather_output(local, world)
            g1.record(cap)
            torch.cuda.synchronize()
        gms = max_over_ranks(g0.elapsed_time(g1) / n_gather, world)
        total = local.numel() * 2 * world
        allgather = {"bucket_M": buckets[jmax], "ms": gms, "bytes_total": total,
                     "bus_gbs": total * (world - 1) / world / (gms * 1e-3) / 1e9,
                     "how": "torch.distributed.all_gather_into_tensor (NCCL) into [W, M, H/W], reordered to [M, H]"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, threads, sample = cpu_run(args.workload)
        cpu = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong" if world > 1 else "strong", "vs_baseline": None, "dtype": "s8" if int8 else "bf16",
                "data": "synthetic (seeded N(0,1) or Student-t activations, uniform int8 / N(0,0.02) bf16 weights)",
                "config": {"workload": desc, "tokens_per_step": tokens, "K": K, "H": H, "H_per_gpu": h,
                           "parallelism": f"H-shard x{world}" if world > 1 else (
                               f"rank 0 of an H-shard x{shard_world}, alone on one GPU (its tokens/s, not the job's)"
                               if shard_world > 1 else "1 GPU"),
                           "lanes": [[buckets[j] for j in ln] for ln in lanes],
                           "lane_sms": shares.split if shares.streams else "whole GPU",
                           "l2": f"{copies} rotating weight copies ({copies * 2 * h * K * (1 if int8 else 2) / 1e6:.0f} MB > 126 MB L2), "
                                 "a different copy on consecutive calls"},
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "clocks": clocks,
                "allgather": allgather, "prefill": prefill, "ref_kernel": ref_kernel, "cfg4": cfg4,
                "device_status": status, "timing": "CUDA-graph replay of the captured step",
                "eager_ms_per_step": eager_ms}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def measure_int8_peak():
    """Dense INT8 tensor throughput reference: torch._int_mm at 8192^3, best of 10 (CUDA events)."""
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda").t()
    for _ in range(3):
        torch._int_mm(a, b)
    best = None
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) * 1e-3
        best = t if best is None else min(best, t)
    print(json.dumps({"what": "torch._int_mm int8 8192^3 best of 10", "tops": 2 * n ** 3 / best / 1e12,
                      "seconds": best, "torch": torch.__version__}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
