#!/usr/bin/env python
"""Benchmark of the B200-native pytorch_opt.ops hot path.

Default workload (configuration 5): one Muon step over the Llama-3-8B
matrix parameters — 32 layers x {q, o: 4096x4096; k, v: 1024x4096;
gate, up: 14336x4096; down: 4096x14336} = 224 bf16 matrices, grads
0.02*N(0,1), momentum 0.95 Nesterov, 5 Newton–Schulz steps, weight decay 0,
lr 0.02 — sharded per matrix over the ranks (FLOP-balanced) and all-gathered
with NCCL. Metric: ms per step (lower is better), the slowest rank's CUDA-event
time; 665.9 TFLOP of dense Newton–Schulz work per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0. At N = 1 the line also carries the same
Newton-Schulz work through torch/cuBLAS on the GPU (``gpu_library_bar``),
configurations 1-4 of the benchmark suite (``secondary``, each with its clocks and
CPU baseline) and the reference's CPU time per distinct shape
(``cpu_baseline``); at N > 1 a ``scaling_detail`` object (per-rank compute and
exposed exchange time, LPT imbalance). ``--impl reference`` times the
reference's own CPU implementation (its ATen extension compiled under
``oracle/_ref``, else the numpy restatement) on this host's cores: every
timed step is one sampled matrix, cycling the four distinct shapes, and the
full-step value is built from the per-shape sample times.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

LLAMA_LAYER = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096), (4096, 14336)]
LLAMA_DISTINCT = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)]
LLAMA_COUNT = {s: 32 * LLAMA_LAYER.count(s) for s in LLAMA_DISTINCT}
METRIC = "Muon NS5 step ms (8B shapes)"
MEASURED_PEAKS = os.path.join(HERE, "MEASURED_PEAKS.json")



PROFILES = os.path.join(HERE, "profiles")


def profiled_traffic(summary: str):
    """DRAM bytes recorded in a committed ncu summary under profiles/.

    The summary carries one line ``bench-traffic: <bytes> bytes; source
    <fingerprint>``: ncu's dram__bytes_read.sum + dram__bytes_write.sum of the
    workload's product launches, and the fingerprint of the Newton-Schulz
    path's sources (``build.NS_PATH_SOURCES``) in the build that was profiled. Returns (bytes or None, profiled fingerprint,
    whether it equals the current tree's)."""
    from pytorch_opt_b200.build import NS_PATH_SOURCES, source_fingerprint
    current = source_fingerprint(only=NS_PATH_SOURCES)
    try:
        with open(os.path.join(PROFILES, summary)) as f:
            for line in f:
                if line.startswith("bench-traffic:"):
                    parts = line.split()
                    nbytes = int(parts[1])
                    fp = parts[parts.index("source") + 1] if "source" in parts else None
                    return nbytes, fp, fp == current
    except (OSError, ValueError, IndexError):
        pass
    return None, None, False


def llama_shapes():
    return LLAMA_LAYER * 32


from pytorch_opt_b200.dist import ns_executed_flops  # noqa: E402
from pytorch_opt_b200.muon import ns_launches  # noqa: E402


def ns_flops(rows, cols, steps=5):
    m, n = min(rows, cols), max(rows, cols)
    return float(steps) * (4.0 * m * m * n + 2.0 * m ** 3)


def peaks():
    try:
        with open(MEASURED_PEAKS) as f:
            p = json.load(f)
        return {"bf16": float(p["bf16_tflops"]), "bf16_sustained": float(p["bf16_tflops_sustained"]),
                "hbm": float(p["hbm_gbs"]), "source": "measured"}
    except Exception:
        return {"bf16": 1590.0, "bf16_sustained": 1400.0, "hbm": 6650.0, "source": "fallback"}


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while the timed region runs."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: torch.device):
        self.proc = None
        self.path = None
        self.t_begin = self.t_end = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.gpu = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:
            self.gpu = str(device.index or 0)

    def start(self):
        """Start sampling every 200 ms and wait (up to 5 s) for the first sample,
        so that a timed region marked afterwards is covered from its start."""
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", self.gpu], stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 5.0 and self.proc.poll() is None and os.path.getsize(self.path) == 0:
            time.sleep(0.02)

    def mark_begin(self):
        self.t_begin = time.time()

    def mark_end(self):
        self.t_end = time.time()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        if self.t_end is None:
            self.mark_end()
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 10:
                    continue
                try:
                    ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                    rows.append((ts, float(parts[2]), float(parts[3]), parts[6:10]))
                except ValueError:
                    continue
        os.unlink(self.path)
        lo = (self.t_begin if self.t_begin is not None else -math.inf) - 0.05
        hi = self.t_end + 0.25  # a sample is taken up to 200 ms after the state it reports
        inside = [r for r in rows if lo <= r[0] <= hi]
        how = "samples taken during the timed region"
        if not inside and rows and self.t_begin is not None:  # region shorter than the sampling period
            mid = 0.5 * (self.t_begin + self.t_end)
            inside = [min(rows, key=lambda r: abs(r[0] - mid))]
            how = f"timed region ({self.t_end - self.t_begin:.2f} s) shorter than the 200 ms period: nearest sample"
        reasons = set()
        for r in inside:
            for name, val in zip(self.REASONS, r[3]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        sms = [r[1] for r in inside]
        return {"sm_mhz": statistics.median(sms) if sms else None,
                "sm_max_mhz": max(r[2] for r in inside) if inside else None,
                "reasons": sorted(reasons), "samples": len(sms), "how": how}


# ----------------------------------------------------------- CPU baseline
def _ref_ns_fn():
    """The reference's NS5 on the CPU: its own ATen extension (compiled under
    oracle/_ref) when present, else the numpy restatement. Returns
    (callable(G) -> None, kind, description of the implementation)."""
    try:
        from oracle import ref_native
        mod = ref_native.load()
    except Exception:
        mod = None
    if mod is not None:
        return (lambda G: mod.newton_schulz_orthogonalize(G, 5, 3.4445, -4.7750, 2.0315, 1e-7), "reference",
                "the reference's own ATen extension (pytorch_opt_ops.cpp:65-81, compiled under oracle/_ref)")
    from oracle import ops_np
    return (lambda G: ops_np.newton_schulz(G.float().numpy(), 5, out_bf16=True), "port",
            "the reference algorithm restated in numpy (oracle/ops_np.py)")


def _llama_sample(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * 0.02).bfloat16()


def cpu_reference_per_shape():
    """One NS5 of each distinct Llama-3-8B shape by the reference's CPU path
    (all host threads), summed by multiplicity into a full-step estimate."""
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    fn, kind, impl = _ref_ns_fn()
    per = {}
    for i, shape in enumerate(LLAMA_DISTINCT):
        G = _llama_sample(shape, 1000 + i)
        if i == 0:
            fn(G)  # warm-up (thread pools, first-touch)
        t0 = time.perf_counter()
        fn(G)
        per[shape] = (time.perf_counter() - t0) * 1e3
    total = sum(LLAMA_COUNT[s] * per[s] for s in LLAMA_DISTINCT)
    desc = (f"one NS5 per distinct shape by {impl}, bf16 0.02 N(0,1) inputs, {threads} threads; "
            "full step = sum over shapes of multiplicity x time")
    return total, per, kind, threads, desc


def run_reference_arm(args, rank, world):
    """--impl reference: the reference's CPU path on this host, rank 0 only.

    A full Llama-3-8B step takes minutes of CPU time per matrix group, so each
    timed "step" here is one sampled matrix: the four distinct shapes are
    cycled (4096^2, 1024x4096, 14336x4096, 4096x14336), every sample timed,
    and the full-step value is the sum over shapes of multiplicity x the
    shape's median sample time. ms_per_step is the mean measured sample time,
    so ms_per_step x steps is the time actually spent in the timed region.
    """
    if rank != 0:
        return 0
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    fn, kind, impl = _ref_ns_fn()
    inputs = [_llama_sample(s, 1000 + i) for i, s in enumerate(LLAMA_DISTINCT)]
    for i in range(args.warmup):
        fn(inputs[i % len(inputs)])
    samples = {s: [] for s in LLAMA_DISTINCT}
    t_all = time.perf_counter()
    for i in range(args.steps):
        j = i % len(inputs)
        t0 = time.perf_counter()
        fn(inputs[j])
        samples[LLAMA_DISTINCT[j]].append((time.perf_counter() - t0) * 1e3)
    timed_ms = (time.perf_counter() - t_all) * 1e3
    per = {}
    for s in LLAMA_DISTINCT:
        if samples[s]:
            per[s] = statistics.median(samples[s])
    # Shapes not sampled (steps < 4) are scaled from the sampled ones by dense FLOPs.
    rate = sum(ns_flops(*s) for s in per) / sum(per.values())
    for s in LLAMA_DISTINCT:
        per.setdefault(s, ns_flops(*s) / rate)
    value = sum(LLAMA_COUNT[s] * per[s] for s in LLAMA_DISTINCT)
    sample_desc = (f"{args.steps} timed samples cycling the 4 distinct Llama-3-8B shapes, one NS5 each by {impl}, "
                   f"{threads} threads; value = sum over shapes of multiplicity x median sample time")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": "ms", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(timed_ms / args.steps, 3),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": "Muon NS5 step over Llama-3-8B matrix params (224 matrices)", "ns_steps": 5,
                   "parallelism": "host CPU, all threads",
                   "sampled": {"per_shape_ms": {f"{r}x{c}": round(per[(r, c)], 2) for r, c in LLAMA_DISTINCT},
                               "multiplicity": {f"{r}x{c}": LLAMA_COUNT[(r, c)] for r, c in LLAMA_DISTINCT},
                               "note": "each step is one sampled matrix; ms_per_step is the mean sample time, "
                                       "value the full 224-matrix step built from the samples"}},
        "cpu_baseline": {"value": round(value, 1), "unit": "ms", "cores": threads, "kind": kind, "sample": sample_desc},
        "e2e": {"value": round(value, 1), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------- our arm
def fill_normal(t: torch.Tensor, seed: int, scale: float):
    g = torch.Generator(device=t.device).manual_seed(seed)
    t.copy_(torch.randn(t.shape, generator=g, device=t.device, dtype=torch.float32).mul_(scale))


def _torch_ns(G: torch.Tensor, dt: torch.dtype) -> torch.Tensor:
    """NS5 as torch ops in dtype dt: the op sequence of the reference's ATen
    module (pytorch_opt_ops.cpp:65-81; fp32 work dtype) when dt is fp32."""
    a, b, c = 3.4445, -4.7750, 2.0315
    X = G.to(dt)
    tall = X.shape[-2] > X.shape[-1]
    if tall:
        X = X.mT
    X = X / (X.float().norm() + 1e-7).to(dt)
    for _ in range(5):
        A = X @ X.mT
        B = b * A + c * (A @ A)
        X = a * X + B @ X
    if tall:
        X = X.mT
    return X.to(G.dtype)


def gpu_library_bar(mats: list, dev: torch.device) -> dict:
    """The same Newton-Schulz work through torch/cuBLAS on this GPU, one matrix
    at a time as the reference's Muon loop calls it (muon.py:70-98): fp32
    SGEMM (TF32 off; the reference's ATen path on CUDA tensors) over one full
    224-matrix step, and the same chain on bf16 matmuls (a speed bar only: an
    all-bf16 chain misses the 1e-2 tolerance)."""
    old = torch.backends.cuda.matmul.allow_tf32
    out = {}
    try:
        for name, dt, reps in (("torch_fp32_cublas_ms", torch.float32, 1), ("torch_bf16_cublas_ms", torch.bfloat16, 2)):
            torch.backends.cuda.matmul.allow_tf32 = False
            for shape in LLAMA_DISTINCT:  # warm-up: one matrix of each shape
                _torch_ns(next(m for m in mats if tuple(m.shape) == shape), dt)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                for m in mats:
                    _torch_ns(m, dt)
            e1.record()
            torch.cuda.synchronize(dev)
            out[name] = round(e0.elapsed_time(e1) / reps, 1)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    out["how"] = ("torch ops per matrix (cast, transpose if tall, normalise, 5 x 3 matmuls, cast back), CUDA-event "
                  "time of one full step (fp32) / mean of two (bf16), inputs resident")
    return out


def gpu_local_cpus(dev: torch.device) -> set | None:
    """Host CPUs on the NUMA node of the GPU's PCI device (sysfs), or None."""
    try:
        pr = torch.cuda.get_device_properties(dev)
        addr = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{addr}/local_cpulist") as f:
            spec = f.read().strip()
        cpus = set()
        for part in spec.split(","):
            a, _, b = part.partition("-")
            cpus.update(range(int(a), int(b or a) + 1))
        return cpus & os.sched_getaffinity(0) or None
    except (OSError, ValueError, AttributeError):
        return None


def run_ours(args, rank, world, local_rank):
    from pytorch_opt_b200.dist import ShardLayout, ShardedMuon
    import torch.distributed as dist

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1 and os.environ.get("PO_BENCH_NUMA", "0") == "1":
        # PO_BENCH_NUMA=1 (measurement switch): run each rank on its GPU's own
        # NUMA node, so that the pinned gradient buffer of the end-to-end run
        # (first touch) sits in the memory next to the GPU's PCIe link.
        cpus = gpu_local_cpus(dev)
        if cpus:
            os.sched_setaffinity(0, cpus)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    shapes = llama_shapes()
    layout = ShardLayout(shapes, world, chunks=args.exchange_chunks)
    params = torch.zeros(layout.numel, dtype=torch.bfloat16, device=dev)
    grads = torch.zeros(layout.numel, dtype=torch.bfloat16, device=dev)
    for i in range(len(shapes)):
        fill_normal(layout.matrix(params, i), 2000 + i, 0.02)  # every rank holds every parameter
        if layout.offset_of[i][0] == rank:
            fill_normal(layout.matrix(grads, i), 1000 + i, 0.02)  # grads of the local shard
    sm = ShardedMuon(layout, params, grads, rank, lr=0.02, momentum=0.95, nesterov=True, ns_steps=5,
                     weight_decay=0.0)
    local_flops = layout.flops(rank)
    local_exec = sum(ns_executed_flops(*shapes[i]) for i in layout.assign[rank])
    total_flops = sum(ns_flops(r, c) for r, c in shapes)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def all_ranks(x: float) -> list:
        if world == 1:
            return [x]
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        out = torch.empty(world, dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(out, t)
        return out.tolist()

    # ---------------------------------------------------- device-resident run
    clocks = ClockSampler(dev)
    clocks.start()
    for _ in range(args.warmup):
        sm.step()
    barrier()
    ns_events: list = []
    tail_events: list = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.mark_begin()
    e0.record(stream)
    for _ in range(args.steps):
        sm.step(ns_events, tail_events)
    e1.record(stream)
    barrier()
    clocks.mark_end()
    clk = clocks.stop()
    step_ranks = all_ranks(e0.elapsed_time(e1) / args.steps)
    step_ms = max(step_ranks)
    ns_ms_local = sum(a.elapsed_time(b) for a, b in ns_events) / args.steps
    tail_ms_local = sum(a.elapsed_time(b) for a, b in tail_events) / args.steps
    ns_ranks = all_ranks(ns_ms_local)
    tail_ranks = all_ranks(tail_ms_local)
    gemm_tflops = min(all_ranks(local_flops / (ns_ms_local * 1e-3) / 1e12 if ns_ms_local > 0 else 0.0))
    exec_tflops = min(all_ranks(local_exec / (ns_ms_local * 1e-3) / 1e12 if ns_ms_local > 0 else 0.0))
    launches = sm.launches_per_step() * args.steps

    wait_profile = gemm_wait_profile(sm.step, dev) if args.gemm_profile else None

    # -------------------------------------------------------------- e2e run
    e2e = None
    if not args.no_e2e:
        host = torch.empty(layout.slot, dtype=torch.bfloat16, pin_memory=True)
        host.copy_(layout.slot_tensor(grads, rank))
        sq = torch.zeros(1, dtype=torch.float64, device=dev)
        for _ in range(min(args.warmup, 1)):
            sm.step_from_host(host)
        barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(args.steps):
            sm.step_from_host(host)                   # this step's gradients, from pinned host memory
            sq.copy_(sm._sq.sum().reshape(1))
            if world > 1:
                dist.all_reduce(sq)
            _ = float(sq.item())                      # the step's diagnostic, read back on the host
        a1.record(stream)
        barrier()
        e2e = {"value": round(max(all_ranks(a0.elapsed_time(a1) / args.steps)), 3), "unit": "ms",
               "h2d_bytes_per_step": int(layout.slot_elements(rank) * 2), "d2h_bytes_per_step": 8,
               "api": "pytorch_opt_b200.dist.ShardedMuon.step_from_host (per-group H2D copies overlapped with "
                      "the grouped Muon kernels, C ABI) + NCCL all-gather"}

    single = rank == 0 and world == 1
    # ------------------------------------------------ GPU library bar (N = 1)
    bar = None
    if single and not args.no_library_bar:
        mats = [layout.matrix(grads, i) for i in range(len(shapes))]
        bar = gpu_library_bar(mats, dev)
    # --------------------------------------------------------- CPU baseline
    cpu = None
    if single and not args.no_cpu_baseline:
        total, per, kind, threads, desc = cpu_reference_per_shape()
        cpu = {"value": round(total, 1), "unit": "ms", "cores": threads, "kind": kind, "sample": desc,
               "per_shape_ms": {f"{r}x{c}": round(per[(r, c)], 1) for r, c in LLAMA_DISTINCT}}
    # ---------------------------------------- configs 1-4 on this GPU (N = 1)
    secondary = None
    if single and not args.no_secondary:
        del sm, params, grads
        torch.cuda.empty_cache()
        secondary = run_secondary_all(dev, args, with_cpu=not args.no_cpu_baseline)

    pk = peaks()
    if rank == 0:
        traffic, prof_fp, prof_match = profiled_traffic("launches_llama8b_muon_step.md")
        line = {
            "metric": METRIC, "value": round(step_ms, 3), "unit": "ms", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(step_ms, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "precision": "bf16 tensor-core products on every NS step with the exact fp32 diagonal split of A and B "
                         "in the epilogues; fp32 accumulation",
            "config": {"workload": "Muon step over Llama-3-8B matrix params (224 bf16 matrices, 5 NS steps)",
                       "ns_steps": 5, "momentum": 0.95, "nesterov": True,
                       "parallelism": f"per-matrix FLOP-balanced shard x{world} + NCCL all-gather"
                                      + (f" in {layout.chunks} chunks overlapped with the step"
                                         if world > 1 and layout.chunks > 1 else ""),
                       "l2": "inputs larger than L2 (13.96 GB of bf16 params and grads per step)",
                       "algorithmic_tflop_per_step": round(total_flops / 1e12, 1)},
            "tflops": round(total_flops / (step_ms * 1e-3) / 1e12, 1),
            "roofline": {"bound": "tensor",
                         "kernel": "tc_gemm_pair_kernel (Newton-Schulz products, 256x256 tiles on SM pairs)",
                         "achieved": round(gemm_tflops, 1), "peak": pk["bf16_sustained"], "unit": "TFLOP/s",
                         "frac": round(gemm_tflops / pk["bf16_sustained"], 3),
                         "traffic": traffic if world == 1 else None,
                         "traffic_unit": "DRAM bytes per 1-GPU step summed over the Newton-Schulz product launches "
                                         "(ncu dram__bytes_read.sum + dram__bytes_write.sum, committed launch-list "
                                         "summary)",
                         "traffic_profiled_build": prof_fp, "traffic_matches_this_build": prof_match,
                         "peak_source": pk["source"] + " bf16 sustained (MEASURED_PEAKS.json)",
                         "how": "dense NS FLOPs of the rank's matrices (the reference formula, 5 (4 m^2 n + "
                                "2 m^3) each) / CUDA-event time of its Newton-Schulz calls inside the timed steps "
                                "(includes the momentum and scale kernels); slowest rank. frac exceeds 1 because the "
                                "kernels execute fewer FLOPs than the formula counts (symmetric products on their "
                                "lower tiles; matrices with n >= 2m in groups of steps): see executed",
                         "executed": {"achieved": round(exec_tflops, 1),
                                      "frac": round(exec_tflops / pk["bf16_sustained"], 3),
                                      "tflop_per_step": round(sum(ns_executed_flops(r, c) for r, c in shapes)
                                                              / 1e12, 1),
                                      "how": "FLOPs the tensor cores execute under the library's schedule "
                                             "(dist.ns_executed_flops) / the same time"}},
            "clocks": clk,
            "gpu_launches": int(launches),
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        if bar is not None:
            line["gpu_library_bar"] = bar
        if wait_profile is not None:
            line["gemm_wait_profile"] = wait_profile
        if world > 1:
            fl = [sum(ns_executed_flops(*shapes[i]) for i in layout.assign[r]) / 1e12 for r in range(world)]
            line["scaling_detail"] = {
                "rank_step_ms": [round(x, 2) for x in step_ranks],
                "rank_ns_compute_ms": [round(x, 2) for x in ns_ranks],
                "rank_exposed_exchange_ms": [round(x, 2) for x in tail_ranks],
                "rank_executed_tflop": [round(x, 2) for x in fl],
                "lpt_imbalance_max_over_mean": round(max(fl) / (sum(fl) / len(fl)), 4),
                "exchange_chunks": layout.chunks,
                "how": "per rank: CUDA-event time of its Newton-Schulz calls, and of the wait for the all-gathers "
                       "still in flight after its last kernel (the exposed exchange)"}
        if secondary is not None:
            line["secondary"] = secondary
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def gemm_wait_profile(fn, dev) -> dict:
    """One more (untimed) call of ``fn`` with the two-SM GEMM kernel's wait
    counters on: the share of each role's time spent waiting (SM cycles summed
    over CTAs)."""
    from pytorch_opt_b200 import _lib
    torch.cuda.synchronize(dev)
    _lib.gemm_profile(True)          # zero, then switch on
    fn()
    c = _lib.gemm_profile(False)     # synchronise, read, switch off
    def share(a, b):
        return round(c[a] / c[b], 4) if c[b] else None
    busy = c["mma_total"] - c["mma_full_wait"] - c["mma_tempty_wait"]
    return {"mma_waits_for_operands": share("mma_full_wait", "mma_total"),
            "mma_waits_for_accumulator": share("mma_tempty_wait", "mma_total"),
            "producer_waits_for_stage": share("producer_empty_wait", "producer_total"),
            "epilogue_waits_for_accumulator": share("epilogue_full_wait", "epilogue_total"),
            "epilogue_working": share("epilogue_work", "epilogue_total"),
            "tiles": c["tiles"],
            "mma_issue_cycles_per_tile": round(busy / c["tiles"], 1) if c["tiles"] else None,
            "how": "po_gemm_profile counters over one extra untimed call; clock64 cycles per role summed over CTAs"}


# ------------------------------------------------- secondary workloads (1 GPU)
MIN_TIMED_SECONDS = 1.0


def _timed(fn, steps, warmup, dev, flush=None, min_seconds=None):
    """Per-call CUDA-event time (ms), L2 flushed between calls (outside the timed intervals).

    Short calls are repeated in rounds of ``steps`` until the timed region
    lasts at least ``min_seconds``, so that the clock sampler (200 ms period)
    sees it; the time is the mean over every timed call."""
    if min_seconds is None:
        min_seconds = MIN_TIMED_SECONDS
    clocks = ClockSampler(dev)
    clocks.start()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    pairs = []
    clocks.mark_begin()
    t0 = time.perf_counter()
    while True:
        for _ in range(steps):
            if flush is not None:
                flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            pairs.append((a, b))
        torch.cuda.synchronize(dev)
        if time.perf_counter() - t0 >= min_seconds or len(pairs) >= 200 * steps:
            break
    clocks.mark_end()
    clk = clocks.stop()
    clk["timed_calls"] = len(pairs)
    return sum(a.elapsed_time(b) for a, b in pairs) / len(pairs), clk


def _line(args, metric, value, unit, hib, workload, tflops, clk, launches, cpu, extra=None, traffic=None,
          peak=None, peak_name="bf16 sustained"):
    pk = peaks()
    peak = pk["bf16_sustained"] if peak is None else peak
    line = {"metric": metric, "value": round(value, 4), "unit": unit, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": None, "higher_is_better": hib, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": workload, "l2": "flushed between timed calls (256 MiB write)"},
            "roofline": {"bound": "tensor", "kernel": "tc_gemm_pair_kernel", "achieved": round(tflops, 1),
                         "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(tflops / peak, 3), "traffic": traffic,
                         "peak_source": pk["source"] + f" {peak_name} (MEASURED_PEAKS.json)",
                         "how": "dense algorithmic FLOPs of the call / its CUDA-event time"},
            "clocks": clk, "gpu_launches": launches, "e2e": None, "cpu_baseline": cpu}
    if extra:
        line.update(extra)
    print(json.dumps(line), flush=True)


def _cpu_time(fn, reps=1):
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    fn()
    t0 = time.perf_counter()
    for _ in range(reps):
        fn()
    return (time.perf_counter() - t0) / reps


def _ref_module():
    try:
        from oracle import ref_native
        return ref_native.load()
    except Exception:
        return None


def cfg_ns768(dev, flush, steps, warmup, with_cpu):
    """Config 1: NS5 of one 768 x 3072 fp32 N(0,1) matrix (seed 0)."""
    from pytorch_opt_b200 import native
    g = torch.Generator().manual_seed(0)
    Gc = torch.randn(768, 3072, generator=g)
    G = Gc.to(dev)
    ms, clk = _timed(lambda: native.newton_schulz_orthogonalize(G, 5, 3.4445, -4.7750, 2.0315, 1e-7), steps, warmup,
                     dev, flush)
    fl = ns_flops(768, 3072)
    cpu = None
    ref = _ref_module()
    if with_cpu and ref is not None:
        t = _cpu_time(lambda: ref.newton_schulz_orthogonalize(Gc, 5, 3.4445, -4.7750, 2.0315, 1e-7), reps=3)
        cpu = {"value": round(t * 1e3, 2), "unit": "ms", "cores": len(os.sched_getaffinity(0)), "kind": "reference",
               "sample": "the reference's ATen NS5 (pytorch_opt_ops.cpp:65-81) on the same matrix, mean of 3"}
    return {"metric": "NS5 768x3072 ms", "value": ms, "unit": "ms", "higher_is_better": False,
            "workload": "NS5 of one 768x3072 fp32 matrix, N(0,1), seed 0 (config 1)", "tflops": fl / (ms * 1e-3) / 1e12,
            "clocks": clk, "gpu_launches": ns_launches(768, 3072, 5), "cpu_baseline": cpu}


def cfg_gpt2(dev, flush, steps, warmup, with_cpu):
    """Config 2: Muon step over the 48 GPT-2-small matrices."""
    from pytorch_opt_b200.muon import GroupedMuon, MuonGroup
    shapes = [(768, 2304), (768, 768), (768, 3072), (3072, 768)]
    groups, k = [], 0
    for shp in shapes:
        p = torch.empty(12, *shp, dtype=torch.bfloat16, device=dev)
        gr = torch.empty_like(p)
        for j in range(12):
            fill_normal(p[j], 2000 + k, 0.02)
            fill_normal(gr[j], 1000 + k, 0.02)
            k += 1
        groups.append(MuonGroup(p, gr))
    opt = GroupedMuon(groups, lr=0.02, momentum=0.95, nesterov=True, ns_steps=5)
    fl = 12 * sum(ns_flops(*s) for s in shapes)
    ms, clk = _timed(opt.step, steps, warmup, dev, flush)
    cpu = None
    if with_cpu:
        fn, kind, impl = _ref_ns_fn()
        torch.set_num_threads(len(os.sched_getaffinity(0)))
        per = {}
        for i, shp in enumerate(shapes):
            G = _llama_sample(shp, 1000 + i)
            fn(G)
            t0 = time.perf_counter()
            fn(G)
            per[shp] = (time.perf_counter() - t0) * 1e3
        cpu = {"value": round(12 * sum(per.values()), 1), "unit": "ms", "cores": len(os.sched_getaffinity(0)),
               "kind": kind, "sample": f"one NS5 per distinct shape by {impl}, x12 layers (the elementwise parts "
                                       "of the reference's step are not timed)"}
    return {"metric": "GPT-2-small Muon step ms", "value": ms, "unit": "ms", "higher_is_better": False,
            "workload": "Muon step over 48 GPT-2-small matrices (bf16, 0.02 N(0,1), momentum 0.95 Nesterov, "
                        "5 NS steps) (config 2)", "tflops": fl / (ms * 1e-3) / 1e12, "clocks": clk,
            "gpu_launches": opt.launches_per_step(), "cpu_baseline": cpu}


def cfg_shampoo(dev, flush, steps, warmup, with_cpu):
    """Config 3: inverse 4th roots of 8 SPD factors per size d in {1024, 2048, 4096}."""
    from pytorch_opt_b200 import _lib
    lib = _lib.load()
    res, clk = {}, None
    for d in (1024, 2048, 4096):
        g = torch.Generator(device=dev).manual_seed(d * 100)
        Gs = torch.randn(8, d, 2 * d, generator=g, device=dev)
        L = Gs @ Gs.mT / (2 * d) + 1e-6 * torch.eye(d, device=dev)
        del Gs
        out = torch.empty_like(L)
        its = torch.zeros(8, dtype=torch.int32, device=dev)
        nbytes = lib.po_root_workspace_bytes(8, d, 4)
        ws = _lib.workspace(nbytes, dev)

        def call():
            _lib.check(lib.po_inverse_root(L.data_ptr(), 0, 8, d, d, d * d, out.data_ptr(), d, d * d, 4, 1e-8,
                                           100, 1e-10, its.data_ptr(), ws.data_ptr(), nbytes,
                                           _lib.stream_ptr(dev)), "root")
        ms, c = _timed(call, steps, warmup, dev, flush)
        n_it = its.tolist()
        fl = sum(8.0 * d ** 3 * i for i in n_it)
        res[d] = {"ms": round(ms, 3), "iters": n_it, "tflops": round(fl / (ms * 1e-3) / 1e12, 1)}
        clk = c if d == 4096 else clk
        del L, out, ws
    cpu = None
    ref = _ref_module()
    if with_cpu and ref is not None:
        torch.set_num_threads(len(os.sched_getaffinity(0)))
        t = {}
        for d in (1024, 2048):
            g = torch.Generator().manual_seed(d * 100)
            Gm = torch.randn(d, 2 * d, generator=g)
            Lc = Gm @ Gm.T / (2 * d) + 1e-6 * torch.eye(d)
            t0 = time.perf_counter()
            ref.inverse_matrix_root(Lc, 4, 1e-8, "newton", True, 100, 1e-10)
            t[d] = time.perf_counter() - t0
        total = 8 * (t[1024] + t[2048] + 8 * t[2048])
        cpu = {"value": round(total * 1e3, 1), "unit": "ms", "cores": len(os.sched_getaffinity(0)),
               "kind": "reference", "per_factor_ms": {"1024": round(t[1024] * 1e3, 1), "2048": round(t[2048] * 1e3, 1)},
               "sample": "the reference's ATen coupled Newton (fp64, pytorch_opt_ops.cpp:15-63) on one d=1024 and "
                         "one d=2048 factor; total = 8 x (t1024 + t2048 + 8 t2048), d=4096 scaled from d=2048 by d^3"}
    ms_all = sum(r["ms"] for r in res.values())
    return {"metric": "Shampoo inverse 4th root TFLOP/s (8 x d=4096)", "value": res[4096]["tflops"],
            "unit": "TFLOP/s", "higher_is_better": True,
            "workload": "coupled-Newton inverse 4th roots of 8 SPD factors per size, L = G G^T/2d + 1e-6 I, "
                        "damping 1e-8 (config 3)", "tflops": res[4096]["tflops"], "ms_all_sizes": round(ms_all, 3),
            "per_size": res, "clocks": clk, "gpu_launches": None, "cpu_baseline": cpu,
            "peak_split_bf16": peaks()["bf16_sustained"] / 3.0}


def cfg_kfac(dev, flush, steps, warmup, with_cpu):
    """Config 4: KFAC SYRK+EMA of A and G (8192 x 4096 bf16), then the pi-damped inverses."""
    from pytorch_opt_b200 import native
    g1 = torch.Generator(device=dev).manual_seed(1)
    g2 = torch.Generator(device=dev).manual_seed(2)
    a = torch.randn(8192, 4096, generator=g1, device=dev).bfloat16()
    gr = torch.randn(8192, 4096, generator=g2, device=dev).bfloat16()
    A = torch.empty(4096, 4096, device=dev)
    Gf = torch.empty(4096, 4096, device=dev)
    n = 8192
    native.kron_syrk_ema_(A, a, 1.0 / n, 0.95, True)
    native.kron_syrk_ema_(Gf, gr, float(n), 0.95, True)

    def update():
        native.kron_syrk_ema_(A, a, 1.0 / n, 0.95, False)
        native.kron_syrk_ema_(Gf, gr, float(n), 0.95, False)
    ms_u, clk = _timed(update, steps, warmup, dev, flush)
    tr_a = float(A.diagonal().sum()) / 4096
    tr_g = float(Gf.diagonal().sum()) / 4096
    pi = math.sqrt(tr_a / tr_g)
    ga, gg = pi * math.sqrt(1e-3), math.sqrt(1e-3) / pi

    def inverse():
        native.damped_inverse(A, ga)
        native.damped_inverse(Gf, gg)
    ms_i, _ = _timed(inverse, max(1, steps // 2), 1, dev, flush)
    fl_u = 2 * 2.0 * 8192 * 4096 ** 2
    cpu = None
    if with_cpu:
        torch.set_num_threads(len(os.sched_getaffinity(0)))
        ac = torch.randn(8192, 4096, generator=torch.Generator().manual_seed(1)).bfloat16().float()
        t_u = _cpu_time(lambda: ac.T @ ac / 8192)
        Fc = ac[:2048, :1024].T @ ac[:2048, :1024] / 2048
        t_e = _cpu_time(lambda: torch.linalg.eigh(Fc.double()))
        cpu = {"value": round(2 * t_u * 1e3, 1), "unit": "ms", "cores": len(os.sched_getaffinity(0)),
               "kind": "reference",
               "inverse_ms_both_estimate": round(2 * 64 * t_e * 1e3, 1),
               "sample": "the reference's factor product (torch fp32 a^T a / n on the CPU, kron.py:105-113) on the "
                         "full 8192 x 4096 batch, x2 factors; its fp64 eigh inverse (kfac.py:134-138) timed at "
                         "d = 1024 and scaled by d^3 to 4096 for both factors"}
    return {"metric": "KFAC factor update ms (A and G, 8192x4096 -> 4096^2)", "value": ms_u, "unit": "ms",
            "higher_is_better": False,
            "workload": "KFAC SYRK+EMA of A = a^T a/n and G = (n g)^T (n g)/n, a, g 8192x4096 bf16, beta 0.95; "
                        "then pi-damped inverses (lambda 1e-3) by coupled Newton p=1 (config 4)",
            "tflops": fl_u / (ms_u * 1e-3) / 1e12, "damped_inverse_ms_both": round(ms_i, 3), "clocks": clk,
            "gpu_launches": None, "cpu_baseline": cpu}


SECONDARY = {"ns768": cfg_ns768, "gpt2": cfg_gpt2, "shampoo": cfg_shampoo, "kfac": cfg_kfac}


def run_secondary_all(dev, args, with_cpu: bool) -> dict:
    """Configs 1-4 on this GPU, each with its own clocks and CPU baseline (for the default line)."""
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    pk = peaks()
    out = {}
    for cfg, (name, steps, warmup) in enumerate((("ns768", 10, 3), ("gpt2", 5, 3), ("shampoo", 3, 1),
                                                 ("kfac", 5, 3)), start=1):
        r = SECONDARY[name](dev, flush, steps, warmup, with_cpu)
        peak = r.pop("peak_split_bf16", pk["bf16_sustained"])
        r["value"] = round(r["value"], 4)
        r["tflops"] = round(r["tflops"], 1)
        r["frac_of_peak"] = round(r["tflops"] / peak, 3)
        r["peak"] = round(peak, 1)
        r["peak_source"] = pk["source"] + (" bf16 sustained / 3 (split-bf16 products)" if name == "shampoo"
                                           else " bf16 sustained")
        r["steps"], r["warmup"] = steps, warmup
        out[f"config{cfg}_{name}"] = r
        torch.cuda.empty_cache()
    return out


def run_secondary(args, rank):
    if rank != 0:
        return 0
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    threads = len(os.sched_getaffinity(0))
    w = args.workload
    if w in SECONDARY:
        r = SECONDARY[w](dev, flush, args.steps, args.warmup, not args.no_cpu_baseline)
        peak = r.pop("peak_split_bf16", None)
        extra = {k: v for k, v in r.items() if k not in ("metric", "value", "unit", "higher_is_better", "workload",
                                                         "tflops", "clocks", "gpu_launches", "cpu_baseline")}
        launches = r["gpu_launches"] * args.steps if r["gpu_launches"] else None
        _line(args, r["metric"], r["value"], r["unit"], r["higher_is_better"], r["workload"], r["tflops"],
              r["clocks"], launches, r["cpu_baseline"], extra, peak=peak,
              peak_name="bf16 sustained / 3 (split-bf16 products)" if peak else "bf16 sustained")
        return 0
    ref = _ref_module()
    from pytorch_opt_b200 import native
    if w == "ns4096":      # a batch of q/o-shaped matrices: the profiling case of the main workload's products
        g = torch.Generator().manual_seed(1000)
        Gc = (torch.randn(4, 4096, 4096, generator=g) * 0.02).bfloat16()
        desc, fl = "NS5 of 4 x 4096x4096 bf16 matrices (Llama q/o shape), 0.02 N(0,1)", 4 * ns_flops(4096, 4096)
        G = Gc.to(dev)
        ms, clk = _timed(lambda: native.newton_schulz_orthogonalize(G, 5, 3.4445, -4.7750, 2.0315, 1e-7),
                         args.steps, args.warmup, dev, flush)
        cpu = None
        if ref is not None and not args.no_cpu_baseline:
            t = _cpu_time(lambda: ref.newton_schulz_orthogonalize(Gc[0], 5, 3.4445, -4.7750, 2.0315, 1e-7))
            cpu = {"value": round(t * 1e3 * 4, 2), "unit": "ms", "cores": threads, "kind": "reference",
                   "sample": "the reference's ATen NS5 on one 4096^2 matrix of the workload, x4"}
        traffic, prof_fp, prof_match = profiled_traffic("tc_gemm_pair_ns4096.md")
        extra = {"ms_per_step": round(ms, 4), "traffic_profiled_build": prof_fp, "traffic_matches_this_build": prof_match}
        if args.gemm_profile:
            extra["gemm_wait_profile"] = gemm_wait_profile(
                lambda: native.newton_schulz_orthogonalize(G, 5, 3.4445, -4.7750, 2.0315, 1e-7), dev)
        _line(args, "NS5 4x4096^2 ms", ms, "ms", False, desc, fl / (ms * 1e-3) / 1e12, clk, (2 + 3 * 5) * args.steps,
              cpu, extra, traffic=traffic)
        return 0
    if w == "gemm":        # the product kernel alone, beside cuBLAS on the same shape
        import ctypes
        from pytorch_opt_b200 import _lib
        lib = _lib.load()
        M, N, K = args.gemm
        bf16 = args.gemm_dtype == "bf16"
        dt = torch.bfloat16 if bf16 else torch.float32
        g = torch.Generator(device="cpu").manual_seed(5)
        A = torch.randn(M, K, generator=g).to(dev, dt)
        Bt = torch.randn(N, K, generator=g).to(dev, dt)     # B stored [N][K]: both operands K-major
        C = torch.zeros(M, N, device=dev)
        code = 1 if bf16 else 0
        nb = lib.po_matmul_workspace_bytes(1, M, N, K, code, 0)
        ws = _lib.workspace(nb, dev)
        stream = _lib.stream_ptr(dev)

        def call():
            _lib.check(lib.po_matmul(A.data_ptr(), K, M * K, 0, Bt.data_ptr(), K, N * K, 1,
                                     ctypes.c_void_p(C.data_ptr()), N, M * N, code, 0, 1, M, N, K, 1.0, 0.0,
                                     ws.data_ptr(), nb, stream), "po_matmul")
        ms, clk = _timed(call, args.steps, args.warmup, dev, flush)
        torch.backends.cuda.matmul.allow_tf32 = True
        ms_lib, _ = _timed(lambda: torch.matmul(A, Bt.t()), args.steps, args.warmup, dev, flush)
        fl = 2.0 * M * N * K
        _line(args, f"GEMM {M}x{N}x{K} {args.gemm_dtype} TFLOP/s", fl / (ms * 1e-3) / 1e12, "TFLOP/s", True,
              f"po_matmul, K-major A and B, fp32 C, {args.gemm_dtype} tensor-core operands",
              fl / (ms * 1e-3) / 1e12, clk, args.steps, None,
              {"ms_per_step": round(ms, 4),
               "library_comparison": {"torch.matmul (cuBLAS) TFLOP/s": round(fl / (ms_lib * 1e-3) / 1e12, 1),
                                      "note": "cuBLAS writes a bf16/fp32 C of the operand type"}})
        return 0
    if w == "ekfac":       # section 8f rank 4: EKFAC rotated-diagonal precondition of one layer
        m = n = 4096
        g = torch.Generator(device=dev).manual_seed(6)
        QG = torch.linalg.qr(torch.randn(m, m, generator=g, device=dev))[0]
        QA = torch.linalg.qr(torch.randn(n, n, generator=g, device=dev))[0]
        V = torch.randn(m, n, generator=g, device=dev)
        _, S = native.ekfac_precondition(QG, QA, V, None, 0.95, 1e-3)
        ms, clk = _timed(lambda: native.ekfac_precondition(QG, QA, V, S, 0.95, 1e-3), args.steps, args.warmup, dev,
                         flush)
        fl = 4 * 2.0 * m * n * 4096
        cpu = None
        if not args.no_cpu_baseline:
            from oracle import ops_np as O
            k = 1024  # bounded sample: the same four products at a quarter of each dimension
            qg, qa, v = QG[:k, :k].cpu().numpy(), QA[:k, :k].cpu().numpy(), V[:k, :k].cpu().numpy()
            _, s0 = O.ekfac_precondition(qg, qa, v, None, 0.95, 1e-3)
            t = _cpu_time(lambda: O.ekfac_precondition(qg, qa, v, s0, 0.95, 1e-3))
            cpu = {"value": round(t * 1e3 * 64, 1), "unit": "ms", "cores": threads, "kind": "port",
                   "sample": "the numpy restatement of ekfac.py:44-58 (fp32 BLAS) on 1024x1024 blocks, x64 for the "
                             "4096^2 layer by dense FLOPs"}
        _line(args, "EKFAC precondition ms (one 4096x4096 layer)", ms, "ms", False,
              "EKFAC QG (Vt / (s + 1e-3)) QA^T with Vt = QG^T V QA and the running scales updated in place, "
              "fp32 4096x4096, split-bf16 products", fl / (ms * 1e-3) / 1e12, clk, (4 + 3) * args.steps, cpu,
              {"ms_per_step": round(ms, 4)})
        return 0
    if w == "soap":        # section 8f rank 2: SOAP's basis refresh of one 1024x1024 matrix parameter
        d = 1024
        g = torch.Generator(device=dev).manual_seed(7)
        Gs = [torch.randn(d, d, generator=g, device=dev) * 0.02 for _ in range(12)]
        L = torch.zeros(d, d, device=dev)
        R = torch.zeros(d, d, device=dev)
        for k, G in enumerate(Gs):
            L.mul_(0.95).add_(G @ G.T, alpha=0.05)
            R.mul_(0.95).add_(G.T @ G, alpha=0.05)
            if k == 1:
                QLo = torch.linalg.eigh(L.double())[1].float()
                QRo = torch.linalg.eigh(R.double())[1].float()
        QLn = torch.linalg.eigh(L.double())[1].float()
        QRn = torch.linalg.eigh(R.double())[1].float()
        V0 = torch.rand(d, d, generator=g, device=dev) ** 2
        V = V0.clone()
        ms_tr, clk = _timed(lambda: native.soap_transport_(V, QLo, QLn, QRo, QRn), args.steps, args.warmup, dev, flush)
        st = {"L": L, "R": R, "exp_avg_sq": V0.clone()}

        def refresh(method):
            st.update(Q_L=QLo, Q_R=QRo)
            native.soap_refresh_(st, torch.float32, method, 1)
        ms_sub, _ = _timed(lambda: refresh("subspace"), args.steps, args.warmup, dev, flush)
        ms_eigh, _ = _timed(lambda: refresh("eigh"), args.steps, args.warmup, dev, flush)

        def torch_refresh(Lx, Rx, QLx, QRx, Vx):  # the reference's lines (soap.py:98-108) on the given device
            ql = torch.linalg.eigh(Lx.double())[1].float()
            qr = torch.linalg.eigh(Rx.double())[1].float()
            cl, cr = QLx.T @ ql, QRx.T @ qr
            return cl.pow(2).T @ Vx @ cr.pow(2)
        tf32 = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False  # the reference's fp32 matmuls
        try:
            ms_ref_gpu, _ = _timed(lambda: torch_refresh(L, R, QLo, QRo, V0), args.steps, args.warmup, dev, flush)
        finally:
            torch.backends.cuda.matmul.allow_tf32 = tf32
        cpu = None
        if not args.no_cpu_baseline:
            Lc, Rc, QLc, QRc, Vc = (t.cpu() for t in (L, R, QLo, QRo, V0))
            t = _cpu_time(lambda: torch_refresh(Lc, Rc, QLc, QRc, Vc))
            cpu = {"value": round(t * 1e3, 1), "unit": "ms", "cores": threads, "kind": "reference",
                   "sample": "the reference's refresh lines (soap.py:98-108: two fp64 eigh, the transport in fp32) "
                             "on the same 1024x1024 factors, on the host"}
        fl = 8.0 * d ** 3
        _line(args, "SOAP refresh ms (1024x1024 parameter)", ms_sub, "ms", False,
              "SOAP basis refresh of one 1024x1024 fp32 parameter: warm-started subspace iteration (1 iteration, "
              "CholeskyQR2) for both factors plus the second-moment transport", fl / (ms_tr * 1e-3) / 1e12, clk,
              37 * args.steps, cpu,
              {"ms_per_step": round(ms_sub, 4), "dtype": "f32",
               "transport_ms": round(ms_tr, 4),
               "transport_tflops": round(fl / (ms_tr * 1e-3) / 1e12, 1),
               "refresh_eigh_ms": round(ms_eigh, 3),
               "reference_on_gpu_ms": round(ms_ref_gpu, 3),
               "note": "refresh_eigh: the reference's fp64 eigh bases (library, on the GPU) with the transport on "
                       "this library; reference_on_gpu: the reference's own lines on CUDA tensors (TF32 off); "
                       "the subspace refresh approximates eigh's bases (exact on separated eigenvalues); roofline: "
                       "the transport's four products (8 d^3 FLOPs) on split-tf32 operands",
               "gpu_launches_note": "per refresh: 12 library kernels per basis (three products, each two operand "
                                    "splits and one GEMM), 13 for the transport; plus cuSOLVER's Cholesky and "
                                    "triangular solves"}, peak=peaks()["bf16_sustained"] / 6,
              peak_name="bf16 sustained / 6 (split-tf32: three tf32 passes at half the bf16 rate)")
        return 0
    raise SystemExit(f"unknown workload {w}")


def run_kfac_split(args, rank, world, local_rank):
    """KFAC A and G factor updates (config 4 shapes) shared by all ranks: row bands of each factor
    (``--kfac-split bands``) or whole factors per rank (``--kfac-split factors``)."""
    import torch.distributed as dist
    from pytorch_opt_b200.dist import sharded_factor_updates_, sharded_syrk_ema_
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    g1 = torch.Generator(device=dev).manual_seed(1)
    g2 = torch.Generator(device=dev).manual_seed(2)
    a = torch.randn(8192, 4096, generator=g1, device=dev).bfloat16()
    gr = torch.randn(8192, 4096, generator=g2, device=dev).bfloat16()
    A = torch.empty(4096, 4096, device=dev)
    Gf = torch.empty(4096, 4096, device=dev)
    n = 8192

    def update(first=False):
        if args.kfac_split == "factors":
            sharded_factor_updates_([(A, a, 1.0 / n, 0.95, first), (Gf, gr, float(n), 0.95, first)], rank, world)
        else:
            sharded_syrk_ema_(A, a, 1.0 / n, 0.95, first, rank, world)
            sharded_syrk_ema_(Gf, gr, float(n), 0.95, first, rank, world)
    update(True)
    for _ in range(args.warmup):
        update()

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev)
    clocks.start()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.mark_begin()
    e0.record()
    for _ in range(args.steps):
        update()
    e1.record()
    barrier()
    clocks.mark_end()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if rank == 0:
        fl = 2 * 2.0 * 8192 * 4096 ** 2
        pk = peaks()
        tf = fl / (ms * 1e-3) / 1e12
        print(json.dumps({
            "metric": f"KFAC factor update ms (A and G, 8192x4096 -> 4096^2), split by {args.kfac_split}",
            "value": round(ms, 4),
            "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "KFAC SYRK+EMA of A and G shared by all ranks: "
                                   + ("whole factors per rank (LPT) + one broadcast per factor"
                                      if args.kfac_split == "factors" else
                                      "row bands of equal work, one all_gather and a mirror per factor"),
                       "parallelism": f"{args.kfac_split} x{world}"},
            "roofline": {"bound": "tensor", "kernel": "tc_gemm_kernel (chunked)", "achieved": round(tf, 1),
                         "peak": pk["bf16_sustained"], "unit": "TFLOP/s", "frac": round(tf / pk["bf16_sustained"], 3),
                         "traffic": None, "how": "dense SYRK FLOPs of both factors / the slowest rank's time"},
            "clocks": clk, "gpu_launches": 2 * 2 * args.steps, "e2e": None, "cpu_baseline": None}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-library-bar", action="store_true",
                    help="skip the torch/cuBLAS Newton-Schulz bar of the default workload")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip configs 1-4 in the default workload's line")
    ap.add_argument("--min-timed-seconds", type=float, default=1.0,
                    help="single-GPU workloads repeat their timed calls until the timed region lasts this long "
                         "(so the clock sampler sees it); 0 times exactly --steps calls (for profiling)")
    ap.add_argument("--workload", default="llama8b",
                    choices=("llama8b", "ns768", "ns4096", "gpt2", "shampoo", "kfac", "gemm", "ekfac", "kfac_split",
                             "soap"),
                    help="llama8b (default, config 5); the others are single-GPU measurements of configs 1-4, "
                         "the 4x4096^2 profiling case and the bare product kernel (gemm)")
    ap.add_argument("--gemm", type=int, nargs=3, default=(8192, 8192, 8192), metavar=("M", "N", "K"),
                    help="shape of --workload gemm")
    ap.add_argument("--gemm-dtype", choices=("bf16", "tf32"), default="bf16")
    ap.add_argument("--kfac-split", choices=("factors", "bands"), default="factors",
                    help="--workload kfac_split: whole factors per rank, or row bands of each factor")
    ap.add_argument("--gemm-profile", action="store_true",
                    help="llama8b / ns4096: add the product kernel's wait-cycle shares from one extra untimed step")
    ap.add_argument("--exchange-chunks", type=int, default=None,
                    help="all-gather chunks per step for N > 1 (default 4; 1 = one all-gather after the local step)")
    args = ap.parse_args(argv)
    global MIN_TIMED_SECONDS
    MIN_TIMED_SECONDS = args.min_timed_seconds
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)
    if args.workload == "kfac_split":
        return run_kfac_split(args, rank, world, local_rank)
    if args.workload != "llama8b":
        return run_secondary(args, rank)
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
