#!/usr/bin/env python
"""Benchmark of the B200-native pytorch_opt.ops hot path.

Default workload: one Muon step over the Llama-3-8B
matrix parameters — 32 layers x {q, o: 4096x4096; k, v: 1024x4096;
gate, up: 14336x4096; down: 4096x14336} = 224 bf16 matrices, grads
0.02*N(0,1), momentum 0.95 Nesterov, 5 Newton–Schulz steps, weight decay 0,
lr 0.02 — sharded per matrix over the ranks (FLOP-balanced) and all-gathered
with NCCL. Metric: ms per step (lower is better), the slowest rank's CUDA-event
time; 665.9 TFLOP of dense Newton–Schulz work per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0. ``--impl reference`` times the reference's
own CPU implementation (its ATen extension compiled under ``oracle/_ref``,
else the numpy restatement) on this host's cores over a bounded sample of the
same step, scaled to the full step by FLOPs.
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
METRIC = "Muon NS5 step ms (8B shapes)"
MEASURED_PEAKS = os.path.join(HERE, "MEASURED_PEAKS.json")



# DRAM traffic (ncu dram__bytes_read.sum + dram__bytes_write.sum, summed over
# the Newton-Schulz product launches) of the two captured workloads; the
# commands and per-kernel figures are in profiles/launches_llama8b_muon_step.md
# and profiles/tc_gemm_pair_ns4096.md.
LLAMA_STEP_TRAFFIC = 1_120_000_000_000   # bytes per 1-GPU step (808.5 GB read + 311.5 GB write)
NS4096_CALL_TRAFFIC = 13_660_000_000     # bytes per NS5 call on 4 x 4096^2 (9.65 GB read + 4.01 GB write)

def llama_shapes():
    return LLAMA_LAYER * 32


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

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: torch.device):
        self.proc = None
        self.path = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.gpu = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:
            self.gpu = str(device.index or 0)

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", self.gpu], stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sms, maxes, reasons = [], [], set()
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sms.append(float(parts[1]))
                    maxes.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(self.REASONS, parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(sms)}


# ----------------------------------------------------------- CPU baseline
def cpu_reference_sample(reps: int = 2, warm: int = 1):
    """Time the reference's CPU NS5 on one 4096x4096 bf16 matrix (a q/o projection).

    Returns (seconds per sample, kind, threads, description).
    """
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(1000)
    G = (torch.randn(4096, 4096, generator=g) * 0.02).bfloat16()
    kind, fn = "port", None
    try:
        from oracle import ref_native
        mod = ref_native.load()
        if mod is not None:
            kind = "reference"
            fn = lambda: mod.newton_schulz_orthogonalize(G, 5, 3.4445, -4.7750, 2.0315, 1e-7)  # noqa: E731
    except Exception:
        fn = None
    if fn is None:
        from oracle import ops_np
        Gn = G.float().numpy()
        fn = lambda: ops_np.newton_schulz(Gn, 5, out_bf16=True)  # noqa: E731
    for _ in range(warm):
        fn()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    desc = ("NS5 of one 4096x4096 bf16 matrix (q/o shape) by the reference's own "
            + ("ATen extension (pytorch_opt_ops.cpp, compiled under oracle/_ref)" if kind == "reference"
               else "algorithm restated in numpy (oracle/ops_np.py)")
            + f", median of {reps}, scaled to the 224-matrix step by dense FLOPs")
    return statistics.median(ts), kind, threads, desc


def run_reference_arm(args, rank, world):
    """--impl reference: the reference's CPU path, rank 0 only."""
    if rank != 0:
        return 0
    total = sum(ns_flops(r, c) for r, c in llama_shapes())
    sample = ns_flops(4096, 4096)
    times = []
    kind = threads = desc = None
    for i in range(args.warmup + args.steps):
        t, kind, threads, desc = cpu_reference_sample(reps=1, warm=0)
        if i >= args.warmup:
            times.append(t * total / sample * 1e3)
    ms = statistics.median(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(ms, 3), "unit": "ms", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": "Muon NS5 step over Llama-3-8B matrix params (224 matrices)", "ns_steps": 5,
                   "parallelism": "host CPU, all threads"},
        "cpu_baseline": {"value": round(ms, 3), "unit": "ms", "cores": threads, "kind": kind, "sample": desc},
        "e2e": {"value": round(ms, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------- our arm
def fill_normal(t: torch.Tensor, seed: int, scale: float):
    g = torch.Generator(device=t.device).manual_seed(seed)
    t.copy_(torch.randn(t.shape, generator=g, device=t.device, dtype=torch.float32).mul_(scale))


def run_ours(args, rank, world, local_rank):
    from pytorch_opt_b200.dist import ShardLayout, ShardedMuon
    import torch.distributed as dist

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
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
    total_flops = sum(ns_flops(r, c) for r, c in shapes)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------------------------------------------- device-resident run
    for _ in range(args.warmup):
        sm.step()
    barrier()
    clocks = ClockSampler(dev)
    clocks.start()
    ns_events: list = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        sm.step(ns_events)
    e1.record(stream)
    barrier()
    clk = clocks.stop()
    step_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    ns_ms_local = sum(a.elapsed_time(b) for a, b in ns_events) / args.steps
    gemm_tflops_local = local_flops / (ns_ms_local * 1e-3) / 1e12 if ns_ms_local > 0 else 0.0
    launches = sm.launches_per_step() * args.steps

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
        e2e = {"value": round(max_over_ranks(a0.elapsed_time(a1) / args.steps), 3), "unit": "ms",
               "h2d_bytes_per_step": int(layout.slot_elements(rank) * 2), "d2h_bytes_per_step": 8,
               "api": "pytorch_opt_b200.dist.ShardedMuon.step_from_host (per-group H2D copies overlapped with "
                      "the grouped Muon kernels, C ABI) + NCCL all-gather"}

    # --------------------------------------------------------- CPU baseline
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        t, kind, threads, desc = cpu_reference_sample()
        cpu = {"value": round(t * total_flops / ns_flops(4096, 4096) * 1e3, 1), "unit": "ms", "cores": threads,
               "kind": kind, "sample": desc}

    gemm_tflops = max_over_ranks(-gemm_tflops_local)  # slowest rank's rate
    gemm_tflops = -gemm_tflops
    pk = peaks()
    mix_peak = 1.0 / (0.6 / pk["bf16_sustained"] + 0.4 / (pk["bf16_sustained"] / 2))
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(step_ms, 3), "unit": "ms", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(step_ms, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "precision": "bf16 tensor-core products on NS steps 1-3, tf32 on steps 4-5, fp32 accumulation",
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
                         "traffic": LLAMA_STEP_TRAFFIC if world == 1 else None,
                         "traffic_unit": "DRAM bytes per step of all Newton-Schulz product launches (ncu "
                                         "dram__bytes_read.sum + dram__bytes_write.sum; 1 GPU only, "
                                         "profiles/launches_llama8b_muon_step.md)",
                         "peak_source": pk["source"] + " bf16 sustained (MEASURED_PEAKS.json)",
                         "peak_bf16_tf32_mix": round(mix_peak, 1),
                         "frac_of_mix": round(gemm_tflops / mix_peak, 3),
                         "how": "dense NS FLOPs of the rank's matrices / CUDA-event time of its Newton-Schulz "
                                "calls inside the timed steps (includes two small packing kernels per call)"},
            "clocks": clk,
            "gpu_launches": int(launches),
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------- secondary workloads (1 GPU)
def _timed(fn, steps, warmup, dev, flush=None):
    """Per-call CUDA-event time (ms), L2 flushed between calls (outside the timed intervals)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev)
    clocks.start()
    pairs = []
    for _ in range(steps):
        if flush is not None:
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        pairs.append((a, b))
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    return sum(a.elapsed_time(b) for a, b in pairs) / steps, clk


def _line(args, metric, value, unit, hib, workload, tflops, clk, launches, cpu, extra=None, traffic=None):
    pk = peaks()
    line = {"metric": metric, "value": round(value, 4), "unit": unit, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": None, "higher_is_better": hib, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": workload, "l2": "flushed between timed calls (256 MiB write)"},
            "roofline": {"bound": "tensor", "kernel": "tc_gemm_pair_kernel", "achieved": round(tflops, 1),
                         "peak": pk["bf16_sustained"], "unit": "TFLOP/s",
                         "frac": round(tflops / pk["bf16_sustained"], 3), "traffic": traffic,
                         "peak_source": pk["source"] + " bf16 sustained (MEASURED_PEAKS.json)",
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


def run_secondary(args, rank):
    if rank != 0:
        return 0
    from pytorch_opt_b200 import native
    from pytorch_opt_b200.muon import GroupedMuon, MuonGroup

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    try:
        from oracle import ref_native
        ref = ref_native.load()
    except Exception:
        ref = None
    threads = len(os.sched_getaffinity(0))
    w = args.workload
    if w in ("ns768", "ns4096"):
        if w == "ns768":   # config 1
            g = torch.Generator().manual_seed(0)
            Gc = torch.randn(768, 3072, generator=g)
            desc, fl = "NS5 of one 768x3072 fp32 matrix, N(0,1), seed 0 (config 1)", ns_flops(768, 3072)
        else:              # a batch of q/o-shaped matrices: the profiling case of the main workload's products
            g = torch.Generator().manual_seed(1000)
            Gc = (torch.randn(4, 4096, 4096, generator=g) * 0.02).bfloat16()
            desc, fl = "NS5 of 4 x 4096x4096 bf16 matrices (Llama q/o shape), 0.02 N(0,1)", 4 * ns_flops(4096, 4096)
        G = Gc.to(dev)
        ms, clk = _timed(lambda: native.newton_schulz_orthogonalize(G, 5, 3.4445, -4.7750, 2.0315, 1e-7),
                         args.steps, args.warmup, dev, flush)
        cpu = None
        if ref is not None and not args.no_cpu_baseline:
            one = Gc if Gc.dim() == 2 else Gc[0]
            t = _cpu_time(lambda: ref.newton_schulz_orthogonalize(one, 5, 3.4445, -4.7750, 2.0315, 1e-7))
            cpu = {"value": round(t * 1e3 * (fl / ns_flops(*one.shape)), 2), "unit": "ms", "cores": threads,
                   "kind": "reference", "sample": "the reference's ATen NS5 on one matrix of the workload"}
        m = min(G.shape[-2:])
        launches = 2 + 3 * 5
        _line(args, f"{'NS5 768x3072' if w == 'ns768' else 'NS5 4x4096^2'} ms", ms, "ms", False, desc,
              fl / (ms * 1e-3) / 1e12, clk, launches * args.steps, cpu, {"ms_per_step": round(ms, 4)},
              traffic=NS4096_CALL_TRAFFIC if w == "ns4096" else None)
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
    if w == "gpt2":        # config 2
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
        ms, clk = _timed(opt.step, args.steps, args.warmup, dev, flush)
        cpu = None
        if ref is not None and not args.no_cpu_baseline:
            gs = (torch.randn(768, 2304) * 0.02).bfloat16()
            t = _cpu_time(lambda: ref.newton_schulz_orthogonalize(gs, 5, 3.4445, -4.7750, 2.0315, 1e-7))
            cpu = {"value": round(t * 1e3 * fl / ns_flops(768, 2304), 1), "unit": "ms", "cores": threads,
                   "kind": "reference", "sample": "the reference's ATen NS5 on one 768x2304 matrix, scaled by FLOPs"}
        _line(args, "GPT-2-small Muon step ms", ms, "ms", False,
              "Muon step over 48 GPT-2-small matrices (bf16, 0.02 N(0,1), momentum 0.95 Nesterov, 5 NS steps)",
              fl / (ms * 1e-3) / 1e12, clk, opt.launches_per_step() * args.steps, cpu,
              {"ms_per_step": round(ms, 4)})
        return 0
    if w == "shampoo":     # config 3
        res = {}
        lib_iters = {}
        for d in (1024, 2048, 4096):
            g = torch.Generator(device=dev).manual_seed(d * 100)
            Gs = torch.randn(8, d, 2 * d, generator=g, device=dev)
            L = Gs @ Gs.mT / (2 * d) + 1e-6 * torch.eye(d, device=dev)
            del Gs
            from pytorch_opt_b200 import _lib
            lib = _lib.load()
            out = torch.empty_like(L)
            its = torch.zeros(8, dtype=torch.int32, device=dev)
            nbytes = lib.po_root_workspace_bytes(8, d, 4)
            ws = _lib.workspace(nbytes, dev)

            def call():
                _lib.check(lib.po_inverse_root(L.data_ptr(), 0, 8, d, d, d * d, out.data_ptr(), d, d * d, 4, 1e-8,
                                               100, 1e-10, its.data_ptr(), ws.data_ptr(), nbytes,
                                               _lib.stream_ptr(dev)), "root")
            ms, clk = _timed(call, args.steps, args.warmup, dev, flush)
            n_it = its.tolist()
            fl = sum(8.0 * d ** 3 * i for i in n_it)
            res[d] = {"ms": round(ms, 3), "iters": n_it[0], "tflops": round(fl / (ms * 1e-3) / 1e12, 1)}
            lib_iters[d] = n_it
            del L, out, ws
        cpu = None
        if ref is not None and not args.no_cpu_baseline:
            g = torch.Generator().manual_seed(1024 * 100)
            Gm = torch.randn(1024, 2048, generator=g)
            Lc = Gm @ Gm.T / 2048 + 1e-6 * torch.eye(1024)
            t = _cpu_time(lambda: ref.inverse_matrix_root(Lc, 4, 1e-8, "newton", True, 100, 1e-10))
            cpu = {"value": round(t * 1e3 * 8 * 64, 1), "unit": "ms", "cores": threads, "kind": "reference",
                   "sample": "the reference's ATen coupled Newton (fp64) on one d=1024 factor, x8 factors x (4096/1024)^3"}
        _line(args, "Shampoo inverse 4th root TFLOP/s (8 x d=4096)", res[4096]["tflops"], "TFLOP/s", True,
              "coupled-Newton inverse 4th roots of 8 SPD factors per size, L = G G^T/2d + 1e-6 I, damping 1e-8",
              res[4096]["tflops"], clk, None, cpu, {"ms_per_step": res[4096]["ms"], "per_size": res})
        return 0
    if w == "kfac":        # config 4
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
        ms_u, clk = _timed(update, args.steps, args.warmup, dev, flush)
        tr_a = float(A.diagonal().sum()) / 4096
        tr_g = float(Gf.diagonal().sum()) / 4096
        pi = math.sqrt(tr_a / tr_g)
        ga, gg = pi * math.sqrt(1e-3), math.sqrt(1e-3) / pi

        def inverse():
            native.damped_inverse(A, ga)
            native.damped_inverse(Gf, gg)
        ms_i, _ = _timed(inverse, max(1, args.steps // 2), 1, dev, flush)
        fl_u = 2 * 2.0 * 8192 * 4096 ** 2
        cpu = None
        if not args.no_cpu_baseline:
            ac = torch.randn(2048, 4096).float()
            t = _cpu_time(lambda: ac.T @ ac)
            cpu = {"value": round(t * 1e3 * 4 * 2, 1), "unit": "ms", "cores": threads, "kind": "reference",
                   "sample": "the reference's factor GEMM (torch fp32 a^T a, kron.py:113) on 2048 of the 8192 rows, "
                             "x4 rows x2 factors (update only; its fp64 eigh inverse is ~77 s per factor on 8 cores)"}
        _line(args, "KFAC factor update ms (A and G, 8192x4096 -> 4096^2)", ms_u, "ms", False,
              "KFAC SYRK+EMA of A = a^T a/n and G = (n g)^T (n g)/n, a, g 8192x4096 bf16, beta 0.95; "
              "then pi-damped inverses (lambda 1e-3) by coupled Newton p=1",
              fl_u / (ms_u * 1e-3) / 1e12, clk, None, cpu,
              {"ms_per_step": round(ms_u, 4), "damped_inverse_ms_both": round(ms_i, 3)})
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
    raise SystemExit(f"unknown workload {w}")


def run_kfac_split(args, rank, world, local_rank):
    """KFAC A and G factor updates (config 4 shapes) shared by all ranks: row bands + all_reduce."""
    import torch.distributed as dist
    from pytorch_opt_b200.dist import sharded_syrk_ema_
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
    barrier()
    clocks = ClockSampler(dev)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        update()
    e1.record()
    barrier()
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
            "metric": "KFAC factor update ms (A and G, 8192x4096 -> 4096^2), split by row bands", "value": round(ms, 4),
            "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "KFAC SYRK+EMA of A and G shared by all ranks: row bands of equal work, "
                                   "one all_reduce and a mirror per factor", "parallelism": f"row bands x{world}"},
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
    ap.add_argument("--workload", default="llama8b",
                    choices=("llama8b", "ns768", "ns4096", "gpt2", "shampoo", "kfac", "gemm", "ekfac", "kfac_split"),
                    help="llama8b (default, config 5); the others are single-GPU measurements of configs 1-4, "
                         "the 4x4096^2 profiling case and the bare product kernel (gemm)")
    ap.add_argument("--gemm", type=int, nargs=3, default=(8192, 8192, 8192), metavar=("M", "N", "K"),
                    help="shape of --workload gemm")
    ap.add_argument("--gemm-dtype", choices=("bf16", "tf32"), default="bf16")
    ap.add_argument("--exchange-chunks", type=int, default=None,
                    help="all-gather chunks per step for N > 1 (default 4; 1 = one all-gather after the local step)")
    args = ap.parse_args(argv)
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
