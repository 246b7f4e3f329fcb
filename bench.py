#!/usr/bin/env python
"""Benchmark: block-permute / accumulate HBM GB/s on B200.

Workload (one step, per rank): the U(1) 4-leg TensorMap hom((v, v), (v, v)),
each leg carrying charges -4..4 with degeneracy round(64 exp(-q^2 / 8))
(N = 1,023,777,634 elements, 489 sub-blocks, 17 blocks), synthetic N(0, 1)
data from a seed:
  1. y = permute(x, ((2, 0), (3, 1)))          (alpha = 1, beta = 0)
  2. z = 1 * permute(x, ((2, 0), (3, 1))) + 1 * z   (beta = 1 accumulate)
Algorithmic bytes per step: 2 N s + 3 N s (s = element size).  Inputs (4 GB
for f32) exceed the 126 MB L2, so no flush is needed between steps.

Multi-GPU (torchrun, one process per GPU): ONE tensor is split by sector.
The permute's 489 records are partitioned by longest-processing-time over the
ranks (cost = bytes moved); each rank holds its records' source sub-blocks
compacted in its own HBM and writes their destination sub-blocks compacted,
so the timed kernels need no communication (strong scaling: total work is
fixed as N grows).  The NCCL all-gather of the compacted outputs plus the
engine copy that unpacks them into the packed layout is timed separately.

``--impl reference`` times the reference's own CPU executors (oracle/_ref,
compiled from the reference sources) on the host cores.
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
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "block-permute/accumulate HBM GB/s"
UNIT = "GB/s"


def parse():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--dtype", choices=("f32", "c64"), default="f32")
    p.add_argument("--e2e-steps", type=int, default=None, help="end-to-end steps (default: min(steps, 8))")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-contraction", action="store_true", help="skip the contraction TFLOP/s measurement")
    p.add_argument("--no-trace", action="store_true", help="skip the partial-trace measurement")
    p.add_argument("--no-grouped", action="store_true", help="skip the grouped-transform measurement")
    p.add_argument("--grouped-extent", type=int, default=16,
                   help="grouped workload block extent d (blocks d^4; 16 = the benchmark, smaller for profiling)")
    p.add_argument("--trace-degeneracies", default="4,3",
                   help="Z2 x U(1) trace workload degeneracies for parity 0,1 (4,3 = the benchmark; smaller for profiling)")
    p.add_argument("--scale", type=int, default=64,
                   help="leg degeneracy scale (64 = the benchmark workload; smaller values for profiling)")
    return p.parse_args()


def workload_space(scale: int = 64):
    from tensor0_b200.structure import U1Irrep, hom, space
    degs = {q: int(round(scale * np.exp(-q * q / 8))) for q in range(-4, 5)}
    v = space(U1Irrep, degs)
    return hom((v, v), (v, v)), degs


def workload_config(args, elements: int):
    return {"workload": "u1-4leg permute((2,0),(3,1)) + beta=1 accumulate",
            "legs": f"U1 q=-4..4, deg round({args.scale} exp(-q^2/8))", "elements": elements,
            "sub_blocks": 489, "dtype": args.dtype, "l2": "inputs larger than the 126 MB L2, no flush",
            "parallelism": "single GPU"}


# ---------------------------------------------------------------------------
# CPU: the reference's own executors on a bounded sample.


SAMPLE_SCALE = 40     # degeneracies round(40 exp(-q^2/8)): same structure, ~1/6.8 of the elements


def cpu_reference_steps(dtype_name: str, steps: int, warmup: int, threads: int, scale: int):
    """Time the compiled reference (oracle/_ref) on the workload at degeneracy
    `scale`: instantiated once, then `warmup` untimed and `steps` timed
    executions of the permute-accumulate and the beta = 1 update; GB/s."""
    from oracle import ref
    from tensor0_b200.structure import degeneracy_structure
    from tensor0_b200.tensor_map import permute_plan
    h, degs = workload_space(scale)
    plan = permute_plan(h, (2, 0), (3, 1))
    n = degeneracy_structure(h).total_dim
    dtype = np.float32 if dtype_name == "f32" else np.complex64
    rng = np.random.default_rng(7)
    if dtype == np.complex64:
        x = np.empty(n, np.complex64)
        x.real = rng.standard_normal(n, dtype=np.float32)
        x.imag = rng.standard_normal(n, dtype=np.float32)
    else:
        x = rng.standard_normal(n, dtype=np.float32)
    z = np.zeros(plan.output_size, dtype)
    y = np.empty(plan.output_size, dtype)
    records = np.arange(len(plan.transform.src))
    ones = [np.float32(1.0)] * len(records)
    ref.set_threads(threads)
    accumulate = ref.Prepared(3, plan.words, records, outputs_disjoint=True)
    update = ref.Prepared(1, plan.words)
    item = np.dtype(dtype).itemsize
    step_bytes = 5 * n * item
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        accumulate.accumulation(x, y, ones, threads=threads)
        update.update(x, z, z, np.float32(1.0), np.float32(1.0), threads=threads)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    seconds = sum(times)
    sample = (f"u1-4leg deg round({scale} exp(-q^2/8)) {dict(degs)}, N={n} ({step_bytes / 1e9:.2f} GB "
              f"algorithmic per step), {steps} timed steps after {warmup} warm-up, instantiated once")
    return step_bytes * steps / seconds / 1e9, seconds * 1e3 / steps, sample, n


def run_reference(args, rank: int):
    """The reference's CPU executors on the same workload as the GPU arm (full
    size), on all host cores; rank 0 only."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    value, ms, sample, n = cpu_reference_steps(args.dtype, args.steps, args.warmup, threads, args.scale)
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": args.dtype, "data": "synthetic N(0,1), seeded",
            "config": workload_config(args, n), "impl": "reference",
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU clocks during the timed region.


class ClockSampler:
    """SM clock, power and throttle reasons sampled every 10 ms through NVML
    while the timed region runs (reads only; no setting is changed)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.samples: list[tuple[float, float, float, int]] = []
        self.stop = threading.Event()
        self.thread = None
        self.handle = None
        self.nvml = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            for candidate in (self.uuid, "GPU-" + self.uuid):
                try:
                    self.handle = pynvml.nvmlDeviceGetHandleByUUID(candidate)
                    break
                except pynvml.NVMLError:
                    continue
            if self.handle is not None:
                self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
                self.thread = threading.Thread(target=self._run, daemon=True)
                self.thread.start()
        except Exception:
            self.handle = None
        return self

    def _run(self):
        nvml = self.nvml
        reasons = getattr(nvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nvml.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop.is_set():
            try:
                sm = nvml.nvmlDeviceGetClockInfo(self.handle, nvml.NVML_CLOCK_SM)
                power = nvml.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
                mask = reasons(self.handle)
                util = nvml.nvmlDeviceGetUtilizationRates(self.handle).gpu
                self.samples.append((float(sm), power, float(util), int(mask)))
            except Exception:
                pass
            self.stop.wait(0.01)

    def __exit__(self, *exc):
        self.stop.set()
        if self.thread:
            self.thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        mask = 0
        for s in self.samples:
            mask |= s[3]
        reasons = sorted(name for bit, name in self.REASONS.items() if mask & bit)
        return {"sm_mhz": statistics.median(s[0] for s in self.samples), "sm_max_mhz": float(self.max_mhz),
                "power_w_max": round(max(s[1] for s in self.samples), 1), "reasons": reasons,
                "samples": len(self.samples), "source": "nvml, 10 ms"}


DMRG_DEGENERACIES = [8, 18, 37, 68, 112, 166, 219, 259, 274, 259, 219, 166, 112, 68, 37, 18, 8]


def contraction_bench(device, steps: int, warmup: int):
    """DMRG environment contraction L . A in f64: chi = 2048 over U(1) charges -8..8
    (degeneracies exp(-q^2 / 18) rounded to sum 2048), physical d = 2 {0, 1}, MPO
    bond w = 5 (charge 0).  Times the whole tensorcontract (operand permutes plus
    the grouped sector GEMM) and the sector GEMM launch alone, against an f64 cuBLAS
    GEMM measured here (8192^3, best of 5)."""
    import torch
    from tensor0_b200 import stride
    from tensor0_b200.structure import U1Irrep, degeneracy_structure, hom, space
    from tensor0_b200.tensor_map import TensorMap, contract_plan, permute, tensorcontract
    chi = space(U1Irrep, {q: d for q, d in zip(range(-8, 9), DMRG_DEGENERACIES)})
    phys = space(U1Irrep, {0: 1, 1: 1})
    w = space(U1Irrep, {0: 5})
    a_space, l_space = hom((chi, phys), (chi,)), hom((chi,), (chi, w))
    gen = torch.Generator(device=device)
    gen.manual_seed(4)
    a = TensorMap(a_space, torch.randn(degeneracy_structure(a_space).total_dim, generator=gen, device=device,
                                       dtype=torch.float64))
    l = TensorMap(l_space, torch.randn(degeneracy_structure(l_space).total_dim, generator=gen, device=device,
                                       dtype=torch.float64))
    axes, output = ((1,), (0,)), (((0, 0), (1, 1)), ((0, 2), (1, 2)))
    plan = contract_plan(l_space, a_space, (1,), (0,), output)
    flops = plan.gemm.flops_real
    stream = torch.cuda.current_stream(device)

    def timed(fn, count):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(count):
            fn()
        end.record(stream)
        torch.cuda.synchronize()
        return start.elapsed_time(end) / count

    whole_ms = timed(lambda: tensorcontract(l, a, axes=axes, output=output), steps)
    left, right = (a, l) if plan.reversed_operands else (l, a)
    lcan, rcan = permute(left, plan.left_p).data, permute(right, plan.right_p).data
    out = torch.empty(degeneracy_structure(plan.canonical).total_dim, dtype=torch.float64, device=device)
    gemm_ms = timed(lambda: stride.sector_gemm(plan.gemm, lcan, rcan, out), steps)
    x = torch.randn(8192, 8192, dtype=torch.float64, device=device)
    y = torch.randn(8192, 8192, dtype=torch.float64, device=device)
    cublas_ms = min(timed(lambda: torch.matmul(x, y), 1) for _ in range(5))
    peak = 2 * 8192 ** 3 / (cublas_ms / 1e3) / 1e12
    gemm_tf = flops / (gemm_ms / 1e3) / 1e12
    return {"metric": "contraction TFLOP/s", "value": round(flops / (whole_ms / 1e3) / 1e12, 3), "unit": "TFLOP/s",
            "dtype": "f64", "workload": "DMRG L.A, U1 chi=2048 (sigma=3), d=2, w=5", "sectors": plan.gemm.sectors,
            "flops_per_step": flops, "ms_per_step": round(whole_ms, 4),
            "gemm": {"kernel": "DmmaGemm (sector GEMM launch alone)", "value": round(gemm_tf, 3),
                     "ms": round(gemm_ms, 4), "peak": round(peak, 2), "frac": round(gemm_tf / peak, 4),
                     "peak_kind": "measured here: cuBLAS f64 GEMM 8192^3, best of 5"}}


def trace_bench(device, steps: int, warmup: int, degeneracies=(4, 3)):
    """Partial trace of the Z2 x U(1) 6-leg tensor (degeneracies 4 / 3, q in
    -3..3: all 298,592 sub-blocks, N = 548,896,075 f64) over the leg pairs
    (1, 4) and (2, 5) down to a 2-leg map: one reduction call (two kernels).
    It reads only the 2744 contributing records' diagonal elements; GB/s are
    given at 8 B per element read or written, and at the 32-byte DRAM sector
    each scattered read occupies."""
    import torch
    from tensor0_b200 import _native, stride
    from tensor0_b200.structure import ProductSector, U1Irrep, Z2Irrep, degeneracy_structure, hom, space
    from tensor0_b200.tensor_map import trace_plan
    w = space(ProductSector(Z2Irrep, U1Irrep), {(p, q): degeneracies[p] for p in (0, 1) for q in range(-3, 4)})
    h = hom((w, w, w), (w, w, w))
    n = degeneracy_structure(h).total_dim
    tp = trace_plan(h, (1, 2), (4, 5), (0,), (3,))
    engine = tp.engine_plan(torch.float64)
    gen = torch.Generator(device=device)
    gen.manual_seed(3)
    x = torch.randn(n, generator=gen, device=device, dtype=torch.float64)
    coefficients = torch.as_tensor(tp.coefficients, dtype=torch.float64, device=device)
    out = torch.empty(engine.output_size, dtype=torch.float64, device=device)
    scratch = torch.empty(engine.scratch_elements, dtype=torch.float64, device=device)
    # Elements read: every contributing record's open x traced box.
    words = np.asarray(tp.words, dtype=np.int64).view(np.uint64)
    read = 0
    at = 4
    for _ in range(int(words[3])):
        rank = int(words[at])
        shape = words[at + 3: at + 3 + rank]
        read += int(np.prod(shape))
        at += 3 + 5 * rank
    call = lambda: stride.execute_reduction(x, engine, coefficients, out=out, scratch=scratch)
    for _ in range(warmup):
        call()
    stream = torch.cuda.current_stream(device)
    eager, _ = timed_events(stream, steps, lambda _: call())
    # A call is a few microseconds of device work, less than the host needs to
    # enqueue it from Python: the device time per call is taken from a CUDA
    # graph of `per_graph` consecutive calls (the C ABI allocates nothing and
    # never synchronizes, so it captures as is).
    per_graph = 20
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(per_graph):
            call()
    for _ in range(warmup):
        graph.replay()
    total, _ = timed_events(stream, steps, lambda _: graph.replay())
    ms = total / steps / per_graph
    del graph
    algorithmic = 8 * (read + engine.output_size)
    sectors = 32 * read + 8 * engine.output_size
    peak, peak_kind = load_peaks()
    return {"metric": "partial trace GB/s",
            "workload": f"Z2xU1 6-leg deg {degeneracies[0]}/{degeneracies[1]} q=-3..3, trace (1,4),(2,5), f64",
            "elements": n, "records": int(tp.records), "elements_read": read, "outputs": engine.output_size,
            "ms_per_call": round(ms, 5), "timing": f"CUDA graph of {per_graph} calls, replayed",
            "ms_per_call_enqueued_from_python": round(eager / steps, 5),
            "kernels_per_call": engine.info["kernels_per_call"],
            "value": round(algorithmic / (ms / 1e3) / 1e9, 3), "unit": "GB/s",
            "roofline": {"bound": "hbm (scattered 8-byte reads)", "peak": peak, "peak_kind": peak_kind,
                         "frac_at_8_bytes": round(algorithmic / (ms / 1e3) / 1e9 / peak, 5),
                         "frac_at_32_byte_sectors": round(sectors / (ms / 1e3) / 1e9 / peak, 5)}}


def grouped_bench(device, steps: int, warmup: int, extent: int = 16):
    """Grouped transform of a synthetic SU(2)-like permute: 384 groups of
    1-4 fusion trees (as many destination as source trees; 845 of each with
    this seed) over d^4 blocks (d = 16: 65,536 f64 elements, 512 KiB per
    block), permutation (2, 0, 3, 1), random orthogonal basis matrices,
    packed source and destination storage of 0.44 GB each (larger than the
    L2).  One launch per call; GB/s at one read of every source block and one
    write of every destination block."""
    import torch
    from types import SimpleNamespace
    from tensor0_b200 import _native, stride
    rng = np.random.default_rng(5)
    shape = (extent,) * 4
    permutation = (2, 0, 3, 1)
    logical = tuple(shape[p] for p in permutation)
    count = extent ** 4
    trees = rng.choice([1, 2, 3, 4], size=384, p=[0.3, 0.3, 0.25, 0.15])
    sources, destinations, groups = [], [], []
    for n in trees:
        n = int(n)
        q, _ = np.linalg.qr(rng.standard_normal((n, n)))
        src = list(range(len(sources), len(sources) + n))
        dst = list(range(len(destinations), len(destinations) + n))
        for _ in range(n):
            sources.append(SimpleNamespace(sizes=shape, strides=stride.contiguous_strides(shape),
                                           offset=len(sources) * count))
            destinations.append(SimpleNamespace(sizes=logical, strides=stride.contiguous_strides(logical),
                                                offset=len(destinations) * count))
        groups.append(SimpleNamespace(src_indices=tuple(src), dst_indices=tuple(dst), transform=q))
    words, matrices = stride.encode_grouped(sources, destinations, permutation, groups,
                                            source_size=len(sources) * count,
                                            output_size=len(destinations) * count)
    plan = stride.Plan(_native.OP_GROUPED, words, element_bytes=8)
    gen = torch.Generator(device=device)
    gen.manual_seed(7)
    x = torch.randn(plan.source_size, generator=gen, device=device, dtype=torch.float64)
    out = torch.empty(plan.output_size, device=device, dtype=torch.float64)
    m = torch.from_numpy(np.concatenate(matrices).astype(np.float64)).to(device)
    for _ in range(warmup):
        stride.execute_grouped(x, plan, m, out=out)
    stream = torch.cuda.current_stream(device)
    total, _ = timed_events(stream, steps, lambda _: stride.execute_grouped(x, plan, m, out=out))
    ms = total / steps
    algorithmic = 8 * (plan.source_size + plan.output_size)
    peak, peak_kind = load_peaks()
    achieved = algorithmic / (ms / 1e3) / 1e9
    return {"metric": "grouped transform GB/s",
            "workload": f"SU2-like grouped permute (2,0,3,1): 384 groups of 1-4 trees, {len(sources)} blocks of "
                        f"{extent}^4 f64 per side",
            "groups": len(groups), "blocks": len(sources), "elements_per_side": plan.source_size,
            "ms_per_call": round(ms, 5), "kernels_per_call": plan.info["kernels_per_call"],
            "value": round(achieved, 3), "unit": "GB/s",
            "roofline": {"bound": "hbm", "kernel": "GroupedKernel<double, double>", "peak": peak,
                         "peak_kind": peak_kind, "frac": round(achieved / peak, 4),
                         "algorithmic_bytes_per_launch": algorithmic}}


def gemm_f32_bench(device, steps: int, warmup: int, size: int = 4096, dtype: str = "f32"):
    """One single-precision sector of size^3 through the tcgen05 GEMM
    (three-term TF32 split, FP32 register accumulation per K slice; c64 as four
    real products) beside cuBLAS (TF32 off) on the same operands; TFLOP/s at
    2 size^3 (f32) or 8 size^3 (c64) per call."""
    import torch
    from tensor0_b200 import stride
    tdtype = torch.complex64 if dtype == "c64" else torch.float32
    plan = stride.GemmPlan(np.array([(size, size, size, 0, 0, 0)]))
    gen = torch.Generator(device=device)
    gen.manual_seed(11)
    left = torch.randn(size * size, generator=gen, device=device, dtype=tdtype)
    right = torch.randn(size * size, generator=gen, device=device, dtype=tdtype)
    out = torch.empty(size * size, device=device, dtype=tdtype)
    stream = torch.cuda.current_stream(device)
    for _ in range(warmup):
        stride.sector_gemm(plan, left, right, out)
    total, _ = timed_events(stream, steps, lambda _: stride.sector_gemm(plan, left, right, out))
    a, b = left.view(size, size), right.view(size, size)
    previous = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    for _ in range(warmup):
        torch.matmul(a, b)
    reference, _ = timed_events(stream, steps, lambda _: torch.matmul(a, b))
    torch.backends.cuda.matmul.allow_tf32 = previous
    flops = (8.0 if dtype == "c64" else 2.0) * size ** 3
    wide = torch.complex128 if dtype == "c64" else torch.float64
    exact = a.to(wide) @ b.to(wide)
    error = float((out.view(size, size).to(wide) - exact).abs().max() / exact.abs().max())
    kernel = "TcGemmComplex (tcgen05.mma kind::tf32, 4 products x 3 terms)" if dtype == "c64" else \
        "TcGemm (tcgen05.mma kind::tf32, 3 terms)"
    return {"metric": f"{dtype} sector GEMM TFLOP/s", "kernel": kernel,
            "shape": f"{size}^3", "ms_per_call": round(total / steps, 4),
            "value": round(flops / (total / steps / 1e3) / 1e12, 2), "unit": "TFLOP/s",
            "cublas": round(flops / (reference / steps / 1e3) / 1e12, 2), "max_relative_error": error}


def device_uuid(index: int) -> str:
    import torch
    try:
        return str(torch.cuda.get_device_properties(index).uuid)
    except Exception:
        return ""


# ---------------------------------------------------------------------------
# GPU arm.


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        peaks = json.loads(path.read_text())
        return float(peaks["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic():
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "map_kernel_u1_permute_accumulate.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_update_launch_full_size:"):
            try:
                return float(line.split(":", 1)[1])
            except ValueError:
                return None
    return None


def timed_events(stream, count, body):
    """Device time (ms) of `count` calls of body() on `stream`, and per-call marks."""
    import torch
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(count + 1)]
    torch.cuda.synchronize()
    for k in range(count):
        marks[k].record(stream)
        body(k)
    marks[count].record(stream)
    torch.cuda.synchronize()
    return marks[0].elapsed_time(marks[count]), [marks[k].elapsed_time(marks[k + 1]) for k in range(count)]


def max_over_ranks(value: float, device) -> float:
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_sharded(args, world: int, rank: int, device):
    """The workload split by sector over `world` ranks (see the module docstring)."""
    import torch
    import torch.distributed as dist

    from tensor0_b200 import _native, stride
    from tensor0_b200.sharding import gather_words, shard_capacity, shard_permute

    h, _ = workload_space(args.scale)
    plan = permute_plan_of(h)
    item = 4 if args.dtype == "f32" else 8
    tdtype = torch.float32 if args.dtype == "f32" else torch.complex64
    n = plan.source_size
    shard = shard_permute(plan, rank, world, item)
    records = shard.records.size
    acc = stride.Plan(_native.OP_ACCUMULATION, shard.words, element_bytes=item,
                      coefficient_records=np.arange(records), outputs_disjoint=True)
    upd = stride.Plan(_native.OP_UPDATE, shard.words, element_bytes=item)
    capacity = shard_capacity(plan, world, item)
    gen = torch.Generator(device=device)
    gen.manual_seed(1000 + rank)
    x = torch.randn(shard.local_source_size, generator=gen, device=device, dtype=tdtype)
    z = torch.randn(shard.local_output_size, generator=gen, device=device, dtype=tdtype)
    y_pad = torch.zeros(capacity, device=device, dtype=tdtype)
    y = y_pad[: shard.local_output_size]
    ones = torch.ones(records, dtype=torch.float32, device=device)
    alpha = torch.ones(1, dtype=torch.float32, device=device)
    beta = torch.ones(1, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)

    def step():
        stride.execute_accumulation(x, acc, ones, out=y)
        stride.execute_update(x, z, alpha, beta, upd, out=z)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    launches0 = stride.kernel_launches()
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps + 1)]
    with ClockSampler(device_uuid(device.index)) as clocks:
        torch.cuda.synchronize()
        for k in range(args.steps):
            marks[2 * k].record(stream)
            stride.execute_accumulation(x, acc, ones, out=y)
            marks[2 * k + 1].record(stream)
            stride.execute_update(x, z, alpha, beta, upd, out=z)
        marks[2 * args.steps].record(stream)
        torch.cuda.synchronize()
    launches = stride.kernel_launches() - launches0
    local_ms = marks[0].elapsed_time(marks[2 * args.steps])
    elapsed = max_over_ranks(local_ms, device)
    step_bytes = 5 * n * item
    value = step_bytes * args.steps / (elapsed / 1e3) / 1e9
    update_ms = statistics.mean(marks[2 * k + 1].elapsed_time(marks[2 * k + 2]) for k in range(args.steps))
    permute_ms = statistics.mean(marks[2 * k].elapsed_time(marks[2 * k + 1]) for k in range(args.steps))
    local_update_bytes = 3 * shard.local_output_size * item
    local_permute_bytes = 2 * shard.local_output_size * item

    # Gather: NCCL all-gather of the padded compacted outputs, then one engine
    # copy unpacking them into the packed layout of the whole tensor.
    unpack = stride.Plan(_native.OP_COPY, gather_words(plan, world, item), element_bytes=item)
    gathered = torch.empty(world * capacity, device=device, dtype=tdtype)
    full = torch.empty(plan.output_size, device=device, dtype=tdtype)

    def gather(_=None):
        dist.all_gather_into_tensor(gathered, y_pad)
        stride.execute_copy(gathered, unpack, out=full)

    gather()
    torch.cuda.synchronize()
    dist.barrier()
    gather_steps = max(2, min(args.steps, 5))
    gather_total, _ = timed_events(stream, gather_steps, gather)
    gather_ms = max_over_ranks(gather_total / gather_steps, device)
    received = (world - 1) * capacity * item

    # End to end through the stride API with host buffers: each rank copies its
    # compacted inputs in from pinned memory and its outputs back, every step.
    e2e_steps = args.e2e_steps or min(args.steps, 8)
    x_host = x.cpu().pin_memory()
    z_host = z.cpu().pin_memory()
    y_back = torch.empty(shard.local_output_size, dtype=tdtype).pin_memory()
    z_back = torch.empty(shard.local_output_size, dtype=tdtype).pin_memory()
    xd, zd, yd = torch.empty_like(x), torch.empty_like(z), torch.empty_like(y)
    torch.cuda.synchronize()
    dist.barrier()

    def e2e(_):
        xd.copy_(x_host, non_blocking=True)
        zd.copy_(z_host, non_blocking=True)
        stride.execute_accumulation(xd, acc, ones, out=yd)
        stride.execute_update(xd, zd, alpha, beta, upd, out=zd)
        y_back.copy_(yd, non_blocking=True)
        z_back.copy_(zd, non_blocking=True)

    e2e_total, _ = timed_events(stream, e2e_steps, e2e)
    e2e_ms = max_over_ranks(e2e_total, device)
    e2e_value = step_bytes * e2e_steps / (e2e_ms / 1e3) / 1e9
    peak, peak_kind = load_peaks()
    if rank == 0:
        achieved = local_update_bytes / (update_ms / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": args.dtype,
            "data": "synthetic N(0,1) from seed (no dataset)",
            "config": {**workload_config(args, n), "parallelism": f"sector-sharded over {world} ranks, LPT by bytes, "
                       "compacted shards, no collective in the timed kernels"},
            "roofline": {"bound": "hbm", "kernel": "MapKernel<update> on rank 0's shard",
                         "achieved": round(achieved, 2), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None,
                         "algorithmic_bytes_per_launch": local_update_bytes,
                         "permute_launch": {"achieved": round(local_permute_bytes / (permute_ms / 1e3) / 1e9, 2),
                                            "frac": round(local_permute_bytes / (permute_ms / 1e3) / 1e9 / peak, 4),
                                            "algorithmic_bytes_per_launch": local_permute_bytes}},
            "shards": {"records_rank0": int(records), "elements_rank0": int(shard.local_output_size),
                       "capacity": int(capacity), "elements_total": int(n)},
            "gather": {"what": "NCCL all_gather_into_tensor of padded compacted outputs + engine copy into the "
                               "packed layout, per rank, max over ranks",
                       "ms": round(gather_ms, 4), "received_bytes_per_rank": int(received),
                       "nvlink_gbs_per_rank": round(received / (gather_ms / 1e3) / 1e9, 2)},
            "cpu_baseline": None,
            "e2e": {"value": round(e2e_value, 3), "unit": UNIT, "steps": e2e_steps,
                    "h2d_bytes_per_step": 2 * n * item, "d2h_bytes_per_step": 2 * n * item,
                    "note": "all ranks together; each rank copies its compacted shard"},
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
            "contraction": None,
        }
        print(json.dumps(line), flush=True)


def permute_plan_of(h):
    from tensor0_b200.tensor_map import permute_plan
    return permute_plan(h, (2, 0), (3, 1))


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist

    from tensor0_b200 import _native, stride
    from tensor0_b200.structure import degeneracy_structure
    from tensor0_b200.tensor_map import TensorMap, add_transform, permute, permute_plan

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)
        try:
            run_sharded(args, world, rank, device)
        finally:
            dist.barrier()
            dist.destroy_process_group()
        return

    h, _ = workload_space(args.scale)
    plan = permute_plan(h, (2, 0), (3, 1))
    n = degeneracy_structure(h).total_dim
    tdtype = torch.float32 if args.dtype == "f32" else torch.complex64
    item = 4 if args.dtype == "f32" else 8
    acc_plan = plan.engine_plan(_native.OP_ACCUMULATION, tdtype)
    upd_plan = plan.engine_plan(_native.OP_UPDATE, tdtype)

    # Synthetic N(0, 1) storage.
    gen = torch.Generator(device=device)
    gen.manual_seed(1000)
    x = torch.randn(n, generator=gen, device=device, dtype=tdtype)
    z = torch.randn(n, generator=gen, device=device, dtype=tdtype)
    y = torch.empty_like(x)
    ones = torch.ones(len(plan.transform.src), dtype=torch.float32, device=device)
    alpha = torch.ones(1, dtype=torch.float32, device=device)
    beta = torch.ones(1, dtype=torch.float32, device=device)

    def step():
        stride.execute_accumulation(x, acc_plan, ones, out=y)
        stride.execute_update(x, z, alpha, beta, upd_plan, out=z)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream(device)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps + 1)]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    launches0 = stride.kernel_launches()
    with ClockSampler(device_uuid(local_rank)) as clocks:
        torch.cuda.synchronize()
        start.record(stream)
        for k in range(args.steps):
            marks[2 * k].record(stream)
            stride.execute_accumulation(x, acc_plan, ones, out=y)
            marks[2 * k + 1].record(stream)
            stride.execute_update(x, z, alpha, beta, upd_plan, out=z)
        marks[2 * args.steps].record(stream)
        end.record(stream)
        torch.cuda.synchronize()
    launches = stride.kernel_launches() - launches0
    elapsed = start.elapsed_time(end)
    permute_ms = [marks[2 * k].elapsed_time(marks[2 * k + 1]) for k in range(args.steps)]
    update_ms = [marks[2 * k + 1].elapsed_time(marks[2 * k + 2]) for k in range(args.steps)]
    step_bytes = 5 * n * item
    value = step_bytes * args.steps / (elapsed / 1e3) / 1e9

    peak, peak_kind = load_peaks()
    update_bytes = 3 * n * item
    permute_bytes = 2 * n * item
    achieved = update_bytes / (statistics.mean(update_ms) / 1e3) / 1e9
    permute_achieved = permute_bytes / (statistics.mean(permute_ms) / 1e3) / 1e9

    # End to end through the public API with host buffers: every step copies
    # x and z in from pinned memory and reads y and z back.  Steps alternate
    # between two device buffer sets, and the copies run on their own streams,
    # so step k + 1's host-to-device copies overlap step k's device-to-host
    # reads (PCIe is full duplex); every copy of every step is inside the
    # timed region.
    e2e_steps = args.e2e_steps or min(args.steps, 8)
    x_host = x.cpu().pin_memory()
    z_host = z.cpu().pin_memory()
    y_back = torch.empty_like(x_host).pin_memory()
    z_back = torch.empty_like(z_host).pin_memory()
    xs = [TensorMap(h, torch.empty_like(x)) for _ in range(2)]
    zs = [TensorMap(plan.dst, torch.empty_like(z)) for _ in range(2)]
    permute(xs[0], ((2, 0), (3, 1)))
    h2d = torch.cuda.Stream(device)
    d2h = torch.cuda.Stream(device)
    loaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    drained = [torch.cuda.Event() for _ in range(2)]
    torch.cuda.synchronize()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record(h2d)
    for k in range(e2e_steps):
        i = k % 2
        with torch.cuda.stream(h2d):
            if k >= 2:
                h2d.wait_event(drained[i])
            xs[i].data.copy_(x_host, non_blocking=True)
            zs[i].data.copy_(z_host, non_blocking=True)
            loaded[i].record(h2d)
        stream.wait_event(loaded[i])
        ys = permute(xs[i], ((2, 0), (3, 1)))
        zs[i] = add_transform(zs[i], xs[i], ((2, 0), (3, 1)), 1.0, 1.0, inplace=True)
        computed[i].record(stream)
        with torch.cuda.stream(d2h):
            d2h.wait_event(computed[i])
            ys.data.record_stream(d2h)
            y_back.copy_(ys.data, non_blocking=True)
            z_back.copy_(zs[i].data, non_blocking=True)
            drained[i].record(d2h)
    stream.wait_stream(d2h)
    e_end.record(d2h)
    torch.cuda.synchronize()
    e_elapsed = e_start.elapsed_time(e_end)
    e2e_value = step_bytes * e2e_steps / (e_elapsed / 1e3) / 1e9

    contraction = None
    if not args.no_contraction:
        contraction = contraction_bench(device, max(args.steps, 5), args.warmup)
    trace = None
    if not args.no_trace:
        trace = trace_bench(device, max(args.steps, 5), args.warmup,
                            tuple(int(d) for d in args.trace_degeneracies.split(",")))

    gemm_f32 = gemm_c64 = None
    if not args.no_contraction:
        gemm_f32 = gemm_f32_bench(device, max(args.steps, 5), args.warmup)
        gemm_c64 = gemm_f32_bench(device, max(args.steps, 5), args.warmup, size=2048, dtype="c64")

    grouped = None
    if not args.no_grouped:
        grouped = grouped_bench(device, max(args.steps, 5), args.warmup, args.grouped_extent)

    cpu = None
    if not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        value_cpu, ms_cpu, sample, _ = cpu_reference_steps(args.dtype, 3, 1, threads, SAMPLE_SCALE)
        cpu = {"value": round(value_cpu, 3), "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample}

    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": args.dtype,
        "data": "synthetic N(0,1) from seed (no dataset)", "config": workload_config(args, n),
        "roofline": {"bound": "hbm", "kernel": "MapKernel<update> (beta=1 accumulate launch)",
                     "achieved": round(achieved, 2), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": load_traffic(),
                     "algorithmic_bytes_per_launch": update_bytes,
                     "permute_launch": {"achieved": round(permute_achieved, 2),
                                        "frac": round(permute_achieved / peak, 4),
                                        "algorithmic_bytes_per_launch": permute_bytes}},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_value, 3), "unit": UNIT, "steps": e2e_steps,
                "h2d_bytes_per_step": 2 * n * item, "d2h_bytes_per_step": 2 * n * item},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
        "contraction": contraction,
        "trace": trace,
        "grouped": grouped,
        "gemm_f32": gemm_f32,
        "gemm_c64": gemm_c64,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
