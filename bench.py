"""Benchmark of the TriCast emulation hot path on B200.

Headline workload: the NVFP4 W4A4 emulated GEMM. A = 2048x4096 bf16 ~ N(0,1) with 8 outlier
channels x20, B = 4096x4096 bf16 ~ N(0,0.02) (seeded, synthetic); one step = quantize A and B to NVFP4
(E2M1 elements, UE4M3 scale per 16 along K, fp32 tensor scale) + the Blackwell-FP4 GDFS emulated GEMM
(G=6, F=35, GS=16, KT=64) with fp32 output, bit-exact with TriCast's reference backend.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Multi-GPU (torchrun, one rank per GPU): strong scaling. The one fixed GEMM is split by N-column
slabs: rank r quantizes all of A and its slab of B's rows (the slab's amax joins the others' in one
NCCL all-reduce of a 32-bit word, so the slab quantizes exactly as those rows of the whole B would)
and computes its [2048, 4096/N] output slab. The FP8 CoFDA GEMM (8192^3) is split the same way
(``aux_strong``), and the 196-layer error sweep is split by layer.

``--impl reference`` times TriCast's own CPU implementation of the path, its pure-PyTorch reference
backend (installed under ``baseline/_ref``), on all host cores over a bounded row slab of the same
workload per step; without that install, the numpy restatement under ``oracle/``.
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "bit-exact emulated GEMM GMAC/s + cast GB/s per B200; 1/2/4/8-GPU layer-sweep secs"
M, N, K = 2048, 4096, 4096
WORKLOAD = ("cfg2 NVFP4 W4A4 emulated GEMM 2048x4096x4096: quantize A,B (nvfp4) + Blackwell-FP4 GDFS "
            "(G=6,F=35,GS=16,KT=64) fp32 out")
DATA = "synthetic (seeded N(0,1)/N(0,0.02) bf16, 8 outlier channels x20)"
L2_FLUSH_BYTES = 512 << 20
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) and issue-slot share
# (smsp__issue_active.avg.pct_of_peak_sustained_active / 100) of one gdfs_fp4_tc_kernel<4, 0> launch
# on the cfg2 operands, from an ncu --set full capture of this build's kernel.
GDFS_TRAFFIC_BYTES = 43_782_656 + 4_235_776
GDFS_ISSUE_UTIL = 0.519
CFG1_BYTES_PER_ELEM = 4 + 4 + 0.5 + 1 / 32  # fp32 in, fp32 dequant out, E2M1 nibble, E8M0 byte per 32
REF_SLAB = (64, 1024)  # rows of A x rows of B per CPU sample step (full K)


def tricast_module():
    """TriCast from ``baseline/_ref`` (offline ``pip --target`` install), or None."""
    ref = ROOT / "baseline" / "_ref"
    if ref.is_dir() and str(ref) not in sys.path:
        sys.path.append(str(ref))
    try:
        import tricast

        return tricast
    except ImportError:
        return None


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def measured_peaks() -> dict:
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "sm_max_mhz": 1965.0, "fallback": True}


def _smi_sampler(stop: threading.Event, samples: list, index: int) -> None:
    q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    try:
        proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "200",
                                 "-i", str(index)], stdout=subprocess.PIPE, text=True)
    except OSError:
        return
    try:
        while not stop.is_set():
            line = proc.stdout.readline()
            if not line:
                break
            samples.append([s.strip() for s in line.split(",")])
    finally:
        proc.terminate()
        proc.wait(timeout=5)


def clocks_summary(samples: list) -> dict:
    if not samples:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
    sm = [float(s[1]) for s in samples if s[1].replace(".", "").isdigit()]
    mx = [float(s[2]) for s in samples if s[2].replace(".", "").isdigit()]
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    reasons = sorted({names[i] for s in samples for i in range(4) if len(s) > 5 + i and s[5 + i].lower() == "active"})
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons, "samples": len(samples)}


class Clocks:
    """nvidia-smi sampled every 200 ms while the ``with`` block runs."""

    def __init__(self, index: int):
        self.index, self.samples, self.stop = index, [], threading.Event()

    def __enter__(self):
        self.thread = threading.Thread(target=_smi_sampler, args=(self.stop, self.samples, self.index), daemon=True)
        self.thread.start()
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.stop.set()
        self.thread.join(timeout=5)
        return False

    def summary(self) -> dict:
        return clocks_summary(self.samples)


def event_pair():
    import torch

    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def stats_ms(times: list) -> dict:
    s = sorted(times)
    return {"median": statistics.median(s), "mean": sum(s) / len(s), "p99": s[min(len(s) - 1, int(0.99 * len(s)))],
            "n": len(s)}


# --------------------------------------------------------------------------------------------- cfg1
def measure_cfg1(dev, steps: int, warmup: int, sets: int = 4) -> dict:
    """MXFP4 quantize-dequantize cast of cfg1 with the benchmark's outputs (dequant fp32, packed E2M1
    codes, E8M0 scale bytes) through preallocated plans (``QuantizePlan``), CUDA-event timed per
    launch. Main protocol: ``sets`` copies of the input and of the outputs are used in rotation, back
    to back, so every launch reads an input and writes outputs that were last touched ``sets`` launches
    (over 500 MB of traffic) earlier: nothing of them is left in the 126 MB L2, and each launch pays,
    as in a streaming steady state, for the write-back of the dirty lines the launch before it left.
    A plain device copy of the input (read 4 B + write 4 B per element) under the same protocol is
    reported beside it. For comparison, ``write_flush`` repeats both after filling a 512 MiB buffer
    before each launch (the launch then also pays for writing back the flush's dirty lines)."""
    import torch

    from tricast_b200 import QuantizePlan, workloads
    from tricast_b200.spec import SCHEMES

    x0 = workloads.cfg1_input().to(dev)
    spec = SCHEMES["mxfp4"]
    stream = torch.cuda.current_stream(dev)
    xs = [x0] + [x0.clone() for _ in range(sets - 1)]
    plans = [QuantizePlan(x0.shape, x0.dtype, dev, spec, want_values=False, want_codes=True, want_scale_codes=True,
                          want_dequant=True) for _ in range(sets)]
    ys = [torch.empty_like(x0) for _ in range(sets)]

    def rotating(fn) -> list:
        for i in range(warmup):
            fn(i % sets)
        events = []
        for i in range(steps * sets):
            e0, e1 = event_pair()
            e0.record(stream)
            fn(i % sets)
            e1.record(stream)
            events.append((e0, e1))
        torch.cuda.synchronize(dev)
        return [a.elapsed_time(b) for a, b in events]

    def flushed(fn) -> list:
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        times = []
        for i in range(warmup + steps):
            flush.fill_(1)
            e0, e1 = event_pair()
            e0.record(stream)
            fn(0)
            e1.record(stream)
            e1.synchronize()
            if i >= warmup:
                times.append(e0.elapsed_time(e1))
        del flush
        return times

    cast = lambda i: plans[i].run(xs[i])  # noqa: E731
    copy = lambda i: ys[i].copy_(xs[i])  # noqa: E731
    t = stats_ms(rotating(cast))["mean"]
    tc = stats_ms(rotating(copy))["mean"]
    tf, tcf = stats_ms(flushed(cast))["mean"], stats_ms(flushed(copy))["mean"]
    nbytes = x0.numel() * CFG1_BYTES_PER_ELEM
    gbs = nbytes / (t * 1e-3) / 1e9
    hbm = measured_peaks().get("hbm_gbs", 6650.0)
    return {"workload": "cfg1 MXFP4 quantize-dequantize 4096x4096 fp32 (dequant fp32 + packed E2M1 + E8M0 bytes)",
            "gbs": gbs, "ms": t, "bytes_per_elem": CFG1_BYTES_PER_ELEM, "hbm_frac": gbs / hbm, "hbm_peak_gbs": hbm,
            "protocol": f"{sets} rotating input/output sets back to back ({sets * 136} MB > L2)",
            "copy_same_protocol_gbs": x0.numel() * 8 / (tc * 1e-3) / 1e9, "copy_same_protocol_ms": tc,
            "write_flush": {"gbs": nbytes / (tf * 1e-3) / 1e9, "ms": tf,
                            "copy_gbs": x0.numel() * 8 / (tcf * 1e-3) / 1e9}}


# ------------------------------------------------------------------------------- GEMM steps (sharded)
def gemm_step(name: str, dev, world: int = 1, rank: int = 0, size: int = 0):
    """(step, macs_whole_job, shape) of one config's step on this rank: quantize all of A and this
    rank's N-column slab of B (against the whole B's amax where the scheme needs it), then the emulated
    GEMM of the slab. At world 1 the slab is all of B. ``size`` (cfg3 only) runs a smaller cube."""
    from tricast_b200 import as_operand, gemm_triton, workloads
    from tricast_b200.shard import column_slab, quantize_operands
    from tricast_b200.spec import PRESETS, SCHEMES

    if name == "cfg2":
        a_cpu, b_cpu = workloads.cfg2_inputs()
        scheme_a = scheme_b = SCHEMES["nvfp4"]
        spec = PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32")
    elif name == "cfg3":
        a_cpu, b_cpu = workloads.cfg3_inputs(size)
        scheme_a = scheme_b = SCHEMES["fp8_tensor"]
        spec = PRESETS["nvidia_hopper_fp8"].with_(out_format="fp32")
    else:
        a_cpu, b_cpu = workloads.cfg4_inputs()
        scheme_a, scheme_b = SCHEMES["int8_row"], SCHEMES["int4_g128_zp"]
        spec = workloads.cfg4_spec()
    m, k = a_cpu.shape
    n = b_cpu.shape[0]
    s, e = column_slab(n, world, rank)
    a, b = a_cpu.to(dev), b_cpu[s:e].contiguous().to(dev)

    def operands(xa=a, xb=b):
        qa, qb = quantize_operands(xa, scheme_a, xb, scheme_b)
        if name == "cfg4":
            return workloads.cfg4_operands(qa, qb)
        return as_operand(qa, compact=True), as_operand(qb, compact=True)

    def gemm(opa, opb):
        return gemm_triton(opa, opb, spec)

    def step(xa=a, xb=b):
        return gemm(*operands(xa, xb))

    step.operands, step.gemm = operands, gemm
    return step, m * n * k, (m, n, k), (a_cpu, b_cpu[s:e].contiguous())


class GraphedStep:
    """One rank's step of a config, replayed from CUDA graphs over static device inputs: the same
    public calls as :func:`gemm_step` (quantize A, quantize this rank's slab of B, emulated GEMM),
    captured once, so that a step costs the host a few graph launches instead of the calls' Python
    and ctypes work (which otherwise bounds the short per-rank steps of a split over many GPUs).
    Where B's scheme needs the whole B's amax and there are several ranks, the step is three graphs:
    the slab's amax bits; A's quantization, replayed while the NCCL all-reduce of the bits runs; B's
    quantization against the reduced amax and the GEMM."""

    def __init__(self, name: str, dev, world: int, rank: int, host_inputs):
        import torch
        import torch.distributed as dist

        from tricast_b200 import _native as N
        from tricast_b200 import as_operand, gemm_triton, workloads
        from tricast_b200.quantize import quantize_into
        from tricast_b200.shard import needs_tensor_amax, quantize_shard
        from tricast_b200.spec import PRESETS, SCHEMES

        schemes = {"cfg2": ("nvfp4", "nvfp4"), "cfg3": ("fp8_tensor", "fp8_tensor"),
                   "cfg4": ("int8_row", "int4_g128_zp")}[name]
        sa, sb = SCHEMES[schemes[0]], SCHEMES[schemes[1]]
        spec = {"cfg2": lambda: PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32"),
                "cfg3": lambda: PRESETS["nvidia_hopper_fp8"].with_(out_format="fp32"),
                "cfg4": workloads.cfg4_spec}[name]()
        self.inputs = [h.to(dev) for h in host_inputs]
        xa, xb = self.inputs
        self.world, self.dev = world, dev
        self.split = world > 1 and needs_tensor_amax(sb)
        self.bits = torch.zeros((), dtype=torch.int32, device=dev)
        state = {}

        def amax_bits():
            self.bits.zero_()
            x2d = xb.reshape(-1, xb.shape[-1])
            N.check(N.lib().tc_tensor_amax_bits(N.ptr(x2d), N.dtype_code(x2d.dtype), x2d.numel(), N.ptr(self.bits),
                                                N.stream_of(dev)), "tc_tensor_amax_bits")

        def quant_a():
            state["qa"] = quantize_into(xa, sa)[0]

        def quant_b_gemm():
            if self.split:
                amax = self.bits.view(torch.float32)
                qb = quantize_into(xb, sb, **({"amax": amax} if sb.granularity == "tensor" else {"tensor_amax": amax}))[0]
            else:
                qb = quantize_shard(xb, sb)
            qa = state["qa"]
            ops = workloads.cfg4_operands(qa, qb) if name == "cfg4" else (as_operand(qa, compact=True),
                                                                          as_operand(qb, compact=True))
            state["out"] = gemm_triton(*ops, spec)

        def whole():
            quant_a()
            quant_b_gemm()

        def eager():
            if self.split:
                amax_bits()
                dist.all_reduce(self.bits, op=dist.ReduceOp.MAX)
                whole()
            else:
                whole()

        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            eager()
            n0 = N.lib().tc_launch_count()
            eager()
            self.launches_per_step = N.lib().tc_launch_count() - n0  # the library kernels of one step
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        parts = [amax_bits, quant_a, quant_b_gemm] if self.split else [whole]
        self.graphs = []
        for part in parts:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                part()
            self.graphs.append(graph)
        self.out = state["out"]

    def __call__(self):
        import torch.distributed as dist

        if not self.split:
            self.graphs[0].replay()
            return self.out
        self.graphs[0].replay()
        work = dist.all_reduce(self.bits, op=dist.ReduceOp.MAX, async_op=True)
        self.graphs[1].replay()  # A's quantization runs while the all-reduce is in flight
        work.wait()
        self.graphs[2].replay()
        return self.out

    def release(self) -> None:
        self.graphs = []


def time_steps(step, dev, steps: int, warmup: int, world: int = 1) -> list:
    """Device time of each of ``steps`` calls (after ``warmup``), a 512 MiB L2 flush before each one
    outside its events, all enqueued back to back; barrier + synchronize on both sides."""
    import torch
    import torch.distributed as dist

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(warmup):
        step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    events = []
    for _ in range(steps):
        flush.fill_(1)
        e0, e1 = event_pair()
        e0.record(stream)
        step()
        e1.record(stream)
        events.append((e0, e1))
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    return [a.elapsed_time(b) for a, b in events]


def time_gemm_graphed(step, dev, steps: int, flush=None) -> list:
    """Device time of the GEMM call alone, on operands quantized beforehand: B's encoding is made by a
    first call and kept on its operand (as a weight's is), then the call (A's encoders, the GEMM
    kernel and the exact kernel queued behind it) is captured in a CUDA graph and each of ``steps``
    replays is timed with its own events, an L2 flush before each outside them."""
    import torch

    stream = torch.cuda.current_stream(dev)
    if flush is None:
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    ops = step.operands()
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        step.gemm(*ops)
        step.gemm(*ops)
    stream.wait_stream(side)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step.gemm(*ops)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(dev)
    events = []
    for _ in range(steps):
        flush.fill_(1)
        e0, e1 = event_pair()
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        events.append((e0, e1))
    torch.cuda.synchronize(dev)
    del graph, ops
    return [a.elapsed_time(b) for a, b in events]


def max_over_ranks(values: list, dev, world: int) -> list:
    import torch
    import torch.distributed as dist

    t = torch.tensor(values, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def measure_gemm_config(dev, name: str, steps: int, warmup: int, world: int = 1, rank: int = 0,
                        size: int = 0) -> dict:
    """Device-timed step of cfg3 (FP8 E4M3 W8A8, Hopper CoFDA F=13 CS=32, 8192^3) or cfg4 (INT8 per
    token x INT4 g128 asymmetric, CoFDA F=23 promoted every 128, 4096x12288x4096), split by N-column
    slabs over the ranks (whole job, max over ranks)."""
    step, macs, shape, _ = gemm_step(name, dev, world, rank, size)
    t = statistics.mean(time_steps(step, dev, steps, warmup, world))
    (t,) = max_over_ranks([t], dev, world)
    return {"workload": name, "shape": list(shape), "n_gpus": world, "gmacs": macs / (t * 1e-3) / 1e9, "ms": t,
            "split": "N-column slabs" if world > 1 else "none"}


def measure_decode(dev, calls: int = 200) -> list:
    """Decode-shaped steps (one token: A is 1 x 4096, B a pre-quantized 4096 x 4096 weight): quantize
    the activation + emulated GEMM, through the public API. ``call_us``: wall time per step over
    back-to-back calls (host work included, one synchronisation at the end); ``gpu_us``: device time
    of one step replayed from a CUDA graph, L2 flushed before each replay."""
    import torch

    from tricast_b200 import as_operand, gemm_triton, quantize_triton
    from tricast_b200.spec import PRESETS, SCHEMES

    g = torch.Generator().manual_seed(7)
    w = (torch.randn(4096, 4096, generator=g) * 0.02).bfloat16().to(dev)
    x = torch.randn(1, 4096, generator=g).bfloat16().to(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    out = []
    for scheme, preset in (("nvfp4", "nvidia_blackwell_fp4"), ("fp8_tensor", "nvidia_hopper_fp8")):
        b = as_operand(quantize_triton(w, SCHEMES[scheme]), compact=True)
        spec = PRESETS[preset].with_(out_format="fp32")

        def step():
            return gemm_triton(as_operand(quantize_triton(x, SCHEMES[scheme]), compact=True), b, spec)

        for _ in range(3):
            step()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for _ in range(calls):
            step()
        torch.cuda.synchronize(dev)
        call_us = (time.perf_counter() - t0) / calls * 1e6
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        times = []
        for _ in range(20):
            flush.fill_(1)
            e0, e1 = event_pair()
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1) * 1e3)
        del graph
        out.append({"workload": f"decode M=1 {scheme} x {preset} 1x4096x4096 (quantize activation + GEMM)",
                    "call_us": call_us, "gpu_us": statistics.median(times)})
    return out


# ------------------------------------------------------------------ TriCast's own GPU backend (Triton)
def measure_tricast_triton(dev, ours_cfg2=None) -> dict:
    """TriCast's unmodified Triton backend (``backend="triton"``: ``kernels/quantize.py:192-275``,
    ``kernels/mma.py:821-886``) on this GPU, through its public API, timed with its own protocol
    (``scripts/bench/bench_mma_vs_nadpe.py:47-69``: 3 warm-ups, 5 CUDA-event timed calls; median, mean,
    p99), plus a 512 MiB L2 flush before each timed call as in this benchmark. The first call of each
    config (Triton JIT) is outside the timing. cfg2's output is compared bit for bit with this
    library's."""
    import torch

    if tricast_module() is None:
        return {"unavailable": "TriCast is not installed under baseline/_ref"}
    from tricast.mma.api import gemm
    from tricast.quant.api import quantize

    from tricast_b200 import workloads

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def timed(fn, warmup: int = 3, repeat: int = 5) -> list:
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(dev)
        times = []
        for _ in range(repeat):
            flush.fill_(1)
            e0, e1 = event_pair()
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize(dev)
            times.append(e0.elapsed_time(e1))
        return times

    out = {"protocol": "TriCast timed(): 3 warm-ups + 5 CUDA-event timed calls, L2 flushed before each"}
    try:
        x = workloads.cfg1_input().to(dev)
        quantize(x, "mxfp4", backend="triton")
        t = stats_ms(timed(lambda: quantize(x, "mxfp4", backend="triton")))
        out["cfg1_quantize_mxfp4"] = {**t, "gbs_6.125B_per_elem": x.numel() * 6.125 / (t["median"] * 1e-3) / 1e9}
    except Exception as exc:  # a JIT or launch failure is reported, not fatal
        out["cfg1_quantize_mxfp4"] = {"error": repr(exc)[:300]}
    for name, scheme, preset, size in (("cfg2", "nvfp4", "nvidia_blackwell_fp4", 0),
                                       ("cfg3", "fp8_tensor", "nvidia_hopper_fp8", 0)):
        try:
            a_cpu, b_cpu = workloads.cfg2_inputs() if name == "cfg2" else workloads.cfg3_inputs(size)
            a, b = a_cpu.to(dev), b_cpu.to(dev)
            spec = {"preset": preset, "out_format": "fp32"}

            def step():
                qa, qb = quantize(a, scheme, backend="triton"), quantize(b, scheme, backend="triton")
                return gemm(qa, qb, spec, backend="triton")

            first = step()
            rec = {}
            if name == "cfg2" and ours_cfg2 is not None:
                mine = ours_cfg2()
                rec["bits_differ_from_b200"] = int((first.view(torch.int32) != mine.view(torch.int32)).sum())
            del first
            t = stats_ms(timed(step, 1 if name == "cfg3" else 3, 3 if name == "cfg3" else 5))
            macs = a.shape[0] * b.shape[0] * a.shape[1]
            rec.update({**t, "gmacs": macs / (t["median"] * 1e-3) / 1e9, "shape": [a.shape[0], b.shape[0], a.shape[1]]})
            out[f"{name}_step"] = rec
        except Exception as exc:
            out[f"{name}_step"] = {"error": repr(exc)[:300]}
    return out


def measure_reference_rows(dev, only: str | None = None, triton: bool = True, shapes=None) -> dict:
    """TriCast's own MMA benchmark (``scripts/bench/bench_mma_vs_nadpe.py``: FP8 E4M3 operands
    ``randn * 2`` with unit tensor scales, bf16 output; CoFDA F=13 CS=32, decoupled CoFDA F=13 CS=32
    F2=23, GDFS G=32 F=25 GS=16 KT=32; shapes 2048x1024x3072, 2048x3072x1024, 4096^3), each row run by
    this library and by TriCast's Triton backend on this GPU with that script's protocol, outputs
    compared bit for bit. Seeded like the script (torch.manual_seed(42), operands drawn on the GPU).
    ``only`` keeps the rows whose label starts with it; ``triton=False`` skips TriCast's side
    (profiling one kernel)."""
    import torch

    from tricast_b200 import gemm_triton
    from tricast_b200.formats import FP32, get_format
    from tricast_b200.operand import Operand
    from tricast_b200.spec import MMASpec

    tri = tricast_module() if triton else None
    configs = [("hopper CoFDA F=13 CS=32", dict(algorithm="cofda", f_bits=13, chunk_size=32)),
               ("CoFDA C-decoupled F=13 CS=32", dict(algorithm="cofda", f_bits=13, chunk_size=32, c_mode="decoupled",
                                                     f2_bits=23)),
               ("GDFS G=32 F=25 GS=16", dict(algorithm="gdfs", f_bits=25, g_bits=32, group_size=16, k_tile=32))]
    configs = [c for c in configs if only is None or c[0].startswith(only)]
    shapes = shapes or [(2048, 1024, 3072), (2048, 3072, 1024), (4096, 4096, 4096)]

    def timed(fn, warmup=3, repeat=5):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(dev)
        times = []
        for _ in range(repeat):
            e0, e1 = event_pair()
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize(dev)
            times.append(e0.elapsed_time(e1))
        return times

    torch.manual_seed(42)
    rows = []
    fp8 = get_format("fp8_e4m3")
    for m, n, k in shapes:
        a8 = (torch.randn(m, k, device=dev) * 2).to(torch.float8_e4m3fn)
        w8 = (torch.randn(n, k, device=dev) * 2).to(torch.float8_e4m3fn)
        one = torch.ones((), device=dev)
        a_op, w_op = Operand(a8.float(), fp8, one, FP32, "tensor"), Operand(w8.float(), fp8, one, FP32, "tensor")
        for label, kw0 in configs:
            kw = dict(kw0)
            spec = MMASpec(kw.pop("algorithm"), out_format="bf16", **kw)
            kw["algorithm"] = spec.algorithm
            mine = gemm_triton(a_op, w_op, spec)
            t = stats_ms(timed(lambda: gemm_triton(a_op, w_op, spec)))
            row = {"shape": [m, n, k], "config": label, "b200_tmacs": m * n * k / (t["median"] * 1e-3) / 1e12,
                   "b200_ms": t}
            if tri is not None:
                from tricast import BF16 as T_BF16
                from tricast import FP8_E4M3 as T_FP8
                from tricast import FP32 as T_FP32
                from tricast import MMASpec as T_MMASpec
                from tricast.kernels.mma import gemm_triton as t_gemm_triton
                from tricast.mma.operand import Operand as T_Operand

                ta = T_Operand(a8.float(), T_FP8, one, T_FP32, "tensor")
                tw = T_Operand(w8.float(), T_FP8, one, T_FP32, "tensor")
                tkw = {key: v for key, v in kw.items() if key != "algorithm"}
                tspec = T_MMASpec(kw["algorithm"], out_format=T_BF16, **tkw)
                try:
                    theirs = t_gemm_triton(ta, tw, tspec)
                    tt = stats_ms(timed(lambda: t_gemm_triton(ta, tw, tspec)))
                    row.update({"triton_tmacs": m * n * k / (tt["median"] * 1e-3) / 1e12, "triton_ms": tt,
                                "bit_identical": bool(torch.equal(theirs.view(torch.int16), mine.view(torch.int16)))})
                except Exception as exc:  # JIT or launch failure of the reference is reported
                    row["triton_error"] = repr(exc)[:300]
            rows.append(row)
    return {"source": "TriCast scripts/bench/bench_mma_vs_nadpe.py rows (A100 published: CoFDA 0.15, GDFS 0.11 "
                      "TMAC/s)", "rows": rows}


# ------------------------------------------------------------------------------- the CPU reference
class CpuSample:
    """One bounded sample of the cfg2 step on the host cores: a ``rows`` x ``cols`` slab of the output
    with the whole K (rows of A, rows of B), its operands quantized from the slab rows, then the
    emulated GEMM. ``kind`` "reference": TriCast's pure-PyTorch reference backend from ``baseline/_ref``
    (``backend="reference"``, ``src/tricast/reference/{quantize,mma}.py``) with every host thread;
    "port": the numpy restatement under ``oracle/`` on one core, when TriCast is not installed. Every
    output is computed independently (``reference/mma.py:340``), so slab throughput is whole-job
    throughput."""

    def __init__(self, rows: int, cols: int):
        import torch

        from tricast_b200 import workloads

        a, b = workloads.cfg2_inputs()
        self.a, self.b = a[:rows].float(), b[:cols].float()
        self.rows, self.cols = rows, cols
        self.tricast = tricast_module()
        self.kind = "reference" if self.tricast is not None else "port"
        self.threads = os.cpu_count() or 1
        if self.kind == "reference":
            torch.set_num_threads(self.threads)
        else:
            self.threads = 1

    def describe(self) -> str:
        what = "TriCast reference backend (pure PyTorch)" if self.kind == "reference" else "numpy oracle port"
        return (f"{what}: {self.rows}x{self.cols}x{K} slab of cfg2 per step (quantize both slabs nvfp4 + "
                f"Blackwell-FP4 GDFS, fp32 out), {self.threads} threads on {cpu_model()}")

    def run(self) -> int:
        if self.kind == "reference":
            from tricast.mma.api import gemm
            from tricast.quant.api import quantize

            qa = quantize(self.a, "nvfp4", backend="reference")
            qb = quantize(self.b, "nvfp4", backend="reference")
            gemm(qa, qb, {"preset": "nvidia_blackwell_fp4", "out_format": "fp32"}, backend="reference")
        else:
            import numpy as np

            import oracle
            from oracle.quantize import quantize_reference
            from tricast_b200.spec import PRESETS, SCHEMES

            spec = SCHEMES["nvfp4"]
            qa, qb = quantize_reference(self.a.numpy(), spec), quantize_reference(self.b.numpy(), spec)

            class Op:
                def __init__(self, q):
                    self.values, self.fmt, self.scale = q.values, spec.format, q.scale
                    self.scale_fmt, self.scale_kind, self.k_domain = spec.scale.format, "k", 16
                    self.alpha = np.float32(q.global_scale)

            oracle.gemm_reference(Op(qa), Op(qb), PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32"))
        return self.rows * self.cols * K


def cpu_baseline() -> dict:
    sample = CpuSample(*REF_SLAB)
    sample.run()  # warm-up
    t0 = time.perf_counter()
    macs = sample.run()
    dt = time.perf_counter() - t0
    return {"value": macs / dt / 1e9, "unit": "GMAC/s", "cores": sample.threads, "kind": sample.kind,
            "sample": f"{sample.describe()}; {dt:.2f} s"}


def run_reference(args) -> None:
    """The reference arm: TriCast's CPU implementation on the host cores, rank 0 only, each step one
    bounded slab of the cfg2 workload."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    sample = CpuSample(*REF_SLAB)
    for _ in range(args.warmup):
        sample.run()
    times, macs = [], 0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        macs = sample.run()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = macs * args.steps / total / 1e9
    line = {"metric": METRIC, "value": value, "unit": "GMAC/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int64", "data": DATA,
            "config": {"workload": WORKLOAD, "global_batch": M, "sample": sample.describe(), "l2": "n/a (CPU)"},
            "cpu_baseline": {"value": value, "unit": "GMAC/s", "cores": sample.threads, "kind": sample.kind,
                             "sample": sample.describe()},
            "e2e": {"value": value, "unit": "GMAC/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------ end to end
def gpu_local_cpus(dev) -> set | None:
    """The host CPUs local to the GPU's PCI device (sysfs ``local_cpulist``) that this process may
    use, or None where sysfs does not say."""
    import torch

    try:
        p = torch.cuda.get_device_properties(dev)
        bdf = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        text = open(f"/sys/bus/pci/devices/{bdf}/local_cpulist").read().strip()
    except (OSError, AttributeError, ValueError):
        return None
    cpus = set()
    for part in text.split(","):
        if "-" in part:
            lo, hi = part.split("-")
            cpus.update(range(int(lo), int(hi) + 1))
        elif part:
            cpus.add(int(part))
    cpus &= os.sched_getaffinity(0)
    return cpus or None


def copy_bandwidth(host_inputs, out, dev) -> dict:
    """One host -> device copy of the step's inputs and one device -> host copy of its output, each
    timed with events on a side stream (GB/s): the link the end-to-end number rides on."""
    import torch

    side = torch.cuda.Stream(dev)
    dst = [torch.empty_like(h, device=dev) for h in host_inputs]
    back = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    res = {}
    with torch.cuda.stream(side):
        for name, fn, nbytes in (("h2d_gbs", lambda: [d.copy_(h, non_blocking=True) for d, h in zip(dst, host_inputs)],
                                  sum(h.numel() * h.element_size() for h in host_inputs)),
                                 ("d2h_gbs", lambda: back.copy_(out, non_blocking=True),
                                  out.numel() * out.element_size())):
            fn()
            e0, e1 = event_pair()
            e0.record(side)
            fn()
            e1.record(side)
            e1.synchronize()
            res[name] = nbytes / (e0.elapsed_time(e1) * 1e-3) / 1e9
    torch.cuda.synchronize(dev)
    return res


def e2e_pipelined(steppers, host_inputs, dev, steps: int, warmup: int, world: int) -> tuple[float, int, int]:
    """The step end to end from pinned host memory, as a serving loop runs it: every step copies its
    inputs host -> device (a copy stream), runs the step (the compute stream) and copies its result
    device -> host (a third stream). Two steppers (each a :class:`GraphedStep` with its own static
    inputs and output) and two pinned host outputs alternate, so step i + 1's upload and step i - 1's
    download overlap step i's compute; the ordering is by CUDA events only. Returns (ms per step over
    the K timed steps, from the first upload's start to the last download's end; H2D bytes per step;
    D2H bytes per step).

    With several ranks every rank needs all of A but the ranks share the host's memory: each uploads
    only its 1/world row slab of A (and its own slab of B), and one NCCL all-gather over NVLink,
    ordered on the upload stream, assembles A on every rank before the step reads it."""
    import torch
    import torch.distributed as dist

    comp = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    host_out = [torch.empty(st.out.shape, dtype=st.out.dtype, pin_memory=True) for st in steppers]
    in_ready = [torch.cuda.Event(), torch.cuda.Event()]
    in_free = [torch.cuda.Event(), torch.cuda.Event()]
    out_free = [torch.cuda.Event(), torch.cuda.Event()]
    a_host = host_inputs[0]
    split_a = world > 1 and a_host.shape[0] % world == 0
    uploads = list(host_inputs)
    if split_a:
        rows = a_host.shape[0] // world
        rank = dist.get_rank()
        uploads[0] = a_host[rank * rows:(rank + 1) * rows]  # a view of the pinned buffer
        a_parts = [torch.empty(uploads[0].shape, dtype=a_host.dtype, device=dev) for _ in steppers]

    def run(n: int) -> None:
        for i in range(n):
            j = i & 1
            st = steppers[j]
            if i >= 2:
                up.wait_event(in_free[j])    # step i - 2 is done reading these inputs
                comp.wait_event(out_free[j])  # and its result has been downloaded
            with torch.cuda.stream(up):
                if split_a:
                    a_parts[j].copy_(uploads[0], non_blocking=True)
                    st.inputs[1].copy_(uploads[1], non_blocking=True)
                    dist.all_gather_into_tensor(st.inputs[0], a_parts[j])  # the upload stream waits for it
                else:
                    for d, h in zip(st.inputs, uploads):
                        d.copy_(h, non_blocking=True)
                in_ready[j].record(up)
            comp.wait_event(in_ready[j])
            out = st()
            in_free[j].record(comp)
            down.wait_stream(comp)
            with torch.cuda.stream(down):
                host_out[j].copy_(out, non_blocking=True)
                out_free[j].record(down)

    run(warmup)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = event_pair()
    start.record(up)
    run(steps)
    end.record(down)
    end.synchronize()
    torch.cuda.synchronize(dev)
    h2d = sum(h.numel() * h.element_size() for h in uploads)
    return start.elapsed_time(end) / steps, h2d, steppers[0].out.numel() * steppers[0].out.element_size()


# ------------------------------------------------------------------------------------ the headline
def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from tricast_b200.sweep import SweepConfig, measure_costs, run_sweep

    step, macs, _, host_inputs = gemm_step("cfg2", dev, world, rank)
    stream = torch.cuda.current_stream(dev)
    # The step's public calls captured as CUDA graphs (GraphedStep); two more for the end-to-end
    # pipeline's double-buffered inputs.
    graphed = [GraphedStep("cfg2", dev, world, rank, host_inputs) for _ in range(3)]
    gstep = graphed[0]

    # The headline: K steps enqueued back to back (no host wait per step), each with its own events,
    # a 512 MiB L2 flush between steps outside them; max over ranks.
    for _ in range(args.warmup):
        gstep()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    with Clocks(local) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        step_events = []
        for _ in range(args.steps):
            flush.fill_(1)
            s0, s1 = event_pair()
            s0.record(stream)
            gstep()
            s1.record(stream)
            step_events.append((s0, s1))
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        launches = gstep.launches_per_step * args.steps  # graph replays launch the captured kernels
        # The GEMM call alone (A's encoders and the GDFS kernel; B's encoding kept on its operand),
        # graph-replayed so that the host's work per call does not show between the events.
        gemm_ms = time_gemm_graphed(step, dev, args.steps, flush)
        # End to end through the public API from pinned host memory. The host buffers are pinned by a
        # thread held to the GPU's local CPUs (their pages land on its NUMA node), as a serving
        # process bound to its GPU would hold them; the process's affinity is restored afterwards.
        affinity = os.sched_getaffinity(0)
        local_cpus = gpu_local_cpus(dev)
        if local_cpus:
            os.sched_setaffinity(0, local_cpus)
        try:
            pinned = [h.pin_memory() for h in host_inputs]
            links = copy_bandwidth(pinned, graphed[1].out, dev)
            t_e2e, h2d, d2h = e2e_pipelined(graphed[1:], pinned, dev, args.steps, args.warmup, world)
        finally:
            os.sched_setaffinity(0, affinity)
        links["host_cpus"] = "gpu-local NUMA node" if local_cpus else "process default (no sysfs locality)"
        # Layer sweep (cfg5): per-shape costs measured at full size (which also warms every shape
        # up), LPT on them, then the device-timed sweep, max over ranks.
        cfg = SweepConfig()
        costs = measure_costs(cfg, dev)
        breakdown = {}
        _, sweep_secs = run_sweep(cfg, costs=costs, breakdown=breakdown)
        # The FP8 CoFDA GEMM (cfg3, 8192^3) split the same way as the headline.
        strong = None if (args.quick and world == 1) else measure_gemm_config(dev, "cfg3", 3, 1, world, rank)
    step_ms = [a.elapsed_time(b) for a, b in step_events]

    t_step, t_gemm, t_e2e = max_over_ranks([statistics.mean(step_ms), statistics.mean(gemm_ms), t_e2e], dev, world)
    sizes = torch.tensor([h2d, d2h], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(sizes)
    h2d_all, d2h_all = (int(v) for v in sizes.tolist())
    if rank == 0:
        clk = clocks.summary()
        peaks = measured_peaks()
        sm_mhz = clk["sm_mhz"] or peaks.get("sm_max_mhz", 1965.0)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        # The group dot products are exact integer sums; their bound is the CUDA cores' integer
        # dot-product rate: SMs x 64 DP4A lanes per clock x 4 MAC x SM clock.
        peak_gmacs = sms * 64 * 4 * sm_mhz * 1e6 / 1e9
        rank_macs = macs / world
        achieved = rank_macs / (t_gemm * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": macs / (t_step * 1e-3) / 1e9, "unit": "GMAC/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int64", "data": DATA,
            "config": {"workload": WORKLOAD, "global_batch": M, "seq_len": K,
                       "parallelism": f"N-column slabs x{world} (one fixed GEMM)" if world > 1 else "single GPU",
                       "l2": "flushed between steps (512 MiB write)"},
            "e2e": {"value": macs / (t_e2e * 1e-3) / 1e9, "unit": "GMAC/s", "h2d_bytes_per_step": h2d_all,
                    "d2h_bytes_per_step": d2h_all,
                    "protocol": "K steps pipelined from pinned host memory: upload, compute and download on three "
                                "streams with double-buffered inputs and outputs; timed from the first upload to "
                                "the last download; bytes summed over ranks; with several ranks each uploads "
                                "its 1/N row slab of A and A is all-gathered over NVLink",
                    "links_rank0": {k: (round(v, 1) if isinstance(v, float) else v) for k, v in links.items()}},
            "gpu_launches": int(launches),
            "graphs": "each step replays CUDA graphs of its public calls; gpu_launches = the library kernels "
                      "one step launches (counted on an eager step) x steps",
            "roofline": {"bound": "alu", "achieved": achieved, "peak": peak_gmacs, "unit": "GMAC/s",
                         "frac": achieved / peak_gmacs, "traffic": GDFS_TRAFFIC_BYTES if world == 1 else None,
                         "issue_util": GDFS_ISSUE_UTIL,
                         "note": f"emulated GEMM per rank (operand encoders + GDFS kernel, CUDA events on its stream); "
                                 "the group dot products run on tcgen05 int8 MMAs and the exact int64/fp64 tile "
                                 f"arithmetic on the CUDA cores bounds the kernel; peak = {sms} SMs x 64 DP4A lanes x "
                                 f"4 MAC x {sm_mhz:.0f} MHz (sampled); traffic and issue_util: DRAM bytes and "
                                 "issue-slot share of one GDFS launch on cfg2 from one ncu capture"},
            "gemm_ms": t_gemm,
            "aux_sweep": {"workload": "cfg5 per-layer error sweep: 196 Qwen3-0.6B-shaped layers x "
                                      "(MXFP4, NVFP4, FP8 E4M3, INT4-g128) vs fp64, 2048 tokens",
                          "secs": sweep_secs, "n_gpus": world, "sharding": "LPT on measured per-shape layer time",
                          "per_rank": breakdown, "layer_cost_s": {f"{a}x{b}": v for (a, b), v in costs.items()},
                          "collective": "NCCL all_gather of [layers, 4, 6] fp64 metric sums"},
            "clocks": clk,
        }
        if strong is not None:
            line["aux_strong"] = strong
        if world == 1:
            line["aux_cast"] = measure_cfg1(dev, args.steps, args.warmup)
            line["aux_gemm"] = [measure_gemm_config(dev, "cfg4", max(3, args.steps // 3), 1)]
            line["aux_decode"] = measure_decode(dev)
            if not args.quick:
                line["aux_triton"] = measure_tricast_triton(dev, step)
                line["aux_reference_rows"] = measure_reference_rows(dev)
            if not args.no_cpu_baseline:
                line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    from tricast_b200.sweep import release_graphs

    release_graphs()
    for g in graphed:
        g.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quick", action="store_true", help="skip the slow auxiliary measurements (Triton, cfg3)")
    ap.add_argument("--workload", default="all", choices=["all", "cfg2step", "cfg2gemm", "cfg1", "cfg3", "cfg4", "decode",
                                                      "triton", "rows", "gdfs_row", "sweep"],
                    help="run only that measurement on one GPU (for profiling)")
    ap.add_argument("--cube", type=int, default=0,
                    help="with --workload cfg3: run an M = N = K = CUBE case instead of 8192 (profiling)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.workload != "all":
        import torch

        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        if args.workload == "cfg1":
            print(json.dumps(measure_cfg1(dev, args.steps, args.warmup)))
        elif args.workload == "cfg2gemm":  # the GEMM call alone, graph-replayed
            step, macs, shape, _ = gemm_step("cfg2", dev)
            t = statistics.mean(time_gemm_graphed(step, dev, max(args.steps, 1)))
            print(json.dumps({"workload": "cfg2 GEMM", "shape": list(shape), "ms": t, "gmacs": macs / (t * 1e-3) / 1e9}))
        elif args.workload == "sweep":  # the cfg5 layer sweep on this GPU
            from tricast_b200.sweep import SweepConfig, measure_costs, run_sweep

            cfg = SweepConfig()
            breakdown = {}
            _, secs = run_sweep(cfg, costs=measure_costs(cfg, dev), breakdown=breakdown)
            print(json.dumps({"workload": "cfg5 sweep", "secs": secs, "per_rank": breakdown}))
        elif args.workload == "cfg2step":
            step, macs, shape, _ = gemm_step("cfg2", dev)
            t = statistics.mean(time_steps(step, dev, args.steps, args.warmup))
            print(json.dumps({"workload": "cfg2 step", "shape": list(shape), "ms": t, "gmacs": macs / (t * 1e-3) / 1e9}))
        elif args.workload == "decode":
            print(json.dumps(measure_decode(dev, calls=args.steps)))
        elif args.workload == "triton":
            print(json.dumps(measure_tricast_triton(dev)))
        elif args.workload == "rows":
            print(json.dumps(measure_reference_rows(dev)))
        elif args.workload == "gdfs_row":  # this library's GDFS G=32 row at 4096^3 alone
            print(json.dumps(measure_reference_rows(dev, only="GDFS", triton=False, shapes=[(4096, 4096, 4096)])))
        else:
            print(json.dumps(measure_gemm_config(dev, args.workload, args.steps, args.warmup, size=args.cube)))
        return
    run_b200(args)


if __name__ == "__main__":
    main()
