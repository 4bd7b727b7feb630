"""Per-layer error sweep over a Qwen3-0.6B-shaped model (the synthetic restatement of TriCast's
``analysis.layer_report``, ``src/tricast/analysis.py:274-411``).

28 blocks x 7 Linears = 196 layers (q 1024->2048, k/v 1024->1024, o 2048->1024, gate/up
1024->3072, down 3072->1024). Layer ``l`` has weights ``W_l ~ N(0, 0.02)`` (seed ``1000 + l``) and
2048 tokens of activations ``X_l ~ N(0, 1)`` (seed ``2000 + l``) with ``in/200`` outlier channels
scaled by 30, both bf16, drawn on the device with a seeded Philox generator so every GPU count sees
identical tensors. For each layer the reference output is ``X W^T`` under TriCast's fp64 MMA
(``MMASpec("fp64", out_format="fp32")``, ``analysis.py:325``) and each of four formats is emulated:

* MXFP4     ``quantize(X|W, "mxfp4")`` + ``nvidia_blackwell_fp4`` (recipe ``mxfp4_w_a``)
* NVFP4     ``quantize(X|W, "nvfp4")`` + ``nvidia_blackwell_fp4`` (recipe ``nvfp4_w_a``)
* FP8 E4M3  ``quantize(X|W, "fp8_tensor")`` + ``nvidia_hopper_fp8`` (recipe ``hopper_fp8_w8a8``)
* INT4-g128 ``int8_row`` activations x ``int4_g128_zp`` weights as exact INT32 sums promoted
            every 128 with fp32 scales (CoFDA F=23, CS=32, promote 128; fp32 out)

Recipe presets keep TriCast's default ``out_format=bf16``. Metrics are TriCast's ``_ErrorStats``
(``analysis.py:29-62``): MSE, SQNR (dB), max abs error, relative Frobenius norm and cosine, from
fp64 sums computed on the device.

Layers are sharded across ranks by longest-processing-time on the measured device time of one layer
of each shape (:func:`measure_costs`, which also warms every shape up at full size) or, without
measurements, on their MAC count; the collectives are an NCCL ``all_gather`` of the
``[layers, formats, 6]`` fp64 metric sums and two small ones for the cost table and the per-rank
timing breakdown. With
``out_dir`` each finished layer writes a JSON record and a rerun skips recorded layers.
"""

from __future__ import annotations

import hashlib
import json
import os
import time
from dataclasses import dataclass
from pathlib import Path

import torch

from .formats import FP16, IntFormat
from .metrics import ErrorStats, finish
from .mma import gemm_triton
from .operand import Operand, as_operand
from .quantize import quantize_triton
from .spec import PRESETS, SCHEMES, MMASpec

LINEARS = (("q_proj", 1024, 2048), ("k_proj", 1024, 1024), ("v_proj", 1024, 1024), ("o_proj", 2048, 1024),
           ("gate_proj", 1024, 3072), ("up_proj", 1024, 3072), ("down_proj", 3072, 1024))
FORMATS = ("mxfp4", "nvfp4", "fp8_e4m3", "int4_g128")
METRIC_FIELDS = ("signal", "estimate", "error", "dot", "max_abs", "nonfinite")


@dataclass(frozen=True)
class SweepConfig:
    blocks: int = 28
    tokens: int = 2048
    hidden_scale: int = 1   # divide every layer dimension by this (small configurations for tests)

    def layers(self) -> list[tuple[int, str, int, int]]:
        out = []
        for b in range(self.blocks):
            for name, fin, fout in LINEARS:
                out.append((len(out), f"model.layers.{b}.{name}", fin // self.hidden_scale, fout // self.hidden_scale))
        return out

    def identity(self) -> str:
        return hashlib.sha256(json.dumps([self.blocks, self.tokens, self.hidden_scale, FORMATS]).encode()).hexdigest()[:16]


def make_layer(index: int, fin: int, fout: int, tokens: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """(X [tokens, in] bf16 with in/200 outlier channels x30, W [out, in] bf16), seeded per layer."""
    g = torch.Generator(device=device)
    g.manual_seed(1000 + index)
    w = (torch.randn(fout, fin, generator=g, device=device) * 0.02).bfloat16()
    g.manual_seed(2000 + index)
    x = torch.randn(tokens, fin, generator=g, device=device)
    n_out = max(1, fin // 200)
    idx = torch.randperm(fin, generator=g, device=device)[:n_out]
    x[:, idx] *= 30
    return x.bfloat16(), w


def emulate(x: torch.Tensor, w: torch.Tensor, fmt: str) -> torch.Tensor:
    """One layer's emulated output under one of the four formats."""
    if fmt == "int4_g128":
        qa = quantize_triton(x, SCHEMES["int8_row"])
        qw = quantize_triton(w, SCHEMES["int4_g128_zp"])
        zeros = qw.zero_point.repeat_interleave(128, dim=1)[:, : w.shape[1]]
        b = Operand(qw.values.float() - zeros, IntFormat("int5", 5), qw.scale, FP16, "k", 128)
        spec = MMASpec("cofda", f_bits=23, chunk_size=32, promote_interval=128, out_format="fp32")
        return gemm_triton(as_operand(qa, compact=True), b, spec)
    scheme, preset = {"mxfp4": ("mxfp4", "nvidia_blackwell_fp4"), "nvfp4": ("nvfp4", "nvidia_blackwell_fp4"),
                      "fp8_e4m3": ("fp8_tensor", "nvidia_hopper_fp8")}[fmt]
    qa = quantize_triton(x, SCHEMES[scheme])
    qw = quantize_triton(w, SCHEMES[scheme])
    return gemm_triton(as_operand(qa, compact=True), as_operand(qw, compact=True), PRESETS[preset])


def reference(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return gemm_triton(as_operand(x, compact=True), as_operand(w, compact=True), MMASpec("fp64", out_format="fp32"))


def shard(layers: list, world: int, rank: int, cost: dict | None = None) -> list:
    """Longest-processing-time assignment of layers to ranks (deterministic). A layer's cost is
    ``cost[(in, out)]`` (e.g. measured seconds per layer of that shape) or, without a table, its MAC
    count."""
    def weight(e):
        return cost[(e[2], e[3])] if cost else e[2] * e[3]

    loads = [0.0] * world
    owner = {}
    for entry in sorted(layers, key=lambda e: (-weight(e), e[0])):
        r = min(range(world), key=lambda i: (loads[i], i))
        owner[entry[0]] = r
        loads[r] += weight(entry)
    return [e for e in layers if owner[e[0]] == rank]


def shapes(layers: list) -> list[tuple[int, int, int]]:
    """(first layer index, in, out) of each distinct Linear shape, in layer order."""
    seen = {}
    for index, _, fin, fout in layers:
        seen.setdefault((fin, fout), index)
    return [(index, fin, fout) for (fin, fout), index in seen.items()]


def measure_costs(cfg: SweepConfig, device, repeats: int = 2) -> dict:
    """Device seconds of one layer's full work (make the tensors, fp64 reference, four emulated formats
    and their error sums) for each distinct shape, at the configuration's token count. The first pass
    of each shape is a warm-up (allocations, first launches); the cost is the minimum of ``repeats``
    timed passes. With several ranks the table is averaged over them (one all-reduce), so that every
    rank derives the same LPT assignment from it."""
    import torch.distributed as dist

    table = {}
    for index, fin, fout in shapes(cfg.layers()):
        entry = [(index, "", fin, fout)]
        run_layers(entry, cfg, device)
        best = float("inf")
        for _ in range(repeats):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            run_layers(entry, cfg, device)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1) / 1e3)
        table[(fin, fout)] = best
    if dist.is_initialized() and dist.get_world_size() > 1:
        keys = sorted(table)
        t = torch.tensor([table[k] for k in keys], dtype=torch.float64, device=device)
        dist.all_reduce(t)
        t /= dist.get_world_size()
        table = dict(zip(keys, t.tolist()))
    return table


def layer_sums(x: torch.Tensor, w: torch.Tensor, sums: torch.Tensor) -> None:
    """One layer's work: the fp64 reference output, the four emulated outputs and their error sums,
    added into ``sums`` [formats, 6]."""
    ref = reference(x, w)
    for col, fmt in enumerate(FORMATS):
        stats = ErrorStats(x.device)
        stats.sums = sums[col]
        stats.update(ref, emulate(x, w, fmt))


class LayerGraph:
    """:func:`layer_sums` for one layer shape captured once as a CUDA graph over static input and
    output buffers. A layer then costs the host two input copies, one replay and one copy of the sums,
    instead of the ~15 library calls and ~30 tensor operations of an eager pass (about 3 ms of Python
    per layer, as long as the device work itself)."""

    def __init__(self, fin: int, fout: int, tokens: int, device):
        device = torch.device(device)
        g = torch.Generator(device=device)
        g.manual_seed(fin * 7919 + fout)
        self.x = torch.randn((tokens, fin), generator=g, device=device).bfloat16()
        self.w = (torch.randn((fout, fin), generator=g, device=device) * 0.02).bfloat16()
        self.sums = torch.zeros((len(FORMATS), len(METRIC_FIELDS)), dtype=torch.float64, device=device)
        current = torch.cuda.current_stream(device)
        side = torch.cuda.Stream(device)
        side.wait_stream(current)
        with torch.cuda.stream(side):  # one eager pass first: allocations and first launches
            self._body()
        current.wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._body()

    def _body(self) -> None:
        self.sums.zero_()
        layer_sums(self.x, self.w, self.sums)

    def run(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> None:
        self.x.copy_(x)
        self.w.copy_(w)
        self.graph.replay()
        out.copy_(self.sums)


_GRAPHS: dict = {}


def layer_graph(fin: int, fout: int, tokens: int, device) -> LayerGraph:
    key = (torch.device(device).index, fin, fout, tokens)
    if key not in _GRAPHS:
        _GRAPHS[key] = LayerGraph(fin, fout, tokens, device)
    return _GRAPHS[key]


def release_graphs() -> None:
    """Drop the captured layer graphs (before the process group is destroyed, or to free memory)."""
    _GRAPHS.clear()


def run_layers(entries: list, cfg: SweepConfig, device, out_dir: str | None = None,
               graphs: bool = True) -> torch.Tensor:
    """Metric sums [len(entries), len(FORMATS), 6] (fp64, on the device) for this rank's layers; with
    ``graphs`` each layer replays its shape's captured :class:`LayerGraph`, else runs eagerly."""
    sums = torch.zeros((len(entries), len(FORMATS), len(METRIC_FIELDS)), dtype=torch.float64, device=device)
    for row, (index, name, fin, fout) in enumerate(entries):
        record = None if out_dir is None else Path(out_dir) / f"layer_{index:04d}.json"
        if record is not None and record.exists():
            saved = json.loads(record.read_text())
            if saved.get("identity") == cfg.identity():
                sums[row] = torch.tensor(saved["sums"], dtype=torch.float64, device=device)
                continue
        x, w = make_layer(index, fin, fout, cfg.tokens, device)
        if graphs:
            layer_graph(fin, fout, cfg.tokens, device).run(x, w, sums[row])
        else:
            layer_sums(x, w, sums[row])
        if record is not None:
            record.parent.mkdir(parents=True, exist_ok=True)
            record.write_text(json.dumps({"identity": cfg.identity(), "layer": index, "name": name,
                                          "sums": sums[row].tolist()}))
    return sums


def gather(entries: list, sums: torch.Tensor, n_layers: int, world: int) -> torch.Tensor:
    """All ranks' sums into one [n_layers, formats, 6] tensor (NCCL all_gather when world > 1)."""
    import torch.distributed as dist

    index = torch.tensor([e[0] for e in entries], dtype=torch.float64, device=sums.device)
    local = torch.cat((index[:, None, None].expand(-1, len(FORMATS), 1), sums), dim=2)
    if world == 1:
        parts = [local]
    else:
        count = torch.tensor([local.shape[0]], device=sums.device)
        counts = [torch.zeros_like(count) for _ in range(world)]
        dist.all_gather(counts, count)
        most = int(max(c.item() for c in counts))
        padded = torch.full((most, len(FORMATS), local.shape[2]), -1.0, dtype=torch.float64, device=sums.device)
        padded[: local.shape[0]] = local
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded)
    table = torch.zeros((n_layers, len(FORMATS), len(METRIC_FIELDS)), dtype=torch.float64, device=sums.device)
    for part in parts:
        for row in part:
            if row[0, 0] >= 0:
                table[int(row[0, 0].item())] = row[:, 1:]
    return table


def results(table: torch.Tensor, cfg: SweepConfig) -> list[dict]:
    """TriCast-style per-layer metric records from the gathered sums."""
    out = []
    sizes = {e[0]: cfg.tokens * e[3] for e in cfg.layers()}
    names = {e[0]: e[1] for e in cfg.layers()}
    for index, per_format in enumerate(table.tolist()):
        row = {"layer": index, "name": names[index]}
        for fmt, s in zip(FORMATS, per_format):
            if s[5]:
                row[fmt] = {"error": "non-finite values"}
            else:
                row[fmt] = finish(sizes[index], s[0], s[1], s[2], s[3], s[4])
        out.append(row)
    return out


def run_sweep(cfg: SweepConfig | None = None, *, out_dir: str | None = None, costs: dict | None = None,
              breakdown: dict | None = None, graphs: bool = True) -> tuple[list[dict] | None, float]:
    """Run the sweep on this process's rank (torch.distributed initialised for world > 1).
    Returns (records on rank 0 else None, seconds = max over ranks of the device-timed span from the
    first layer's first kernel to the last one's end). ``costs``: per-shape layer costs for the LPT
    assignment (see :func:`measure_costs`; MAC counts without). ``breakdown``, when given, receives per
    rank: layers, assigned cost, device seconds and host seconds spent enqueueing the work."""
    import torch.distributed as dist

    cfg = cfg or SweepConfig()
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    device = torch.device("cuda", torch.cuda.current_device())
    layers = cfg.layers()
    mine = shard(layers, world, rank, costs)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    start.record()
    sums = run_layers(mine, cfg, device, out_dir, graphs)
    end.record()
    host = time.perf_counter() - t0
    end.synchronize()
    secs = max(start.elapsed_time(end) / 1e3, 0.0)
    assigned = sum(costs[(e[2], e[3])] for e in mine) if costs else float(sum(e[2] * e[3] for e in mine))
    mine_stats = torch.tensor([len(mine), assigned, secs, host], dtype=torch.float64, device=device)
    every = [mine_stats]
    if world > 1:
        every = [torch.empty_like(mine_stats) for _ in range(world)]
        dist.all_gather(every, mine_stats)
    every = torch.stack(every).tolist()
    if breakdown is not None:
        breakdown.update({"layers": [int(r[0]) for r in every], "assigned_cost": [r[1] for r in every],
                          "device_s": [r[2] for r in every], "host_enqueue_s": [r[3] for r in every]})
    table = gather(mine, sums, len(layers), world)
    return (results(table, cfg) if rank == 0 else None), max(r[2] for r in every)


def main() -> None:
    import argparse

    import torch.distributed as dist

    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--blocks", type=int, default=28)
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--out", default=None, help="directory of per-layer records (resume)")
    ap.add_argument("--json", default=None, help="write the per-layer metric table here (rank 0)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    cfg = SweepConfig(args.blocks, args.tokens)
    costs = measure_costs(cfg, torch.device("cuda", local))
    records, secs = run_sweep(cfg, out_dir=args.out, costs=costs)
    if records is not None:
        summary = {"layers": len(records), "formats": list(FORMATS), "seconds": secs, "n_gpus": world}
        if args.json:
            Path(args.json).write_text(json.dumps({"summary": summary, "layers": records}, indent=1))
        print(json.dumps(summary))
    release_graphs()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
