"""Loaders for the committed golden fixtures (``tests/golden``), shared by CPU and GPU tests."""

from __future__ import annotations

import functools
import json
from pathlib import Path
from types import SimpleNamespace

import numpy as np

from tricast_b200.formats import FP8_E4M3, FP32, FP4_E2M1, E8M0, UE4M3, get_format
from tricast_b200.spec import MMASpec, QuantSpec, ScaleSpec

GOLDEN = Path(__file__).resolve().parent / "golden"


@functools.lru_cache(maxsize=None)
def load(name: str):
    meta = json.loads((GOLDEN / f"{name}.json").read_text())
    arrays = np.load(GOLDEN / f"{name}.npz")
    return meta, {k: arrays[k] for k in arrays.files}


def qspec(d: dict) -> QuantSpec:
    scale = None
    if d["scale"] is not None:
        s = d["scale"]
        scale = ScaleSpec(get_format(s["format"]), s["method"], s["rounding"], s["two_level"], s["percentile"],
                          s["mse_grid"], tuple(s["search"]))
    return QuantSpec(get_format(d["format"]), d["granularity"], d["group_size"], tuple(d["block"]), scale,
                     d["zero_point"], d["rounding"], d["sr_bits"], d["saturate"], d["mma_input"],
                     get_format(d["dequant_format"]))


def mspec(d: dict) -> MMASpec:
    d = dict(d)
    d["out_format"] = get_format(d["out_format"])
    return MMASpec(**d)


def mma_operand(case: dict, arrays: dict, side: str) -> SimpleNamespace:
    o = case[side]
    cid = case["id"]
    return SimpleNamespace(values=arrays[f"{cid}|{side}|values"], fmt=get_format(o["fmt"]),
                           scale=arrays.get(f"{cid}|{side}|scale"),
                           scale_fmt=None if o["scale_fmt"] is None else get_format(o["scale_fmt"]),
                           scale_kind=o["scale_kind"], k_domain=o["k_domain"],
                           alpha=arrays.get(f"{cid}|{side}|alpha"))


def nadpe_cases():
    """(file key, case index, operand a, operand b, spec, expected bf16 bits) for all vectors."""
    meta, arrays = load("nadpe")
    out = []
    for entry in meta:
        key = entry["key"]
        if entry["kind"] == "fp8":
            ops = [SimpleNamespace(values=arrays[f"{key}|{s}"], fmt=FP8_E4M3,
                                   scale=np.float32(entry[f"scale_{t}"]), scale_fmt=FP32, scale_kind="tensor",
                                   k_domain=0, alpha=None) for s, t in (("a", "a"), ("b", "b"))]
            for i, c in enumerate(entry["cases"]):
                spec = MMASpec("gdfs" if c["algorithm"] == 1 else "cofda", f_bits=c["f_bits"], g_bits=c["g_bits"] or 32,
                               group_size=c["group_size"] or 16, chunk_size=c["chunk_size"] or 32, k_tile=32,
                               f2_bits=23, c_mode="decoupled" if c["algorithm"] == 3 else "fused",
                               out_format="bf16")
                out.append((key, i, ops[0], ops[1], spec, arrays[f"{key}|out|{i}"]))
        else:
            sfmt = UE4M3 if entry["scale_format"] == "ue4m3" else E8M0
            ops = []
            for side in ("a", "w"):
                alpha = np.float32(entry["alpha"]) if side == "a" and entry["scale_format"] == "ue4m3" else None
                ops.append(SimpleNamespace(values=arrays[f"{key}|{side}"], fmt=FP4_E2M1,
                                           scale=arrays[f"{key}|{side}_scale"], scale_fmt=sfmt, scale_kind="k",
                                           k_domain=entry["block"], alpha=alpha))
            for i, c in enumerate(entry["cases"]):
                if c["algorithm"] == 1:
                    spec = MMASpec("gdfs", f_bits=c["f_bits"], g_bits=c["g_bits"], group_size=c["group_size"],
                                   k_tile=64, out_format="bf16")
                else:
                    spec = MMASpec("cofda", f_bits=c["f_bits"], chunk_size=c["chunk_size"], out_format="bf16")
                out.append((key, i, ops[0], ops[1], spec, arrays[f"{key}|out|{i}"]))
    return out


def bf16_bits(values_f32: np.ndarray) -> np.ndarray:
    """int16 bit patterns of bf16 values held exactly in fp32."""
    return (np.asarray(values_f32, np.float32).view(np.uint32) >> 16).astype(np.uint16).view(np.int16)
