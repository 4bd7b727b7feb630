"""Quantization and MMA specs, mirrored from TriCast so the backend runs standalone.

``ScaleSpec``/``QuantSpec``/``SCHEMES`` follow ``tricast/quant/spec.py:46-405``; ``MMASpec``/
``PRESETS`` follow ``tricast/mma/spec.py:223-330``. The backend itself only reads attributes, so
TriCast's own spec objects are accepted unchanged when it runs as TriCast's GPU backend.
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field, replace

from .formats import BF16, E8M0, FP4_E2M1, FP16, FP32, UE4M3, IntFormat, emax_elem, get_format
from .rounding import Rounding

FOUR_OVER_SIX = (1.0, 1.5)
_GRANULARITY = {"channel": "row", "token": "row", "per_channel": "row", "per_token": "row",
                "per_tensor": "tensor"}
SCALE_METHODS = ("absmax", "pow2_floor", "pow2_ceil", "mse", "percentile")


@dataclass(frozen=True)
class ScaleSpec:
    format: object = FP32
    method: str = "absmax"
    rounding: Rounding = Rounding.RNE
    two_level: bool = False
    percentile: float = 99.99
    mse_grid: int = 20
    search: tuple = ()

    def __post_init__(self) -> None:
        if self.method == "four_over_six":
            object.__setattr__(self, "method", "mse")
            object.__setattr__(self, "search", FOUR_OVER_SIX)
        object.__setattr__(self, "format", get_format(self.format))
        object.__setattr__(self, "rounding", Rounding.parse(self.rounding))
        object.__setattr__(self, "search", tuple(float(r) for r in self.search))
        if self.method not in SCALE_METHODS:
            raise ValueError(f"unknown scale method {self.method!r}")
        if any(r <= 0 for r in self.search) or self.mse_grid < 1:
            raise ValueError("search ratios must be > 0 and mse_grid >= 1")
        if self.format.kind == "pow2" and self.method not in ("pow2_floor", "pow2_ceil"):
            raise ValueError("a power-of-two scale format needs method pow2_floor or pow2_ceil")
        if self.format.kind == "int":
            raise ValueError("integer scale formats are not supported; use a float or e8m0")
        if not 0 < self.percentile <= 100:
            raise ValueError("percentile must be in (0, 100]")


@dataclass(frozen=True)
class QuantSpec:
    format: object
    granularity: str = "tensor"
    group_size: int = 0
    block: tuple = (0, 0)
    scale: ScaleSpec | None = field(default_factory=ScaleSpec)
    zero_point: str = "none"
    rounding: Rounding = Rounding.RNE
    sr_bits: int = 32
    saturate: bool = True
    mma_input: str = "scaled"
    dequant_format: object = BF16
    observer: object = None

    def __post_init__(self) -> None:
        setter = lambda k, v: object.__setattr__(self, k, v)  # noqa: E731 (frozen)
        setter("format", get_format(self.format))
        setter("dequant_format", get_format(self.dequant_format))
        setter("rounding", Rounding.parse(self.rounding))
        setter("granularity", _GRANULARITY.get(self.granularity, self.granularity))
        setter("block", tuple(self.block))
        if not 1 <= self.sr_bits <= 32:
            raise ValueError("sr_bits must be in [1, 32]")
        if self.granularity not in ("tensor", "row", "group", "block"):
            raise ValueError(f"unknown granularity {self.granularity!r}")
        if self.granularity == "group" and self.group_size <= 0:
            raise ValueError("granularity 'group' needs group_size > 0")
        if self.granularity == "block" and min(self.block) <= 0:
            raise ValueError("granularity 'block' needs block=(rows, cols) > 0")
        if self.format.kind == "pow2":
            raise ValueError("e8m0 is a scale format, not an element format")
        if self.zero_point not in ("none", "int", "float"):
            raise ValueError(f"unknown zero_point {self.zero_point!r}")
        if self.zero_point != "none":
            if self.format.kind != "int":
                raise ValueError("zero points need an integer element format")
            if self.mma_input != "dequant":
                raise ValueError("zero points need mma_input='dequant'")
            if self.scale is None or self.scale.two_level:
                raise ValueError("zero points need a single-level scale")
            if self.zero_point == "float" and self.format.signed:
                raise ValueError("float zero points (KIVI/HQQ offset = min) need an unsigned format")
        if self.scale is None and self.granularity != "tensor":
            raise ValueError("a direct cast (scale=None) has no granularity")
        if self.dequant_format.kind != "float":
            raise ValueError("dequant_format must be a float format")

    @property
    def emax_elem(self) -> int:
        return emax_elem(self.format)

    def with_(self, **changes) -> "QuantSpec":
        return replace(self, **changes)


def _mx(element) -> QuantSpec:
    return QuantSpec(element, "group", group_size=32, scale=ScaleSpec(E8M0, "pow2_floor"))


def bfp(mbits: int, block: int) -> QuantSpec:
    """Block floating point: shared E8M0 exponent per ``block`` and sign-magnitude mantissas."""
    return QuantSpec(IntFormat(f"bfp_m{mbits}", mbits, frac_bits=mbits - 2), "group", group_size=block,
                     scale=ScaleSpec(E8M0, "pow2_floor"))


SCHEMES = {
    "mxfp8_e4m3": _mx("fp8_e4m3"), "mxfp8_e5m2": _mx("fp8_e5m2"),
    "mxfp6_e3m2": _mx("fp6_e3m2"), "mxfp6_e2m3": _mx("fp6_e2m3"),
    "mxfp4": _mx("fp4_e2m1"), "mxint8": _mx("mxint8"), "mxint4": _mx("mxint4"),
    "nvfp4": QuantSpec(FP4_E2M1, "group", group_size=16, scale=ScaleSpec(UE4M3, "absmax", two_level=True)),
    "nvfp4_4o6": QuantSpec(FP4_E2M1, "group", group_size=16,
                           scale=ScaleSpec(UE4M3, "mse", two_level=True, search=FOUR_OVER_SIX)),
    "msfp12": bfp(4, 16), "msfp16": bfp(8, 16),
    "fp8_tensor": QuantSpec("fp8_e4m3", "tensor"),
    "fp8_row": QuantSpec("fp8_e4m3", "row"),
    "fp8_group128": QuantSpec("fp8_e4m3", "group", group_size=128),
    "fp8_block128": QuantSpec("fp8_e4m3", "block", block=(128, 128)),
    "int8_tensor": QuantSpec("int8", "tensor"),
    "int8_row": QuantSpec("int8", "row"),
    "int4_g128": QuantSpec("int4", "group", group_size=128, scale=ScaleSpec(FP16), mma_input="dequant"),
    "int4_g128_zp": QuantSpec("uint4", "group", group_size=128, scale=ScaleSpec(FP16), zero_point="int",
                              mma_input="dequant"),
    "kivi2": QuantSpec("uint2", "group", group_size=32, scale=ScaleSpec(FP16), zero_point="float",
                       mma_input="dequant", dequant_format=FP16),
    "kivi4": QuantSpec("uint4", "group", group_size=32, scale=ScaleSpec(FP16), zero_point="float",
                       mma_input="dequant", dequant_format=FP16),
    "bf16": QuantSpec(BF16, scale=None), "fp16": QuantSpec(FP16, scale=None),
    "fp32": QuantSpec(FP32, scale=None), "tf32": QuantSpec("tf32", scale=None),
}

_BFP = re.compile(r"^bfp(\d+)_b(\d+)$")


def get_scheme(name):
    if not isinstance(name, str):
        return name
    key = name.strip().lower()
    if key in SCHEMES:
        return SCHEMES[key]
    m = _BFP.match(key)
    if m:
        return bfp(int(m.group(1)), int(m.group(2)))
    raise ValueError(f"unknown scheme {name!r}; known: {sorted(SCHEMES)} or bfp<m>_b<block>")


MAX_F_BITS = 48
ALGORITHMS = ("cofda", "gdfs", "fp32_fma", "fp64", "int_exact")
SCALE_APPLY = ("auto", "epilogue", "product", "group", "promote", "operand")


@dataclass(frozen=True)
class MMASpec:
    algorithm: str = "cofda"
    f_bits: int = 23
    chunk_size: int = 32
    c_mode: str = "fused"
    f2_bits: int = 23
    g_bits: int = 32
    group_size: int = 16
    k_tile: int = 64
    norm_rounding: str = "rtz"
    scale_apply: str = "auto"
    promote_interval: int = 0
    out_format: object = BF16
    name: str = ""

    def __post_init__(self) -> None:
        object.__setattr__(self, "out_format", get_format(self.out_format))
        if self.algorithm not in ALGORITHMS:
            raise ValueError(f"unknown algorithm {self.algorithm!r}")
        if self.scale_apply not in SCALE_APPLY:
            raise ValueError(f"unknown scale_apply {self.scale_apply!r}")
        if self.promote_interval < 0 or (self.promote_interval and self.algorithm != "cofda"):
            raise ValueError("promote_interval (> 0) is a cofda option")
        if self.promote_interval and self.promote_interval % self.chunk_size:
            raise ValueError("promote_interval must be a multiple of chunk_size")
        if self.out_format.kind != "float":
            raise ValueError("out_format must be a float format")
        if self.algorithm in ("cofda", "gdfs"):
            if not 1 <= self.f_bits <= MAX_F_BITS:
                raise ValueError(f"f_bits must be in [1, {MAX_F_BITS}]")
            if self.norm_rounding not in ("rtz", "rne"):
                raise ValueError("norm_rounding must be 'rtz' or 'rne'")
        if self.algorithm == "cofda":
            if self.chunk_size < 1:
                raise ValueError("chunk_size must be >= 1")
            if self.c_mode not in ("fused", "decoupled"):
                raise ValueError("c_mode must be 'fused' or 'decoupled'")
            if self.c_mode == "decoupled" and not 1 <= self.f2_bits <= MAX_F_BITS:
                raise ValueError(f"f2_bits must be in [1, {MAX_F_BITS}]")
        if self.algorithm == "gdfs":
            if not 1 <= self.g_bits <= MAX_F_BITS:
                raise ValueError(f"g_bits must be in [1, {MAX_F_BITS}]")
            if self.group_size < 1 or self.k_tile % self.group_size:
                raise ValueError("k_tile must be a positive multiple of group_size")
            if not 1 <= self.k_tile // self.group_size <= 8:
                raise ValueError("k_tile / group_size (groups per tile) must be in [1, 8]")

    @property
    def groups_per_tile(self) -> int:
        return self.k_tile // self.group_size

    def with_(self, **changes) -> "MMASpec":
        return replace(self, name="", **changes)


PRESETS = {
    "nvidia_ada_fp8": MMASpec("cofda", f_bits=13, chunk_size=16, name="nvidia_ada_fp8"),
    "nvidia_hopper_fp8": MMASpec("cofda", f_bits=13, chunk_size=32, name="nvidia_hopper_fp8"),
    "nvidia_blackwell_fp8": MMASpec("cofda", f_bits=25, chunk_size=32, name="nvidia_blackwell_fp8"),
    "nvidia_blackwell_fp4": MMASpec("gdfs", f_bits=35, g_bits=6, group_size=16, k_tile=64,
                                    name="nvidia_blackwell_fp4"),
    "deepseek_fp8_promote128": MMASpec("cofda", f_bits=13, chunk_size=32, promote_interval=128,
                                       name="deepseek_fp8_promote128"),
    "fp32_fma": MMASpec("fp32_fma", name="fp32_fma"),
    "fp64": MMASpec("fp64", name="fp64"),
    "int_exact": MMASpec("int_exact", name="int_exact"),
}


def get_preset(name):
    if not isinstance(name, str):
        return name
    try:
        return PRESETS[name.strip().lower()]
    except KeyError:
        raise ValueError(f"unknown MMA preset {name!r}; known: {sorted(PRESETS)}") from None


def mma_spec_from(spec):
    """An MMASpec from a spec object, a preset name or ``{"preset": name, **overrides}``."""
    if isinstance(spec, dict):
        d = dict(spec)
        if "preset" in d:
            base = get_preset(d.pop("preset"))
            return base.with_(**d) if d else base
        return MMASpec(**d)
    return get_preset(spec)
