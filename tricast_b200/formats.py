"""Number-format descriptors for the B200 backend.

These mirror TriCast's format vocabulary (``tricast/formats.py``) so that the backend can be
driven on a machine where TriCast itself is not installed. Every attribute the kernels read is
named as in TriCast (``ebits``, ``mbits``, ``bias``, ``special``, ``signed``, ``subnormals`` for
floats; ``bits``, ``signed``, ``symmetric``, ``frac_bits`` for integers; ``ebits``/``bias`` for
powers of two), so TriCast's own format objects are accepted by duck typing as well.

Grid rules (reference ``src/tricast/formats.py:29-201``):

* float ``e<E>m<M>``: emin = 1 - bias, emax = top exponent field - bias (one field fewer for
  ``ieee``), max_normal loses the all-ones fraction for ``fn``;
* int: ``value = k * 2**-frac_bits`` with k in [qmin, qmax] (symmetric signed by default);
* pow2 (E8M0): ``2**(field - bias)``, exponents ``[-bias, 2**ebits - 2 - bias]``.
"""

from __future__ import annotations

import math
import re
from dataclasses import dataclass, field

SPECIALS = ("ieee", "fn", "fnuz", "none")


@dataclass(frozen=True)
class FloatFormat:
    name: str
    ebits: int
    mbits: int
    bias: int = field(default=-1)
    special: str = "ieee"
    signed: bool = True
    subnormals: bool = True

    kind = "float"

    def __post_init__(self) -> None:
        if not 1 <= self.ebits <= 8:
            raise ValueError(f"{self.name}: ebits must be in [1, 8], got {self.ebits}")
        if not 0 <= self.mbits <= 23:
            raise ValueError(f"{self.name}: mbits must be in [0, 23], got {self.mbits}")
        if self.special not in SPECIALS:
            raise ValueError(f"{self.name}: special must be one of {SPECIALS}")
        if self.special == "fn" and self.mbits == 0:
            raise ValueError(f"{self.name}: 'fn' needs mbits >= 1 (use Pow2Format for ExM0)")
        if self.bias == -1:
            object.__setattr__(self, "bias", (1 << (self.ebits - 1)) - 1)
        if self.emin < -126 or self.emax > 127:
            raise ValueError(f"{self.name}: exponent range [{self.emin}, {self.emax}] exceeds fp32")

    @property
    def bits(self) -> int:
        return self.ebits + self.mbits + int(self.signed)

    @property
    def precision(self) -> int:
        return self.mbits + 1

    @property
    def emin(self) -> int:
        return 1 - self.bias

    @property
    def emax(self) -> int:
        top_field = (1 << self.ebits) - 1 - (1 if self.special == "ieee" else 0)
        return top_field - self.bias

    @property
    def max_normal(self) -> float:
        kept = self.mbits - 1 if self.special == "fn" else self.mbits
        return (2.0 - 2.0 ** -kept) * 2.0 ** self.emax

    @property
    def min_normal(self) -> float:
        return 2.0 ** self.emin

    @property
    def min_subnormal(self) -> float:
        return 2.0 ** (self.emin - self.mbits) if self.subnormals else self.min_normal

    @property
    def has_inf(self) -> bool:
        return self.special == "ieee"

    @property
    def has_nan(self) -> bool:
        return self.special != "none"

    def __str__(self) -> str:
        return self.name


@dataclass(frozen=True)
class IntFormat:
    name: str
    bits: int
    signed: bool = True
    symmetric: bool = True
    frac_bits: int = 0

    kind = "int"
    has_inf = False
    has_nan = False

    def __post_init__(self) -> None:
        if not 1 <= self.bits <= 24:
            raise ValueError(f"{self.name}: bits must be in [1, 24], got {self.bits}")
        if self.signed and self.bits < 2:
            raise ValueError(f"{self.name}: signed ints need bits >= 2")

    @property
    def qmin(self) -> int:
        if not self.signed:
            return 0
        return -(1 << (self.bits - 1)) + (1 if self.symmetric else 0)

    @property
    def qmax(self) -> int:
        return (1 << (self.bits - 1)) - 1 if self.signed else (1 << self.bits) - 1

    @property
    def max_normal(self) -> float:
        return self.qmax * 2.0 ** -self.frac_bits

    @property
    def min_normal(self) -> float:
        return 2.0 ** -self.frac_bits

    @property
    def magnitude_bits(self) -> int:
        return self.bits - 1 if self.signed else self.bits

    def __str__(self) -> str:
        return self.name


@dataclass(frozen=True)
class Pow2Format:
    name: str = "e8m0"
    ebits: int = 8
    bias: int = 127

    kind = "pow2"
    has_inf = False
    has_nan = True
    signed = False

    @property
    def emin(self) -> int:
        return -self.bias

    @property
    def emax(self) -> int:
        return (1 << self.ebits) - 2 - self.bias

    @property
    def max_normal(self) -> float:
        return 2.0 ** self.emax

    @property
    def min_normal(self) -> float:
        return 2.0 ** self.emin

    def __str__(self) -> str:
        return self.name


FP32 = FloatFormat("fp32", 8, 23)
TF32 = FloatFormat("tf32", 8, 10)
BF16 = FloatFormat("bf16", 8, 7)
FP16 = FloatFormat("fp16", 5, 10)
FP8_E4M3 = FloatFormat("fp8_e4m3", 4, 3, special="fn")
FP8_E5M2 = FloatFormat("fp8_e5m2", 5, 2)
FP8_E4M3FNUZ = FloatFormat("fp8_e4m3fnuz", 4, 3, bias=8, special="fnuz")
FP8_E5M2FNUZ = FloatFormat("fp8_e5m2fnuz", 5, 2, bias=16, special="fnuz")
FP6_E3M2 = FloatFormat("fp6_e3m2", 3, 2, special="none")
FP6_E2M3 = FloatFormat("fp6_e2m3", 2, 3, special="none")
FP4_E2M1 = FloatFormat("fp4_e2m1", 2, 1, special="none")
UE4M3 = FloatFormat("ue4m3", 4, 3, special="fn", signed=False)
E8M0 = Pow2Format("e8m0")
INT8 = IntFormat("int8", 8)
INT4 = IntFormat("int4", 4)
INT2 = IntFormat("int2", 2)
UINT8 = IntFormat("uint8", 8, signed=False)
UINT4 = IntFormat("uint4", 4, signed=False)
MXINT8 = IntFormat("mxint8", 8, frac_bits=6)
MXINT4 = IntFormat("mxint4", 4, frac_bits=2)

REGISTRY = {f.name: f for f in (
    FP32, TF32, BF16, FP16, FP8_E4M3, FP8_E5M2, FP8_E4M3FNUZ, FP8_E5M2FNUZ, FP6_E3M2, FP6_E2M3,
    FP4_E2M1, UE4M3, E8M0, INT8, INT4, INT2, UINT8, UINT4, MXINT8, MXINT4)}

ALIASES = {
    "float32": "fp32", "float": "fp32", "bfloat16": "bf16", "float16": "fp16", "half": "fp16",
    "e4m3": "fp8_e4m3", "e4m3fn": "fp8_e4m3", "fp8": "fp8_e4m3", "e5m2": "fp8_e5m2",
    "e4m3fnuz": "fp8_e4m3fnuz", "e5m2fnuz": "fp8_e5m2fnuz", "e3m2": "fp6_e3m2", "e2m3": "fp6_e2m3",
    "e2m1": "fp4_e2m1", "fp4": "fp4_e2m1", "ue8m0": "e8m0",
}

_FLOAT_NAME = re.compile(r"^(u)?e(\d+)m(\d+)$")
_INT_NAME = re.compile(r"^(u)?int(\d+)$")


def get_format(spec):
    """Resolve a name (TriCast's grammar, ``formats.py:252-300``), a dict or a format object.

    Format objects from TriCast itself are returned unchanged: the backend only reads their
    attributes.
    """
    if hasattr(spec, "kind") and getattr(spec, "kind") in ("float", "int", "pow2") and not isinstance(spec, (str, dict)):
        return spec
    if isinstance(spec, dict):
        d = dict(spec)
        kind = d.pop("kind", "float")
        cls = {"float": FloatFormat, "int": IntFormat, "pow2": Pow2Format}.get(kind)
        if cls is None:
            raise ValueError(f"unknown format kind {kind!r}")
        return cls(**d)
    if not isinstance(spec, str):
        raise TypeError(f"cannot interpret {spec!r} as a format")
    raw, *opts = [part.strip() for part in spec.strip().lower().split(":")]
    head = ALIASES.get(raw, raw)
    if head in REGISTRY and not opts:
        return REGISTRY[head]
    keyed = dict(o.split("=", 1) for o in opts if "=" in o)
    flags = {o for o in opts if "=" not in o}
    m = _FLOAT_NAME.match(raw)
    if m:
        _allowed(spec, flags, keyed, {*SPECIALS, "nosub"}, {"bias"})
        chosen = flags & set(SPECIALS)
        if len(chosen) > 1:
            raise ValueError(f"{spec!r}: choose one of {SPECIALS}")
        unsigned, e, mb = m.group(1) is not None, int(m.group(2)), int(m.group(3))
        if e >= 1 and mb == 0 and not chosen:
            return Pow2Format(name=spec, ebits=e, bias=int(keyed.get("bias", (1 << (e - 1)) - 1)))
        special = next(iter(chosen)) if chosen else ("ieee" if e >= 5 else "none")
        return FloatFormat(spec, e, mb, bias=int(keyed["bias"]) if "bias" in keyed else -1,
                           special=special, signed=not unsigned, subnormals="nosub" not in flags)
    m = _INT_NAME.match(raw)
    if m:
        _allowed(spec, flags, keyed, {"full"}, {"frac"})
        return IntFormat(spec, int(m.group(2)), signed=m.group(1) is None, symmetric="full" not in flags,
                         frac_bits=int(keyed.get("frac", 0)))
    if head in REGISTRY:
        raise ValueError(f"options {opts} are not supported on registered format {head!r}")
    raise ValueError(f"unknown format {spec!r}; registered: {sorted(REGISTRY)}")


def _allowed(spec, flags, keyed, ok_flags, ok_keys) -> None:
    bad = sorted(flags - ok_flags) + sorted(set(keyed) - ok_keys)
    if bad:
        raise ValueError(f"{spec!r}: unsupported option(s) {bad}; allowed: "
                         f"{sorted(ok_flags)} and {sorted(k + '=' for k in ok_keys)}")


def format_of_dtype(dtype):
    """The float format whose grid equals a torch floating dtype."""
    import torch

    table = {torch.float32: FP32, torch.bfloat16: BF16, torch.float16: FP16}
    for name, fmt in (("float8_e4m3fn", FP8_E4M3), ("float8_e5m2", FP8_E5M2),
                      ("float8_e4m3fnuz", FP8_E4M3FNUZ), ("float8_e5m2fnuz", FP8_E5M2FNUZ)):
        if hasattr(torch, name):
            table[getattr(torch, name)] = fmt
    if dtype not in table:
        raise ValueError(f"no TriCast format for dtype {dtype}")
    return table[dtype]


def _holds(fmt, grid) -> bool:
    """Every value of ``fmt`` is exact in ``grid`` (bits, top exponent and finest quantum)."""
    finest = grid.emin - grid.mbits
    if fmt.kind == "float":
        return fmt.mbits <= grid.mbits and fmt.emax <= grid.emax and fmt.emin - fmt.mbits >= finest
    if fmt.kind == "int":
        span = max(abs(fmt.qmin), abs(fmt.qmax)).bit_length()
        return span <= grid.mbits + 1 and -fmt.frac_bits >= finest and fmt.max_normal <= grid.max_normal
    return fmt.emin >= finest and fmt.emax <= grid.emax


def container_dtype(fmt):
    """Smallest torch float dtype holding every value of ``fmt`` exactly (bf16, fp16, else fp32)."""
    import torch

    if _holds(fmt, BF16):
        return torch.bfloat16
    if _holds(fmt, FP16):
        return torch.float16
    return torch.float32


def emax_elem(fmt) -> int:
    """``floor(log2(max_normal))`` of an element format (pow2 scale offset)."""
    return math.frexp(fmt.max_normal)[1] - 1
