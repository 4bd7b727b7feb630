"""Oracle emulated MMA: exact-integer CoFDA / GDFS datapaths and IEEE FMA chains
(TEST INFRASTRUCTURE ONLY).

Restates ``src/tricast/reference/mma.py`` with numpy int64 arrays, vectorised over the [M, N]
outputs and looping over K chunks, tiles and groups in the reference's order. Terms are
(negative, exponent, significand, zero, nan, inf) arrays; a significand is an integer at an
explicit radix, so ``value = (-1)**negative * significand * 2**(exponent - radix)``.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np

from .cast import decode, round_to_format

FP32_FMT = SimpleNamespace(kind="float", name="fp32", ebits=8, mbits=23, bias=127, emin=-126, emax=127,
                           special="ieee", signed=True, subnormals=True, max_normal=float(np.finfo(np.float32).max),
                           min_normal=2.0 ** -126, min_subnormal=2.0 ** -149)
FIELDS = ("neg", "exp", "sig", "zero", "nan", "inf")


class Terms:
    __slots__ = FIELDS

    def __init__(self, neg, exp, sig, zero, nan, inf):
        self.neg, self.exp, self.sig, self.zero, self.nan, self.inf = neg, exp, sig, zero, nan, inf

    def take(self, index) -> "Terms":
        return Terms(*(getattr(self, f)[index] for f in FIELDS))


def _np(t):
    if t is None:
        return None
    if hasattr(t, "detach"):
        t = t.detach().cpu().float().numpy()
    return np.asarray(t, np.float32)


def shift(x, amount):
    """Signed shift of a nonnegative integer; shifts of 64 or more give zero (``mma.py:25-33``)."""
    amount = np.asarray(amount, np.int64)
    x = np.asarray(x, np.int64)
    with np.errstate(over="ignore"):
        left = x << np.clip(amount, 0, 63)
    right = x >> np.clip(-amount, 0, 63)
    return np.where(np.abs(amount) >= 64, 0, np.where(amount >= 0, left, right))


def ilog2(x) -> np.ndarray:
    """floor(log2(x)) of nonnegative int64 by bisection; 0 for 0 (``mma.py:36-43``)."""
    x = np.asarray(x, np.int64).copy()
    out = np.zeros_like(x)
    for step in (32, 16, 8, 4, 2, 1):
        high = x >= (1 << step)
        out += high * step
        x = np.where(high, x >> step, x)
    return out


def rounded_shift(x, amount):
    """Shift with round-half-even on the discarded bits (``mma.py:46-52``)."""
    amount = np.asarray(amount, np.int64)
    kept = shift(x, amount)
    discard = np.clip(-amount, 0, 63)
    rem = x - (kept << discard)
    half = np.int64(1) << np.clip(discard - 1, 0, 62)
    up = (rem > half) | ((rem == half) & ((kept & 1) != 0))
    return kept + ((amount < 0) & (amount > -64) & up).astype(np.int64)


def mul_shift(a, b, amount: int):
    """Exact ``(a * b)`` shifted by ``amount``; products wider than int64 go through Python ints
    (``mma.py:55-72``)."""
    a, b = np.asarray(a, np.int64), np.asarray(b, np.int64)
    if amount >= 0:
        return (a * b) << amount
    wide = a.astype(object) * b.astype(object)
    shifted = wide >> (-amount) if -amount < 4096 else wide * 0
    return np.asarray(shifted, dtype=object).astype(np.int64)


def decoded(values, fmt):
    """Decode with specials flagged and decoded as a placeholder (``mma.py:75-82``)."""
    values = np.asarray(values, np.float32)
    finite = np.isfinite(values)
    neg, exp, sig, radix = decode(np.where(finite, values, np.float32(fmt.min_normal)), fmt)
    return Terms(np.signbit(values) | neg, exp, sig, values == 0, np.isnan(values), np.isinf(values)), radix


def fp32_terms(values, radix: int) -> Terms:
    """The running fp32 register as a term, subnormals normalised (``mma.py:85-91``)."""
    t, _ = decoded(values, FP32_FMT)
    lead = ilog2(t.sig)
    t.exp = t.exp + lead - 23
    t.sig = shift(t.sig, radix - lead)
    return t


def combine(a: Terms, b: Terms, sig) -> Terms:
    """Product of two terms' flags and exponents (``mma.py:94-97``)."""
    nan = a.nan | b.nan | (a.inf & b.zero) | (b.inf & a.zero)
    return Terms(a.neg ^ b.neg, a.exp + b.exp, sig, a.zero | b.zero, nan, (a.inf | b.inf) & ~nan)


def sum_terms(t: Terms):
    """Align to the largest active exponent with truncation and sum exactly (``mma.py:104-115``)."""
    active = ~(t.zero | t.nan | t.inf)
    emax = np.where(active, t.exp, -4096).max(axis=-1)
    mag = shift(t.sig, t.exp - emax[..., None])
    total = np.where(active, np.where(t.neg, -mag, mag), 0).sum(axis=-1)
    pos = (t.inf & ~t.neg).any(axis=-1)
    neg = (t.inf & t.neg).any(axis=-1)
    nan = t.nan.any(axis=-1) | (pos & neg)
    special = np.where(nan, np.float32(np.nan), np.where(neg, np.float32(-np.inf), np.float32(np.inf)))
    return total, emax, nan | pos | neg, special


def fixed_to_fp32(total, exponent, radix: int, norm: str, *, fda: bool = True) -> np.ndarray:
    """Normalise an exact fixed-point sum into fp32 bits (``mma.py:118-137``)."""
    total = np.asarray(total, np.int64)
    exponent = np.asarray(exponent, np.int64)
    mag = np.abs(total)
    lead = ilog2(mag)
    biased = lead + exponent - radix + 127
    precision = min(radix, 23) if fda else 23
    amount = precision - lead
    kept = rounded_shift(mag, amount) if norm == "rne" else shift(mag, amount)
    carry = kept >= (np.int64(1) << (precision + 1))
    kept = np.where(carry, kept >> 1, kept)
    nexp = biased + carry
    normal = (nexp << 23) | ((kept << (23 - precision)) & 0x7FFFFF)
    normal = np.where(nexp >= 255, 0x7F800000, normal)
    sub_shift = 149 + exponent - radix
    sub = shift(mag, sub_shift) if fda else rounded_shift(mag, sub_shift)
    bits = np.where(biased <= 0, sub, normal) | ((total < 0).astype(np.int64) << 31)
    bits = np.where(total == 0, 0, bits)
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def fda(terms: Terms, c, radix: int, norm: str) -> np.ndarray:
    """One fused dot-add of ``terms`` (last axis) with the running value ``c`` (``mma.py:140-151``)."""
    c = np.asarray(c, np.float32)
    acc = fp32_terms(c[..., None], radix)
    n = np.broadcast_shapes(*(np.shape(getattr(terms, f)) for f in FIELDS))[-1]
    joined = Terms(*(np.concatenate((np.broadcast_to(getattr(terms, f), c.shape + (n,)), getattr(acc, f)), axis=-1)
                     for f in FIELDS))
    total, emax, exceptional, special = sum_terms(joined)
    result = fixed_to_fp32(total, emax, radix, norm)
    result = np.where(joined.zero.all(axis=-1), c, result)
    return np.where(exceptional, special, result).astype(np.float32)


def fp32_fma(a, b, c) -> np.ndarray:
    """binary32 fused multiply-add from an exact fp64 product, TwoSum residual and a midpoint
    correction of the fp64 -> fp32 double rounding (``mma.py:154-168``)."""
    a, b, c = (np.asarray(v, np.float32) for v in (a, b, c))
    with np.errstate(invalid="ignore", over="ignore"):
        p = a.astype(np.float64) * b.astype(np.float64)
        add = c.astype(np.float64)
        value = p + add
        z = value - p
        residual = (p - (value - z)) + (add - z)
        rounded = value.astype(np.float32)
        nearest = rounded.astype(np.float64)
        toward = np.where(value > nearest, np.float32(np.inf), np.float32(-np.inf))
        neighbour = np.nextafter(rounded, toward).astype(np.float64)
        midpoint = np.abs(value - nearest) == np.abs(neighbour - nearest) * 0.5
        midpoint |= np.abs(value) == 2.0 ** 128 - 2.0 ** 103
        corrected = np.nextafter(value, np.where(residual > 0, np.inf, -np.inf)).astype(np.float32)
    return np.where(midpoint & (residual != 0) & np.isfinite(value), corrected, rounded).astype(np.float32)


def integer_bits(fmt) -> int:
    if fmt.kind == "int":
        return max(abs(fmt.qmin), fmt.qmax).bit_length() + max(0, -fmt.frac_bits)
    return 1


def resolve_scale_apply(spec, a, b) -> str:
    """Where operand scales enter the arithmetic (``mma.py:184-202``)."""
    k_scaled = [op for op in (a, b) if op.scale_kind == "k"]
    expected = {"gdfs": "group", "cofda": "promote" if spec.promote_interval else "product",
                "fp32_fma": "operand", "fp64": "operand", "int_exact": "epilogue"}[spec.algorithm]
    mode = expected if k_scaled else "epilogue"
    if spec.scale_apply != "auto":
        mode = spec.scale_apply
        if mode not in ("epilogue", expected):
            raise ValueError(f"scale_apply={mode!r} is incompatible with {spec.algorithm} "
                             f"and promote_interval={spec.promote_interval}; expected {expected!r}")
    if k_scaled and (mode == "epilogue" or spec.algorithm == "int_exact"):
        raise ValueError(f"{spec.algorithm}: K-varying scales cannot be applied in the epilogue")
    span = spec.group_size if mode == "group" else spec.promote_interval if mode == "promote" else 0
    for op in k_scaled:
        if span and any(s // op.k_domain != (min(s + span, op.values.shape[1]) - 1) // op.k_domain
                        for s in range(0, op.values.shape[1], span)):
            raise ValueError(f"{mode} interval/group size {span} crosses K scale domain {op.k_domain}")
    return mode


def scale_terms(op, start: int, end: int, side: str):
    """Per-product K-scale terms; standard E8M0 2**-127 counts as zero (``mma.py:241-252``)."""
    if op.scale_kind != "k":
        return None
    index = np.arange(start, end) // op.k_domain
    scale = op.scale[:, index]
    fmt = op.scale_fmt or FP32_FMT
    t, radix = decoded(scale, fmt)
    if fmt.kind == "pow2" and fmt.ebits == 8 and fmt.bias == 127:
        t.zero = t.zero | (scale == np.float32(2.0 ** -127))
        t.sig = np.where(t.zero, 0, t.sig)
    return t.take((slice(None), None, slice(None)) if side == "a" else (None, slice(None), slice(None))), radix


def apply_scales(t: Terms, radix: int, target: int, a, b, start: int, end: int, *, group=False) -> Terms:
    """Multiply terms by their K scales and move them to radix ``target`` (``mma.py:255-277``)."""
    factors = [f for f in (scale_terms(a, start, end, "a"), scale_terms(b, start, end, "b")) if f is not None]
    if not factors:
        t.sig = shift(t.sig, target - radix)
        return t
    scale, srad = factors[0]
    if len(factors) == 2:
        other, orad = factors[1]
        scale = combine(scale, other, scale.sig * other.sig)
        srad += orad
    out = combine(t, scale, mul_shift(t.sig, scale.sig, target - radix - srad))
    if group:
        nan, zero = t.nan, t.zero
        for f, _ in factors:
            nan, zero = nan | f.nan, zero | f.zero
        out.nan, out.zero = nan, zero & ~nan
        out.inf = (t.inf | scale.inf) & ~(nan | zero)
    return out


def products(at: Terms, bt: Terms, start: int, end: int) -> Terms:
    ta = at.take((slice(None), None, slice(start, end)))
    tb = bt.take((None, slice(None), slice(start, end)))
    return combine(ta, tb, ta.sig * tb.sig)


def _cofda(a, b, spec, mode, c):
    """Chunked fused dot-add along K, optional decoupled merge and promotion (``mma.py:286-315``)."""
    at, ar = decoded(a.values, a.fmt)
    bt, br = decoded(b.values, b.fmt)
    K = a.values.shape[1]
    interval = spec.promote_interval or max(K, 1)
    acc = c
    for begin in range(0, K, interval):
        partial = np.zeros_like(c) if spec.promote_interval else acc
        for start in range(begin, min(begin + interval, K), spec.chunk_size):
            end = min(start + spec.chunk_size, begin + interval, K)
            terms = products(at, bt, start, end)
            if mode == "product":
                terms = apply_scales(terms, ar + br, spec.f_bits, a, b, start, end)
            else:
                terms.sig = shift(terms.sig, spec.f_bits - ar - br)
            if spec.c_mode == "decoupled" and not spec.promote_interval:
                p = fda(terms, np.zeros_like(c), spec.f_bits, spec.norm_rounding)
                partial = fda(fp32_terms(p[..., None], spec.f2_bits), partial, spec.f2_bits, spec.norm_rounding)
            else:
                partial = fda(terms, partial, spec.f_bits, spec.norm_rounding)
        if spec.promote_interval:
            weight = np.ones_like(c)
            if a.scale_kind == "k":
                weight = (weight * a.scale[:, begin // a.k_domain, None]).astype(np.float32)
            if b.scale_kind == "k":
                weight = (weight * b.scale[None, :, begin // b.k_domain]).astype(np.float32)
            acc = fp32_fma(partial, weight, acc)
        else:
            acc = partial
    return acc


def _gdfs(a, b, spec, c):
    """Group sums at G bits, group-level scales, one F-bit FDA per K tile (``mma.py:318-336``)."""
    at, ar = decoded(a.values, a.fmt)
    bt, br = decoded(b.values, b.fmt)
    K = a.values.shape[1]
    for tile in range(0, K, spec.k_tile):
        groups = []
        for start in range(tile, min(tile + spec.k_tile, K), spec.group_size):
            end = min(start + spec.group_size, K)
            prods = products(at, bt, start, end)
            prods.sig = shift(prods.sig, spec.g_bits - ar - br)
            total, emax, exceptional, special = sum_terms(prods)
            with np.errstate(invalid="ignore"):
                g = Terms(total < 0, emax, np.abs(total), (total == 0) & ~exceptional,
                          np.isnan(special) & exceptional, np.isinf(special) & exceptional)
            g.neg = np.where(g.inf, np.signbit(special), g.neg)
            g = g.take((..., None))
            groups.append(apply_scales(g, spec.g_bits, spec.f_bits, a, b, start, start + 1, group=True))
        joined = Terms(*(np.concatenate([np.broadcast_to(getattr(g, f), c.shape + (1,)) for g in groups], axis=-1)
                         for f in FIELDS))
        c = fda(joined, c, spec.f_bits, spec.norm_rounding)
    return c


def gemm_reference(a, b, spec, bias=None) -> np.ndarray:
    """``a @ b.T`` with the spec's arithmetic, independently per output (``mma.py:339-384``).

    ``a``/``b`` carry values [rows, K] (fp32 grid values), fmt, scale, scale_fmt, scale_kind,
    k_domain and alpha, as numpy arrays or torch tensors. Returns fp32 grid values of
    ``spec.out_format``."""
    a = SimpleNamespace(values=_np(a.values), fmt=a.fmt, scale=_np(a.scale), scale_fmt=a.scale_fmt,
                        scale_kind=a.scale_kind, k_domain=a.k_domain, alpha=_np(a.alpha))
    b = SimpleNamespace(values=_np(b.values), fmt=b.fmt, scale=_np(b.scale), scale_fmt=b.scale_fmt,
                        scale_kind=b.scale_kind, k_domain=b.k_domain, alpha=_np(b.alpha))
    bias = _np(bias)
    if a.values.shape[1] != b.values.shape[1]:
        raise ValueError(f"operand K dimensions differ: {a.values.shape[1]} != {b.values.shape[1]}")
    mode = resolve_scale_apply(spec, a, b)
    M, N, K = a.values.shape[0], b.values.shape[0], a.values.shape[1]
    acc = np.zeros((M, N), np.float32)
    if M and N:
        if spec.algorithm == "cofda":
            acc = _cofda(a, b, spec, mode, acc)
        elif spec.algorithm == "gdfs":
            acc = _gdfs(a, b, spec, acc)
        elif spec.algorithm == "int_exact":
            at, _ = decoded(a.values, a.fmt)
            bt, _ = decoded(b.values, b.fmt)
            if (at.nan | at.inf).any() or (bt.nan | bt.inf).any():
                raise ValueError("int_exact requires finite integer operands")
            total = np.zeros((M, N), np.int64)
            for start in range(0, K, 32):
                t = products(at, bt, start, min(start + 32, K))
                total += np.where(t.neg, -t.sig, t.sig).sum(axis=-1)
            acc = fixed_to_fp32(total, np.full((M, N), -a.fmt.frac_bits - b.fmt.frac_bits), 0, "rne", fda=False)
        else:
            av, bv = a.values, b.values
            if mode == "operand":
                if a.scale_kind == "k":
                    av = (av * np.repeat(a.scale, a.k_domain, axis=1)[:, :K]).astype(np.float32)
                if b.scale_kind == "k":
                    bv = (bv * np.repeat(b.scale, b.k_domain, axis=1)[:, :K]).astype(np.float32)
            if spec.algorithm == "fp64":
                accd = np.zeros((M, N), np.float64)
                with np.errstate(invalid="ignore", over="ignore"):
                    for k in range(K):
                        accd = av[:, k, None].astype(np.float64) * bv[None, :, k].astype(np.float64) + accd
                acc = accd.astype(np.float32)
            else:
                for k in range(K):
                    acc = fp32_fma(av[:, k, None], bv[None, :, k], acc)
    with np.errstate(invalid="ignore", over="ignore"):
        if b.scale_kind in ("tensor", "row"):
            acc = (np.asarray(b.scale, np.float32).reshape(1, -1) * acc).astype(np.float32)
        if a.scale_kind in ("tensor", "row"):
            acc = (np.asarray(a.scale, np.float32).reshape(-1, 1) * acc).astype(np.float32)
        alpha = None
        for op in (a, b):
            if op.alpha is not None:
                v = np.float32(np.asarray(op.alpha).reshape(()))
                alpha = v if alpha is None else np.float32(alpha * v)
        if alpha is not None:
            acc = (alpha * acc).astype(np.float32)
        if bias is not None:
            acc = (acc + bias.reshape(1, -1)).astype(np.float32)
    return round_to_format(acc, spec.out_format, "rne", saturate=False)
