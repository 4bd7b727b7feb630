"""Oracle casts in fp64 numpy (TEST INFRASTRUCTURE ONLY).

Restates ``src/tricast/reference/cast.py``: inputs go to fp64, where every fp32 value and every
power-of-two rescaling is exact, so each cast is one exact rescale plus one rounding decision.
"""

from __future__ import annotations

import numpy as np

ROUNDING_NAMES = ("rne", "rna", "rtz", "rup", "rdn", "sr")


def rounding_name(r) -> str:
    name = getattr(r, "value", r)
    name = str(name).lower()
    name = {"even": "rne", "trunc": "rtz", "truncate": "rtz", "stochastic": "sr"}.get(name, name)
    if name not in ROUNDING_NAMES:
        raise ValueError(f"unknown rounding {r!r}")
    return name


def floor_log2(ax: np.ndarray) -> np.ndarray:
    """Exact floor(log2) of positive finite fp64 values; 0 elsewhere (``cast.py:86-90``)."""
    _, e = np.frexp(ax)
    ok = (ax > 0) & np.isfinite(ax)
    return np.where(ok, e.astype(np.int64) - 1, 0)


def ldexp(x, e) -> np.ndarray:
    """x * 2**e in fp64, applied in two factors so shifts beyond one exponent range stay exact
    (``cast.py:93-109``)."""
    e = np.asarray(e, dtype=np.int64)
    first = np.clip(e, -1022, 1023)
    rest = np.clip(e - first, -1022, 1023)
    return np.ldexp(np.ldexp(np.asarray(x, np.float64), first.astype(np.int32)), rest.astype(np.int32))


def round_up(frac, k, negative, rounding: str, noise, sr_bits: int) -> np.ndarray:
    """Whether to add one quantum to the truncated magnitude (``cast.py:112-135``)."""
    if rounding == "rne":
        return (frac > 0.5) | ((frac == 0.5) & (np.remainder(k, 2) == 1))
    if rounding == "rna":
        return frac >= 0.5
    if rounding == "rtz":
        return np.zeros(np.shape(frac), bool)
    if rounding == "rup":
        return (frac > 0) & ~negative
    if rounding == "rdn":
        return (frac > 0) & negative
    if not 1 <= sr_bits <= 32:
        raise ValueError("sr_bits must be in [1, 32]")
    if noise is None:
        raise ValueError("stochastic rounding requires explicit noise or generator")
    u = np.floor(np.asarray(noise, np.int64).astype(np.float64) / 2.0 ** (32 - sr_bits)) / 2.0 ** sr_bits
    return u < frac


def round_to_format(x, fmt, rounding="rne", *, saturate=True, noise=None, sr_bits=32) -> np.ndarray:
    """Grid value nearest to ``x`` under ``rounding``; fp32 out (``cast.py:18-83``)."""
    rounding = rounding_name(rounding)
    xd = np.asarray(x, np.float32).astype(np.float64)
    if fmt.kind == "pow2":
        return _round_pow2(xd, fmt, rounding, saturate)
    if fmt.kind == "float":
        if not fmt.subnormals:
            xd = np.where(np.abs(xd) < fmt.min_normal, np.copysign(0.0, xd), xd)
        quantum = np.maximum(floor_log2(np.abs(xd)), fmt.emin) - fmt.mbits
    elif fmt.kind == "int":
        quantum = np.full(xd.shape, -fmt.frac_bits, np.int64)
    else:
        raise TypeError(f"unsupported format {fmt!r}")
    ax = np.abs(xd)
    finite = np.isfinite(xd)
    with np.errstate(invalid="ignore"):
        y = ldexp(np.where(finite, ax, 0.0), -quantum)
        k = np.floor(y)
        frac = y - k
        if noise is not None:
            noise = np.broadcast_to(np.asarray(noise, np.int64), xd.shape)
        inc = round_up(frac, k, xd < 0, rounding, noise, sr_bits)
        mag = ldexp(k + inc, quantum)
        isnan = np.isnan(xd)
        if fmt.kind == "int":
            neg_bound = -fmt.qmin * 2.0 ** -fmt.frac_bits
            mag = np.where(xd < 0, np.minimum(mag, neg_bound), np.minimum(mag, fmt.max_normal))
            if not fmt.signed:
                mag = np.where(xd < 0, 0.0, mag)
            bound = np.where(xd < 0, neg_bound, fmt.max_normal)
            if not fmt.signed:
                bound = np.where(xd < 0, 0.0, bound)
            mag = np.where(finite, mag, np.where(isnan, np.abs(xd), bound))
            out = np.copysign(mag, xd) if fmt.signed else mag
            return np.where(isnan, xd, out).astype(np.float32)
        over = (mag > fmt.max_normal) | np.isinf(xd)
        mag = np.where(over, _overflow(xd, fmt, rounding, saturate), mag)
        out = np.where(isnan, xd, np.copysign(mag, xd))
        if fmt.special == "fnuz" or not fmt.signed:
            out = np.where(out == 0, 0.0, out)
        if not fmt.signed:
            out = np.where(xd < 0, 0.0 if saturate else np.nan, out)
    return out.astype(np.float32)


def _overflow(xd, fmt, rounding: str, saturate: bool) -> np.ndarray:
    """Value of an overflowing magnitude (``cast.py:138-147``)."""
    top = np.full(xd.shape, fmt.max_normal)
    if saturate or fmt.special == "none":
        return top
    if fmt.special in ("fn", "fnuz"):
        return np.full(xd.shape, np.nan)
    negative = xd < 0
    away = {"rtz": np.zeros_like(negative), "rup": ~negative, "rdn": negative}.get(
        rounding, np.ones_like(negative))
    return np.where(away, np.inf, top)


def _round_pow2(xd, fmt, rounding: str, saturate: bool) -> np.ndarray:
    """Round |x| to a power of two by value, ties up (``cast.py:156-179``)."""
    if rounding == "sr":
        raise ValueError("stochastic rounding is not defined for power-of-two formats")
    ax = np.abs(xd)
    e = floor_log2(ax)
    with np.errstate(invalid="ignore", divide="ignore"):
        frac = np.where(np.isfinite(ax), ax / ldexp(np.ones_like(ax), e) - 1.0, 0.0)
        if rounding in ("rne", "rna"):
            up = frac >= 0.5
        elif rounding == "rup":
            up = frac > 0
        else:
            up = np.zeros(ax.shape, bool)
        e = np.maximum(e + up, fmt.emin)
        over = (e > fmt.emax) | np.isinf(ax)
        out = ldexp(np.ones_like(ax), np.minimum(e, fmt.emax))
        out = np.where(over, fmt.max_normal, out)
        out = np.where(ax == 0, fmt.min_normal, out)
        bad = np.isnan(xd) | (xd < 0) | (over & (not saturate))
        out = np.where(bad, np.nan, out)
    return out.astype(np.float32)


def decode(v, fmt):
    """Grid values -> (negative, exponent, significand, radix) with the format-native,
    unnormalised convention (``cast.py:186-236``). Raises on off-grid values."""
    vd = np.asarray(v, np.float64)
    if not np.isfinite(vd).all():
        raise ValueError("decode() takes finite grid values; handle NaN/Inf before decoding")
    negative = vd < 0
    ax = np.abs(vd)
    if fmt.kind == "float":
        exp = np.maximum(floor_log2(ax), fmt.emin)
        radix = fmt.mbits
    elif fmt.kind == "int":
        exp = np.zeros(ax.shape, np.int64)
        radix = fmt.frac_bits
    else:
        exp = floor_log2(ax)
        radix = 0
    sig_f = ldexp(ax, radix - exp)
    if not np.array_equal(sig_f, np.floor(sig_f)):
        raise ValueError(f"values are not on the {fmt} grid")
    if fmt.kind == "float":
        bad = ax > fmt.max_normal
        if not fmt.subnormals:
            bad |= (ax > 0) & (ax < fmt.min_normal)
        bad |= (vd < 0) & (not fmt.signed)
    elif fmt.kind == "int":
        k = np.where(vd < 0, -sig_f, sig_f)
        bad = (k < fmt.qmin) | (k > fmt.qmax)
    else:
        bad = (vd <= 0) | (sig_f != 1) | (exp < fmt.emin) | (exp > fmt.emax)
    if bad.any():
        raise ValueError(f"values are outside the representable range of {fmt}")
    sig = sig_f.astype(np.int64)
    exp = np.where(sig == 0, 0, exp)
    return negative, exp, sig, radix
