"""Oracle quantization with explicit fp32 scale arithmetic (TEST INFRASTRUCTURE ONLY).

Restates ``src/tricast/reference/quantize.py``. Every fp32 operation is computed in fp64 and rounded
once to fp32, which is exact IEEE binary32 for fp32 operands (``quantize.py:17-40``).
"""

from __future__ import annotations

import math
from types import SimpleNamespace

import numpy as np

from .cast import ldexp, rounding_name, round_to_format, round_up


def f32(v) -> np.ndarray:
    return np.asarray(v, np.float64).astype(np.float32)


def _div(a, b):
    """binary32 a / b (``quantize.py:17-22``); Python-float divisors are taken as fp64."""
    a = np.asarray(a, np.float32).astype(np.float64)
    b = float(b) if isinstance(b, (int, float)) else np.asarray(b, np.float32).astype(np.float64)
    with np.errstate(divide="ignore", invalid="ignore"):
        return (a / b).astype(np.float32)


def _mul(a, b):
    a = np.asarray(a, np.float32).astype(np.float64)
    b = float(b) if isinstance(b, (int, float)) else np.asarray(b, np.float32).astype(np.float64)
    with np.errstate(invalid="ignore", over="ignore"):
        return (a * b).astype(np.float32)


def _sub(a, b):
    a = float(a) if isinstance(a, (int, float)) else np.asarray(a, np.float32).astype(np.float64)
    b = float(b) if isinstance(b, (int, float)) else np.asarray(b, np.float32).astype(np.float64)
    with np.errstate(invalid="ignore"):
        return np.asarray(a - b).astype(np.float32)


def _add(a, b):
    a = np.asarray(a, np.float32).astype(np.float64)
    b = float(b) if isinstance(b, (int, float)) else np.asarray(b, np.float32).astype(np.float64)
    with np.errstate(invalid="ignore"):
        return (a + b).astype(np.float32)


def domain_shape(spec, rows: int, K: int) -> tuple[int, int]:
    """Nominal (rows, cols) of one scale domain (``quantize.py:65,77``)."""
    if spec.granularity == "tensor":
        return rows, K
    if spec.granularity == "row":
        return 1, K
    if spec.granularity == "group":
        return 1, spec.group_size
    return tuple(spec.block)


def layout(spec, rows: int, K: int) -> tuple:
    """Scale layout (``quantize.py:50-58``)."""
    if spec.granularity == "tensor":
        return ()
    dr, dc = domain_shape(spec, rows, K)
    return (-(-rows // dr), -(-K // dc))


def domain_view(x2d: np.ndarray, spec):
    """Domains packed row-major as [domains, elements] plus a validity mask (``quantize.py:71-85``)."""
    rows, K = x2d.shape
    if spec.granularity == "tensor":
        data = x2d.reshape(1, -1)
        return data, np.ones(data.shape, bool)
    dr, dc = domain_shape(spec, rows, K)
    dr, dc = min(dr, rows), min(dc, K)
    nr, nc = -(-rows // dr), -(-K // dc)
    padded = np.zeros((nr * dr, nc * dc), x2d.dtype)
    padded[:rows, :K] = x2d
    valid = np.zeros(padded.shape, bool)
    valid[:rows, :K] = True
    shape = (nr, dr, nc, dc)
    return (padded.reshape(shape).transpose(0, 2, 1, 3).reshape(nr * nc, dr * dc),
            valid.reshape(shape).transpose(0, 2, 1, 3).reshape(nr * nc, dr * dc))


def expand(t: np.ndarray, spec, rows: int, K: int) -> np.ndarray:
    """Scale or zero point per element (``quantize.py:124-131``)."""
    t = np.asarray(t)
    if spec.granularity in ("tensor", "row"):
        return np.broadcast_to(t, (rows, K))
    if spec.granularity == "group":
        return np.repeat(t, spec.group_size, axis=1)[:, :K]
    br, bc = spec.block
    return np.repeat(np.repeat(t, br, axis=0), bc, axis=1)[:rows, :K]


def _nan_amax(data: np.ndarray, valid: np.ndarray) -> np.ndarray:
    a = np.where(valid, np.abs(data), np.float32(0))
    out = a.max(axis=1)
    return np.where(np.isnan(a).any(axis=1), np.float32(np.nan), out).astype(np.float32)


def _min_subnormal(fmt) -> float:
    return getattr(fmt, "min_subnormal", fmt.min_normal)


def absmax_scale(amax, spec, global_scale, scale_noise=None) -> np.ndarray:
    """``s = cast(RN(RN(amax / M) / d2))``, 0 -> min subnormal, amax 0 -> 1 (``quantize.py:134-145``)."""
    sf = spec.scale
    t = _div(amax, spec.format.max_normal)
    if global_scale is not None:
        t = _div(t, global_scale)
    s = round_to_format(t, sf.format, sf.rounding, saturate=True, noise=scale_noise)
    s = np.where(s == 0, np.float32(_min_subnormal(sf.format)), s)
    return np.where(np.asarray(amax) == 0, np.float32(1.0), s).astype(np.float32)


def pow2_scale(amax, spec) -> np.ndarray:
    """``2**(floor(log2 amax) - emax_elem)`` (+1 for ceil when it clips) (``quantize.py:148-159``)."""
    sf = spec.scale
    a = np.where(np.asarray(amax) == 0, 2.0 ** -126, np.asarray(amax, np.float32).astype(np.float64))
    emax_elem = math.frexp(spec.format.max_normal)[1] - 1
    with np.errstate(invalid="ignore"):
        _, ex = np.frexp(a)
        e = ex.astype(np.int64) - 1 - emax_elem
        if sf.method == "pow2_ceil":
            e = e + (ldexp(np.full(a.shape, spec.format.max_normal), e) < a)
        overflow = (e > sf.format.emax) | ~np.isfinite(a)
        e = np.clip(e, sf.format.emin, sf.format.emax)
        s = ldexp(np.ones(a.shape), e).astype(np.float32)
    return np.where(overflow, np.float32(np.nan), s).astype(np.float32)


def global_scale(amax: float, spec) -> np.float32:
    """One exact rounding of ``amax / (M * SF.max)`` to binary32 (``quantize.py:195-219``)."""
    value = float(np.float32(amax))
    if not math.isfinite(value):
        return np.float32(value)
    if value == 0:
        return np.float32(1.0)
    num, den = value.as_integer_ratio()
    pn, pd = (spec.format.max_normal * spec.scale.format.max_normal).as_integer_ratio()
    num, den = num * pd, den * pn
    negative = num < 0
    num = abs(num)
    e = num.bit_length() - den.bit_length()
    if (num < (den << e)) if e >= 0 else ((num << -e) < den):
        e -= 1
    quantum = max(e, -126) - 23
    if quantum < 0:
        num <<= -quantum
    else:
        den <<= quantum
    kept, rem = divmod(num, den)
    if 2 * rem > den or (2 * rem == den and kept % 2 == 1):
        kept += 1
    result = math.ldexp(kept, quantum)
    result = -result if negative else result
    return np.float32(1.0) if result == 0 else np.float32(result)


def signed_zero_extrema(data: np.ndarray, valid: np.ndarray):
    """Domain min/max with -0 below +0 and NaN propagation (``quantize.py:88-115,162-173``)."""
    big = np.float32(np.inf)
    lo = np.where(valid, data, big).min(axis=1)
    hi = np.where(valid, data, -big).max(axis=1)
    nan = (np.isnan(data) & valid).any(axis=1)
    zero = (data == 0) & valid
    neg_zero = (zero & np.signbit(data)).any(axis=1)
    pos_zero = (zero & ~np.signbit(data)).any(axis=1)
    lo = np.where(lo == 0, np.where(neg_zero, np.float32(-0.0), np.float32(0.0)), lo)
    hi = np.where(hi == 0, np.where(pos_zero, np.float32(0.0), np.float32(-0.0)), hi)
    lo = np.where(nan, np.float32(np.nan), lo).astype(np.float32)
    hi = np.where(nan, np.float32(np.nan), hi).astype(np.float32)
    return lo, hi


def zero_point_scale(lo, hi, spec, scale_noise=None):
    """Affine scale and zero point from the domain range (``quantize.py:176-192``)."""
    fmt, sf = spec.format, spec.scale
    if spec.zero_point == "int":
        lo = np.where(lo > 0, np.float32(0.0), lo).astype(np.float32)  # clamp(max=0) keeps -0 and NaN
        hi = np.where(hi < 0, np.float32(0.0), hi).astype(np.float32)
    raw = _div(_sub(hi, lo), float(fmt.qmax - fmt.qmin))
    s = round_to_format(raw, sf.format, sf.rounding, saturate=True, noise=scale_noise)
    s = np.where(s == 0, np.float32(_min_subnormal(sf.format)), s)
    s = np.where(hi == lo, np.float32(1.0), s).astype(np.float32)
    z = lo
    if spec.zero_point == "int":
        with np.errstate(invalid="ignore"):
            z = np.round(_sub(float(fmt.qmin), _div(lo, s)))  # numpy rounds half to even, as torch.round
            z = np.clip(z, fmt.qmin, fmt.qmax).astype(np.float32)
    return s, z


def percentile_amax(data, valid, percentile) -> np.ndarray:
    """Linear quantile of |x| per domain (``quantize.py:233-241``); torch.lerp's two-sided form."""
    ordered = np.sort(np.where(valid, np.abs(data), np.float32(np.inf)), axis=1)
    rank = (valid.sum(axis=1) - 1).astype(np.float64) * (percentile / 100)
    below = np.floor(rank).astype(np.int64)
    above = np.ceil(rank).astype(np.int64)
    lo = np.take_along_axis(ordered, below[:, None], 1)[:, 0].astype(np.float64)
    hi = np.take_along_axis(ordered, above[:, None], 1)[:, 0].astype(np.float64)
    w = rank - below
    with np.errstate(invalid="ignore"):
        value = np.where(w < 0.5, lo + w * (hi - lo), hi - (hi - lo) * (1 - w)).astype(np.float32)
    return np.where(np.isnan(data).any(axis=1), np.float32(np.nan), value).astype(np.float32)


def compute_scale(x2d, spec, amax=None, *, noise=None, scale_noise=None):
    """Per-domain scales, zero points and the global scale (``quantize.py:244-305``)."""
    x2d = np.asarray(x2d, np.float32)
    rows, K = x2d.shape
    if amax is not None:
        if spec.granularity != "tensor" or np.size(amax) != 1:
            raise ValueError("amax override requires tensor granularity and a scalar")
        amax = np.float32(np.asarray(amax, np.float32).reshape(()))
    if spec.scale is None:
        return None, None, None
    sf = spec.scale
    if rounding_name(sf.rounding) == "sr":
        if sf.format.kind == "pow2" or sf.method in ("pow2_floor", "pow2_ceil"):
            raise ValueError("stochastic rounding is not supported for power-of-two scales")
        if scale_noise is None:
            raise ValueError("scale stochastic rounding requires explicit scale_noise")
    shape = layout(spec, rows, K)
    if scale_noise is not None:
        scale_noise = np.broadcast_to(np.asarray(scale_noise, np.int64), shape).reshape(-1)
    data, valid = domain_view(x2d, spec)
    if spec.zero_point != "none":
        lo, hi = signed_zero_extrema(data, valid)
        s, z = zero_point_scale(lo, hi, spec, scale_noise)
        return s.reshape(shape), z.reshape(shape), None
    maxima = _nan_amax(data, valid) if amax is None else amax.reshape(1)
    gscale = None
    if sf.two_level:
        gscale = global_scale(_nan_amax(x2d.reshape(1, -1), np.ones((1, x2d.size), bool))[0]
                              if amax is None else amax, spec)
    if not sf.two_level and sf.method in ("pow2_floor", "pow2_ceil"):
        return pow2_scale(maxima, spec).reshape(shape), None, gscale
    if amax is None and sf.method == "percentile":
        maxima = percentile_amax(data, valid, sf.percentile)
    if amax is None and sf.method == "mse":
        if rounding_name(spec.rounding) == "sr" and noise is None:
            raise ValueError("MSE with stochastic rounding requires explicit noise")
        domain_noise = None
        if noise is not None:
            domain_noise, _ = domain_view(np.broadcast_to(np.asarray(noise, np.int64), x2d.shape), spec)
        ratios = ([float(np.float32(r)) for r in sf.search] if sf.search else
                  [float(np.float32(v)) for v in np.linspace(1.0, 0.5, sf.mse_grid, dtype=np.float32)])
        best = scales = None
        for ratio in ratios:
            cand = absmax_scale(_mul(maxima, ratio), spec, gscale, scale_noise)
            q = quantize_elements(data, spec, cand[:, None], global_scale=gscale, noise=domain_noise)
            restored = _mul(q, cand[:, None])
            if gscale is not None:
                restored = _mul(restored, gscale)
            err = np.where(valid, (data.astype(np.float64) - restored.astype(np.float64)) ** 2, 0.0).sum(axis=1)
            if best is None:
                scales, best = cand, err
            else:
                better = err < best
                scales = np.where(better, cand, scales)
                best = np.where(better, err, best)
    else:
        scales = absmax_scale(maxima, spec, gscale, scale_noise)
    return np.asarray(scales, np.float32).reshape(shape), None, gscale


def quantize_elements(x2d, spec, scale_pe, zp_pe=None, global_scale=None, noise=None) -> np.ndarray:
    """Round elements under given scales (``quantize.py:308-334``)."""
    x = np.asarray(x2d, np.float32)
    if zp_pe is not None and spec.zero_point == "float":
        x = _sub(x, zp_pe)
    if scale_pe is not None:
        eff = np.asarray(scale_pe, np.float32)
        if global_scale is not None:
            eff = _mul(eff, global_scale)
        x = _div(x, eff)
    if zp_pe is not None:
        with np.errstate(invalid="ignore"):
            mag = np.abs(x.astype(np.float64))
            integer = np.floor(mag)
            inc = round_up(mag - integer, integer, x < 0, rounding_name(spec.rounding),
                           None if noise is None else np.broadcast_to(np.asarray(noise, np.int64), x.shape),
                           spec.sr_bits)
            rounded = np.copysign(integer + inc, x.astype(np.float64))
            if spec.zero_point == "int":
                rounded = rounded + np.asarray(zp_pe, np.float32).astype(np.float64)
            return np.clip(rounded, spec.format.qmin, spec.format.qmax).astype(np.float32)
    return round_to_format(x, spec.format, spec.rounding, saturate=spec.saturate, noise=noise,
                           sr_bits=spec.sr_bits)


def quantize_reference(x, spec, *, amax=None, noise=None, scale_noise=None) -> SimpleNamespace:
    """QTensor fields as numpy arrays: values (grid values, fp32), scale, zero_point, global_scale
    (``quantize.py:337-350``)."""
    x = np.asarray(x, np.float32)
    if x.ndim == 0 or x.size == 0:
        raise ValueError("quantization needs a nonempty tensor of shape [..., K]")
    x2d = x.reshape(-1, x.shape[-1])
    if noise is not None:
        noise = np.broadcast_to(np.asarray(noise, np.int64), x.shape).reshape(x2d.shape)
    scale, zero, gscale = compute_scale(x2d, spec, amax, noise=noise, scale_noise=scale_noise)
    rows, K = x2d.shape
    spe = None if scale is None else expand(scale, spec, rows, K)
    zpe = None if zero is None else expand(zero, spec, rows, K)
    values = quantize_elements(x2d, spec, spe, zpe, gscale, noise)
    return SimpleNamespace(values=values, scale=scale, zero_point=zero,
                           global_scale=None if gscale is None else np.float32(gscale), spec=spec,
                           shape=tuple(x.shape))


def dequantize(q: SimpleNamespace) -> np.ndarray:
    """``((v - z) * s [+ z]) * d2`` with one fp32 rounding per step (``qtensor.py:40-55``)."""
    spec = q.spec
    x = np.asarray(q.values, np.float32)
    rows, K = x.shape
    zero = None
    if q.zero_point is not None:
        zero = expand(q.zero_point, spec, rows, K)
        if spec.zero_point == "int":
            x = _sub(x, zero)
    if q.scale is not None:
        x = _mul(x, expand(q.scale, spec, rows, K))
    if zero is not None and spec.zero_point == "float":
        x = _add(x, zero)
    if q.global_scale is not None:
        x = _mul(x, q.global_scale)
    return x.reshape(q.shape)
