"""Cast and quantize on the B200 library: the drop-in replacements of TriCast's
``tricast.kernels.quantize`` module (``src/tricast/kernels/quantize.py:161-275``).

``round_to_format_triton`` and ``quantize_triton`` keep TriCast's names, arguments, outputs and
error messages so TriCast's dispatchers (``quant/api.py:49-52``) call them unchanged. Every cast
and scale computation runs in ``libtricast_b200`` on the current CUDA stream of the input's
device; nothing here computes values on the host.
"""

from __future__ import annotations

import ctypes as C

from dataclasses import dataclass

import torch

from . import _native as N
from .formats import container_dtype, get_format
from .operand import qtensor_class
from .rounding import Rounding


def _require_cuda(x: torch.Tensor) -> None:
    if not x.is_cuda:
        raise ValueError("the B200 backend requires a CUDA tensor")


def _noise(noise, shape, device):
    """uint32 noise broadcast to ``shape``; TriCast passes uint32 values in an int64 tensor."""
    if noise is None:
        return None
    n = torch.broadcast_to(noise.to(device=device), shape)
    if n.dtype != torch.int32:
        n = n.to(torch.int64).to(torch.int32)  # keeps the low 32 bits
    return n.contiguous()


def round_to_format_triton(x: torch.Tensor, fmt, rounding=Rounding.RNE, *, saturate: bool = True,
                           noise: torch.Tensor | None = None, sr_bits: int = 32) -> torch.Tensor:
    """Cast onto ``fmt``'s grid (TriCast ``round_to_format``); fp32 out, same shape."""
    f = get_format(fmt)
    code = N.rounding_code(rounding)
    if f.kind == "pow2" and code == 5:
        raise ValueError("stochastic rounding is not defined for power-of-two formats")
    if not 1 <= sr_bits <= 32:
        raise ValueError("sr_bits must be in [1, 32]")
    _require_cuda(x)
    x = x.to(torch.float32).contiguous()
    nz = _noise(noise, x.shape, x.device)
    out = torch.empty_like(x)
    if x.numel():
        with torch.cuda.device(x.device):
            N.check(N.lib().tc_cast(N.ptr(x), N.ptr(out), N.ptr(nz), x.numel(), N.tc_format(f), code, int(saturate),
                                    sr_bits, N.stream_of(x.device)), "tc_cast")
    return out


def layout(spec, rows: int, K: int) -> tuple:
    """Scale layout of ``spec`` for a [rows, K] view (``reference/quantize.py:50-58``)."""
    if spec.granularity == "tensor":
        return ()
    if spec.granularity == "row":
        return (rows, 1)
    if spec.granularity == "group":
        return (rows, -(-K // spec.group_size))
    br, bc = spec.block
    return (-(-rows // br), -(-K // bc))


def _validate_scale_spec(spec, scale_noise) -> None:
    """TriCast ``_validate_scale_spec`` (``reference/quantize.py:222-230``)."""
    sf = spec.scale
    if sf is None:
        return
    if Rounding.parse(sf.rounding) is Rounding.SR:
        if sf.format.kind == "pow2" or sf.method in ("pow2_floor", "pow2_ceil"):
            raise ValueError("stochastic rounding is not supported for power-of-two scales")
        if scale_noise is None:
            raise ValueError("scale stochastic rounding requires explicit scale_noise")


def _qspec(spec) -> N.TcQuantSpec:
    s = N.TcQuantSpec()
    s.format = N.tc_format(spec.format)
    s.granularity = N.GRANULARITY_CODES[spec.granularity]
    s.group_size = int(spec.group_size)
    s.block_rows, s.block_cols = (int(v) for v in spec.block)
    s.rounding = N.rounding_code(spec.rounding)
    s.sr_bits = int(spec.sr_bits)
    s.saturate = int(bool(spec.saturate))
    s.zero_point = N.ZERO_POINT_CODES[spec.zero_point]
    sf = spec.scale
    if sf is not None:
        s.has_scale = 1
        s.scale_format = N.tc_format(sf.format)
        s.scale_method = N.METHOD_CODES[sf.method]
        s.scale_rounding = N.rounding_code(sf.rounding)
        s.two_level = int(bool(sf.two_level))
        s.percentile = float(sf.percentile)
        if sf.method == "mse":
            # The candidate ratios exactly as TriCast forms them (src/tricast/reference/quantize.py:290-291).
            search = tuple(getattr(sf, "search", ()) or ())
            ratios = (torch.tensor(search, dtype=torch.float32).tolist() if search else
                      torch.linspace(1.0, 0.5, int(sf.mse_grid), dtype=torch.float32, device="cpu").tolist())
            s.n_search = len(ratios)
            s.mse_search = (C.c_float * len(ratios))(*ratios)  # kept alive by the structure
    return s


def _bits_of(fmt) -> int:
    f = get_format(fmt)
    if f.kind == "float":
        return f.ebits + f.mbits + int(f.signed)
    if f.kind == "int":
        return f.bits
    return f.ebits


@dataclass
class QuantExtras:
    """Optional outputs written by the same pass as the QTensor fields."""
    codes: torch.Tensor | None = None        # uint8: 4-bit formats packed two per byte (low nibble first)
    scale_codes: torch.Tensor | None = None  # uint8 per scale (E8M0: exponent + 127)
    dequant: torch.Tensor | None = None      # fp32 dequantized values


def quantize_into(x: torch.Tensor, spec, *, amax=None, noise=None, seed: int = 0, scale_noise=None,
                  want_codes: bool = False, want_scale_codes: bool = False, want_dequant: bool = False,
                  want_values: bool = True, tensor_amax=None):
    """Quantize and return ``(QTensor, QuantExtras)``; the extras are written in the same pass.
    ``want_values=False`` skips the QTensor values (the QTensor then carries ``values=None``).
    ``tensor_amax`` (two-level specs such as NVFP4 only, not part of TriCast's API): the amax of the
    whole tensor of which ``x`` is a row shard, from which the global scale is derived, so that the
    shard's QTensor equals those rows of the whole tensor's."""
    if x.ndim == 0 or x.numel() == 0:
        raise ValueError("quantization needs a nonempty tensor of shape [..., K]")
    _validate_scale_spec(spec, scale_noise)
    _require_cuda(x)
    shape = tuple(x.shape)
    if x.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        x = x.to(torch.float32)
    x2d = x.reshape(-1, shape[-1])
    if not x2d.is_contiguous():
        x2d = x2d.contiguous()
    rows, K = x2d.shape
    device = x.device
    if amax is not None:
        if spec.granularity != "tensor" or amax.numel() != 1:
            raise ValueError("amax override requires tensor granularity and a scalar")
        amax = amax.to(device=device, dtype=torch.float32).reshape(()).contiguous()
    if tensor_amax is not None:
        if amax is not None or spec.scale is None or not spec.scale.two_level or spec.granularity == "tensor":
            raise ValueError("tensor_amax needs a two-level spec of group, row or block granularity")
        if tensor_amax.numel() != 1:
            raise ValueError("tensor_amax must be a scalar")
        amax = tensor_amax.to(device=device, dtype=torch.float32).reshape(()).contiguous()
    if (N.rounding_code(spec.rounding) == 5 and noise is None and spec.scale is not None
            and spec.scale.method == "mse"):
        raise ValueError("MSE with stochastic rounding requires explicit noise")
    if N.rounding_code(spec.rounding) == 5 and noise is None:
        # TriCast's public API refuses SR without noise; the backend itself draws seeded noise.
        gen = torch.Generator(device=device)
        gen.manual_seed(int(seed))
        noise = torch.randint(0, 2 ** 32, shape, generator=gen, device=device, dtype=torch.int64)
    nz = _noise(noise, shape, device)
    nz = None if nz is None else nz.reshape(rows, K)
    sf = spec.scale
    lay = layout(spec, rows, K) if sf is not None else ()
    sn = None
    if sf is not None and scale_noise is not None:
        sn = _noise(scale_noise, lay, device)
    values = torch.empty((rows, K), device=device, dtype=container_dtype(spec.format)) if want_values else None
    scale = zero = gscale = None
    if sf is not None:
        scale = torch.empty(lay, device=device, dtype=torch.float32)
        if spec.zero_point != "none":
            zero = torch.empty(lay, device=device, dtype=torch.float32)
        if sf.two_level:
            gscale = torch.empty((), device=device, dtype=torch.float32)
    extras = QuantExtras()
    if want_codes:
        nbits = _bits_of(spec.format)
        if nbits > 8:
            raise ValueError("element codes need a format of at most 8 bits")
        extras.codes = torch.empty((rows * K + 1) // 2 if nbits <= 4 else rows * K, device=device, dtype=torch.uint8)
    if want_scale_codes and sf is not None:
        extras.scale_codes = torch.empty(lay, device=device, dtype=torch.uint8)
    if want_dequant:
        extras.dequant = torch.empty((rows, K), device=device, dtype=torch.float32)
    qs = _qspec(spec)
    out = N.TcQuantOut()
    out.values = 0 if values is None else values.data_ptr()
    out.values_dtype = N.dtype_code(container_dtype(spec.format))
    for name, t in (("scale", scale), ("zero_point", zero), ("global_scale", gscale), ("codes", extras.codes),
                    ("scale_codes", extras.scale_codes), ("dequant", extras.dequant)):
        setattr(out, name, 0 if t is None else t.data_ptr())
    lib = N.lib()
    with torch.cuda.device(device):
        ws_bytes = lib.tc_quantize_workspace(rows, K, qs)
        ws = torch.empty(max(ws_bytes, 1), device=device, dtype=torch.uint8)
        N.check(lib.tc_quantize(N.ptr(x2d), N.dtype_code(x2d.dtype), rows, K, qs, N.ptr(amax), N.ptr(nz), N.ptr(sn),
                                out, N.ptr(ws), ws.numel(), N.stream_of(device)), "tc_quantize")
    cls = qtensor_class(spec)
    return cls(values, scale, zero, gscale, spec, shape), extras


class QuantizePlan:
    """A quantize call prepared once for a fixed input shape, dtype and spec: outputs, workspace and
    the C descriptors are allocated up front, so ``run(x)`` is one library call that overwrites them
    (for loops that quantize same-shaped tensors repeatedly). Deterministic roundings only."""

    def __init__(self, shape, dtype: torch.dtype, device, spec, *, want_values: bool = True,
                 want_codes: bool = False, want_scale_codes: bool = False, want_dequant: bool = False):
        _validate_scale_spec(spec, None)
        if N.rounding_code(spec.rounding) == 5:
            raise ValueError("QuantizePlan takes deterministic roundings; use quantize_into for 'sr'")
        x = torch.empty(shape, dtype=dtype, device=device)
        _require_cuda(x)
        self.shape, self.dtype, self.spec = tuple(shape), dtype, spec
        self.rows, self.K = x.reshape(-1, self.shape[-1]).shape
        q, extras = quantize_into(x.zero_(), spec, want_values=want_values, want_codes=want_codes,
                                  want_scale_codes=want_scale_codes, want_dequant=want_dequant)
        self.qtensor, self.extras = q, extras
        self.device = x.device
        self._qs = _qspec(spec)
        out = N.TcQuantOut()
        out.values = 0 if q.values is None else q.values.data_ptr()
        out.values_dtype = N.dtype_code(container_dtype(spec.format))
        for name, t in (("scale", q.scale), ("zero_point", q.zero_point), ("global_scale", q.global_scale),
                        ("codes", extras.codes), ("scale_codes", extras.scale_codes), ("dequant", extras.dequant)):
            setattr(out, name, 0 if t is None else t.data_ptr())
        self._out = out
        lib = N.lib()
        with torch.cuda.device(self.device):
            ws_bytes = lib.tc_quantize_workspace(self.rows, self.K, self._qs)
        self._ws = torch.empty(max(ws_bytes, 1), device=self.device, dtype=torch.uint8)
        self._lib = lib

    def run(self, x: torch.Tensor):
        """Quantize ``x`` (the planned shape and dtype, contiguous, on the planned device) into the
        plan's outputs on the current stream; returns ``(QTensor, QuantExtras)``."""
        if tuple(x.shape) != self.shape or x.dtype != self.dtype or x.device != self.device or not x.is_contiguous():
            raise ValueError("QuantizePlan.run needs a contiguous tensor of the planned shape, dtype and device")
        N.check(self._lib.tc_quantize(x.data_ptr(), N.dtype_code(x.dtype), self.rows, self.K, self._qs, None, None,
                                      None, self._out, self._ws.data_ptr(), self._ws.numel(),
                                      N.stream_of(self.device)), "tc_quantize")
        return self.qtensor, self.extras


def quantize_triton(x: torch.Tensor, spec, *, amax: torch.Tensor | None = None, noise: torch.Tensor | None = None,
                    seed: int = 0, scale_noise: torch.Tensor | None = None):
    """Quantize onto ``spec`` (TriCast ``quantize_triton``): returns a QTensor whose values are in
    the container dtype, scales fp32 in the scale layout, and the global scale fp32."""
    return quantize_into(x, spec, amax=amax, noise=noise, seed=seed, scale_noise=scale_noise)[0]


def quantize(x: torch.Tensor, spec, **kwargs):
    """``quantize_triton`` accepting a scheme name as well (TriCast ``quant/api.py:34-55`` on CUDA)."""
    from .spec import get_scheme

    spec = get_scheme(spec)
    if N.rounding_code(spec.rounding) == 5 and kwargs.get("noise") is None:
        raise ValueError("stochastic rounding requires explicit noise")
    return quantize_triton(x, spec, **kwargs)


def element_bits(spec) -> int:
    return _bits_of(spec.format)


__all__ = ["round_to_format_triton", "quantize_triton", "quantize_into", "quantize", "layout", "QuantExtras"]
