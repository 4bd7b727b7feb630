"""``Operand`` and ``QTensor`` containers mirroring ``tricast/mma/operand.py:28-100`` and
``tricast/quant/qtensor.py:16-82``.

When TriCast is installed the backend returns TriCast's own classes instead (see ``qtensor_class``),
so callers above the API see exactly the types they expect.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .formats import container_dtype


@dataclass
class Operand:
    values: torch.Tensor
    fmt: object
    scale: torch.Tensor | None = None
    scale_fmt: object = None
    scale_kind: str = "none"
    k_domain: int = 0
    alpha: torch.Tensor | None = None

    def __post_init__(self) -> None:
        if self.values.dim() != 2:
            raise ValueError("operand values must be 2-D [rows, K]")
        if (self.scale is None) != (self.scale_kind == "none"):
            raise ValueError("scale and scale_kind disagree")
        if self.scale_kind == "k" and self.k_domain <= 0:
            raise ValueError("K-varying scales need k_domain > 0")

    @property
    def rows(self) -> int:
        return self.values.shape[0]

    @property
    def K(self) -> int:
        return self.values.shape[1]

    def scale_per_element(self):
        if self.scale is None:
            return None
        if self.scale_kind == "k":
            return self.scale.repeat_interleave(self.k_domain, dim=1)[:, : self.K]
        return self.scale.expand(self.rows, self.K)


def expand_scale(t: torch.Tensor, spec, rows: int, K: int) -> torch.Tensor:
    """One scale (or zero point) per element, from the domain layout of ``spec``."""
    if spec.granularity in ("tensor", "row"):
        return t.expand(rows, K)
    if spec.granularity == "group":
        return t.repeat_interleave(spec.group_size, dim=1)[:, :K]
    br, bc = spec.block
    return t.repeat_interleave(br, dim=0).repeat_interleave(bc, dim=1)[:rows, :K]


@dataclass
class QTensor:
    values: torch.Tensor
    scale: torch.Tensor | None
    zero_point: torch.Tensor | None
    global_scale: torch.Tensor | None
    spec: object
    shape: tuple

    @property
    def rows(self) -> int:
        return self.values.shape[0]

    @property
    def K(self) -> int:
        return self.values.shape[1]

    def scale_per_element(self):
        if self.scale is None:
            return None
        return expand_scale(self.scale, self.spec, self.rows, self.K)

    def dequantize(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """``((v - z) * s [+ z]) * d2`` with one fp32 rounding per step (``qtensor.py:40-55``)."""
        x = self.values.double()
        zero = None
        if self.zero_point is not None:
            zero = expand_scale(self.zero_point, self.spec, self.rows, self.K)
            if self.spec.zero_point == "int":
                x = (x - zero.double()).float().double()
        if self.scale is not None:
            x = (x * self.scale_per_element().double()).float().double()
        if zero is not None and self.spec.zero_point == "float":
            x = (x + zero.double()).float().double()
        if self.global_scale is not None:
            x = (x * self.global_scale.double()).float().double()
        return x.float().reshape(self.shape).to(dtype)

    def mma_operand(self) -> Operand:
        spec = self.spec
        if spec.mma_input == "dequant":
            from .quantize import round_to_format_triton

            source = self.dequantize().reshape(self.rows, self.K)
            if source.is_cuda:
                values = round_to_format_triton(source, spec.dequant_format, "rne", saturate=False)
            else:
                raise ValueError("the B200 backend builds MMA operands on CUDA tensors only")
            return Operand(values, spec.dequant_format)
        if self.scale is None:
            return Operand(self.values.float(), spec.format)
        scale, kind, width = self.scale, spec.granularity, 0
        if kind == "group":
            kind, width = "k", spec.group_size
        elif kind == "block":
            kind, width = "k", spec.block[1]
            scale = scale.repeat_interleave(spec.block[0], dim=0)[: self.rows]
        return Operand(self.values.float(), spec.format, scale, spec.scale.format, kind, width,
                       self.global_scale)


def qtensor_class(spec):
    """TriCast's QTensor for TriCast specs, this module's QTensor otherwise."""
    if type(spec).__module__.startswith("tricast."):
        from tricast.quant.qtensor import QTensor as TriCastQTensor

        return TriCastQTensor
    return QTensor


def operand_class(like):
    if type(like).__module__.startswith("tricast."):
        from tricast.mma.operand import Operand as TriCastOperand

        return TriCastOperand
    return Operand


def as_operand(x, *, compact: bool = False):
    """A tensor, QTensor or Operand viewed as an MMA operand (``tricast/mma/api.py:19-60``)."""
    from .formats import format_of_dtype

    if isinstance(x, Operand) or type(x).__name__ == "Operand":
        return x
    if isinstance(x, torch.Tensor):
        if x.ndim == 0:
            raise ValueError("an MMA input needs at least one dimension")
        fmt = format_of_dtype(x.dtype)
        dtype = container_dtype(fmt) if compact else torch.float32
        return Operand(x.reshape(math.prod(x.shape[:-1]), x.shape[-1]).to(dtype), fmt)
    spec = x.spec
    if spec.mma_input == "dequant":
        dq = x.mma_operand()
        dtype = container_dtype(spec.dequant_format) if compact else torch.float32
        return Operand(dq.values.reshape(math.prod(x.shape[:-1]), x.shape[-1]).to(dtype), spec.dequant_format)
    values = x.values.to(container_dtype(spec.format) if compact else torch.float32)
    if x.scale is None:
        return Operand(values, spec.format, alpha=x.global_scale)
    scale = x.scale.to(torch.float32)
    kind, domain = spec.granularity, 0
    if kind == "group":
        kind, domain = "k", spec.group_size
    elif kind == "block":
        kind, domain = "k", spec.block[1]
        scale = scale.repeat_interleave(spec.block[0], dim=0)[: values.shape[0]]
    return Operand(values, spec.format, scale, spec.scale.format, kind, domain, x.global_scale)
