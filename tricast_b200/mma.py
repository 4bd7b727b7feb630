"""Emulated GEMM on the B200 library: the drop-in replacement of TriCast's ``tricast.kernels.mma``
module (``src/tricast/kernels/mma.py:821-886``).

``gemm_triton(a, b, spec, bias)`` keeps TriCast's name, operand contract (``Operand`` values
[rows, K] on their format grid, scale layouts none/tensor/row/k, alpha) and error messages. Operand
values are read in whatever float container they arrive in (fp32, bf16 or fp16): no fp32 K-major
copy is made.
"""

from __future__ import annotations

import ctypes as C
import math

import torch

from . import _native as N
from .formats import FP32, container_dtype, get_format


def _integer_bits(fmt) -> int:
    """Integer bits of a format's significand (``reference/mma.py:171-174``)."""
    if fmt.kind == "int":
        return max(abs(fmt.qmin), fmt.qmax).bit_length() + max(0, -fmt.frac_bits)
    return 1


def resolve_scale_apply(spec, a, b) -> str:
    """Where K-varying scales enter the arithmetic (``reference/mma.py:184-202``)."""
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
        # An interval starting at s crosses a domain boundary iff the one starting at s + lcm(span,
        # k_domain) does (same offset inside its domain, never longer), so the first period decides.
        stop = min(op.K, span * op.k_domain // math.gcd(span, op.k_domain)) if span else 0
        if span and any(start // op.k_domain != (min(start + span, op.K) - 1) // op.k_domain
                        for start in range(0, stop, span)):
            raise ValueError(f"{mode} interval/group size {span} crosses K scale domain {op.k_domain}")
    return mode


def check_headroom(a, b, spec, apply: str) -> None:
    """int64 headroom of every aligned sum (``kernels/mma.py:744-765``, ``reference/mma.py:177-181``)."""
    def check(radix: int, integer_bits: int, width: int) -> None:
        if radix + integer_bits + width.bit_length() > 62:
            raise ValueError("MMA aligned sum exceeds int64 headroom (F + int_bits + ceil(log2(n+1)) > 62)")

    ib = _integer_bits(a.fmt) + _integer_bits(b.fmt)
    sb = sum(_integer_bits(op.scale_fmt or FP32) for op in (a, b)
             if op.scale_kind == "k" and getattr(op.scale_fmt, "kind", "float") != "pow2")
    if spec.algorithm == "cofda":
        check(spec.f_bits, ib + (sb if apply == "product" else 0), spec.chunk_size)
        if spec.c_mode == "decoupled" and not spec.promote_interval:
            check(spec.f2_bits, 1, 1)
    elif spec.algorithm == "gdfs":
        check(spec.g_bits, ib, spec.group_size)
        check(spec.f_bits, ib + (spec.group_size - 1).bit_length() + (sb if apply == "group" else 0),
              spec.groups_per_tile)
    elif spec.algorithm == "int_exact":
        if a.fmt.kind != "int" or b.fmt.kind != "int":
            raise ValueError("int_exact requires integer operands")
        check(0, ib, a.K)


def _validate_operand(op) -> None:
    """TriCast ``_validate_operand`` (``kernels/mma.py:801-818``)."""
    if not op.values.is_cuda or not op.values.is_floating_point():
        raise ValueError("gemm_triton requires floating CUDA grid-value tensors")
    if op.scale_kind not in ("none", "tensor", "row", "k"):
        raise ValueError(f"unknown scale_kind {op.scale_kind!r}")
    if op.scale is not None:
        shape = {"tensor": (), "row": (op.rows, 1),
                 "k": (op.rows, -(-op.K // max(op.k_domain, 1)))}[op.scale_kind]
        if tuple(op.scale.shape) != shape:
            raise ValueError(f"scale shape must be {shape}, got {tuple(op.scale.shape)}")
        if op.scale.device != op.values.device:
            raise ValueError("scale and values must be on the same CUDA device")
    if op.alpha is not None and (op.alpha.numel() != 1 or op.alpha.device != op.values.device):
        raise ValueError("alpha must be a scalar on the operand device")


class _Prepared:
    """An operand's tensors in the layouts the C ABI reads, kept alive for the call."""

    def __init__(self, op):
        v = op.values
        if v.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            v = v.to(torch.float32)
        self.values = v.contiguous()
        self.scale = None if op.scale is None else op.scale.to(torch.float32).contiguous()
        self.alpha = None if op.alpha is None else op.alpha.to(torch.float32).reshape(()).contiguous()
        d = N.TcOperand()
        d.values, d.values_dtype = self.values.data_ptr(), N.dtype_code(self.values.dtype)
        d.rows, d.K = op.rows, op.K
        d.fmt = N.tc_format(op.fmt)
        d.scale = 0 if self.scale is None else self.scale.data_ptr()
        d.scale_kind = N.SCALE_KIND_CODES[op.scale_kind]
        if op.scale_kind == "k" and op.scale_fmt is not None:
            d.has_scale_fmt, d.scale_fmt = 1, N.tc_format(op.scale_fmt)
        d.k_domain = int(op.k_domain or 0)
        d.alpha = 0 if self.alpha is None else self.alpha.data_ptr()
        self.desc = d


def mma_spec_struct(spec, apply: str) -> N.TcMmaSpec:
    s = N.TcMmaSpec()
    s.algorithm = N.ALGORITHM_CODES[spec.algorithm]
    s.f_bits, s.chunk_size = spec.f_bits, spec.chunk_size
    s.c_mode = 1 if spec.c_mode == "decoupled" else 0
    s.f2_bits, s.g_bits, s.group_size, s.k_tile = spec.f2_bits, spec.g_bits, spec.group_size, spec.k_tile
    s.norm_rounding = 1 if spec.norm_rounding == "rne" else 0
    s.scale_apply = N.APPLY_CODES[apply]
    s.promote_interval = spec.promote_interval
    s.out_format = N.tc_format(spec.out_format)
    s.out_dtype = N.dtype_code(container_dtype(spec.out_format))
    return s


def _any_nonfinite(values: torch.Tensor) -> bool:
    flag = torch.zeros((), dtype=torch.int32, device=values.device)
    N.check(N.lib().tc_any_nonfinite(N.ptr(values), N.dtype_code(values.dtype), values.numel(), N.ptr(flag),
                                     N.stream_of(values.device)), "tc_any_nonfinite")
    return bool(flag.item())


def gemm_triton(a, b, spec, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``a @ b.T`` under ``spec``'s accumulation rule, bit-exact with TriCast's reference backend."""
    if a.K != b.K or a.values.device != b.values.device:
        raise ValueError("operands must have the same K and CUDA device")
    _validate_operand(a)
    _validate_operand(b)
    apply = resolve_scale_apply(spec, a, b)
    dtype = container_dtype(spec.out_format)
    if spec.algorithm == "int_exact" and (a.scale_kind == "k" or b.scale_kind == "k"):
        raise ValueError("int_exact does not support K-varying scales")
    check_headroom(a, b, spec, apply)
    if bias is not None and (tuple(bias.shape) != (b.rows,) or bias.device != a.values.device):
        raise ValueError("bias must have shape [N] on the operand device")
    device = a.values.device
    out = torch.empty((a.rows, b.rows), device=device, dtype=dtype)
    pa, pb = _Prepared(a), _Prepared(b)
    if spec.algorithm == "int_exact" and (_any_nonfinite(pa.values) or _any_nonfinite(pb.values)):
        raise ValueError("int_exact requires finite integer operands")
    if a.rows == 0 or b.rows == 0:
        return out
    bias_t = None if bias is None else bias.to(torch.float32).contiguous()
    ms = mma_spec_struct(spec, apply)
    lib = N.lib()
    with torch.cuda.device(device):
        ws_bytes = lib.tc_gemm_workspace(pa.desc, pb.desc, ms)
        ws = torch.empty(max(ws_bytes, 1), device=device, dtype=torch.uint8)
        enc = _encoded_b(a, b, spec, apply, pa, pb, ms)
        if enc is None:
            N.check(lib.tc_gemm(pa.desc, pb.desc, ms, N.ptr(bias_t), N.ptr(out), N.ptr(ws), ws.numel(),
                                N.stream_of(device)), "tc_gemm")
        else:
            N.check(lib.tc_gemm_encoded(pa.desc, pb.desc, N.ptr(enc), enc.numel(), ms, N.ptr(bias_t), N.ptr(out),
                                        N.ptr(ws), ws.numel(), N.stream_of(device)), "tc_gemm_encoded")
    return out


def _tensor_state(t) -> tuple | None:
    """What an encoding derived from ``t`` depends on: which tensor, its storage, its layout and its
    in-place version counter (TriCast's ``mma/operand.py:21-26`` rule; edits through ``.data`` or
    inside ``torch.inference_mode`` are not versioned, as there)."""
    if t is None:
        return None
    version = None if t.is_inference() else t._version
    return id(t), t.data_ptr(), tuple(t.shape), t.stride(), version


def _encoded_b(a, b, spec, apply, pa, pb, ms):
    """The fast path's encoding of ``b``, kept on the operand object between calls the way TriCast
    keeps a weight operand's K-major copy (``mma/operand.py:66-75``): encoded on first use for this
    spec and kind of A, reused while B's tensors are unchanged. None when the pair's fast path takes
    no pre-encoded B (or the object cannot hold a cache), in which case tc_gemm encodes per call."""
    cache = getattr(b, "__dict__", None)
    if cache is None:
        return None
    encodings = cache.setdefault("_tc_b_encodings", {})
    # What B's encoding depends on besides B: the C-level spec (scale application included) and the
    # kind of A (more or fewer than 17 rows, its format and K-scale layout).
    d = pa.desc
    key = (bytes(ms), a.rows > 16, bytes(d.fmt), d.scale_kind, d.has_scale_fmt, bytes(d.scale_fmt), d.k_domain)
    state = (_tensor_state(b.values), _tensor_state(b.scale), _tensor_state(b.alpha))
    hit = encodings.get(key)
    if hit is not None and hit[0] == state:
        return hit[1]
    lib = N.lib()
    nbytes = lib.tc_encode_b_bytes(pa.desc, pb.desc, ms)
    enc = None
    if nbytes:
        enc = torch.empty(nbytes, device=b.values.device, dtype=torch.uint8)
        N.check(lib.tc_encode_b(pa.desc, pb.desc, ms, N.ptr(enc), nbytes, N.stream_of(b.values.device)),
                "tc_encode_b")
    encodings[key] = (state, enc)
    return enc


def exact_fallbacks(device=None) -> int:
    """How many times, on ``device``, the exact generic kernel queued behind a fast GEMM kernel has run
    because the fast kernel declined its operands (non-finite or off-grid values, scales it cannot
    fold) or a bounded wait ran out. Synchronises the device."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    count = C.c_uint64(0)
    with torch.cuda.device(device):
        N.check(N.lib().tc_exact_fallbacks(C.byref(count)), "tc_exact_fallbacks")
    return int(count.value)


def _device_counter(name: str, device) -> int:
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    count = C.c_uint64(0)
    with torch.cuda.device(device):
        N.check(getattr(N.lib(), name)(C.byref(count)), name)
    return int(count.value)


def wait_timeouts(device=None) -> int:
    """Of the exact-kernel runs counted by :func:`exact_fallbacks`, those that followed a fast kernel
    whose bounded wait ran out. Synchronises the device."""
    return _device_counter("tc_wait_timeouts", device)


def exact_tile_steps(device=None) -> int:
    """(output, K tile) steps of the tensor-core GDFS-FP4 kernel that failed the single-pass bounds and
    took the exact two-pass step. Synchronises the device."""
    return _device_counter("tc_exact_tile_steps", device)


def gemm(a, b, spec, *, bias: torch.Tensor | None = None) -> torch.Tensor:
    """TriCast ``gemm`` on CUDA operands (``mma/api.py:63-109``): activations [..., K] × weights [N, K]."""
    from .operand import Operand, as_operand
    from .spec import mma_spec_from

    spec = mma_spec_from(spec)
    a_op, b_op = as_operand(a), as_operand(b)
    a_shape = a.values.shape if isinstance(a, Operand) else a.shape
    b_shape = b.values.shape if isinstance(b, Operand) else b.shape
    if len(b_shape) != 2:
        raise ValueError("MMA weights must have shape [N, K]")
    if a_op.K != b_op.K:
        raise ValueError("MMA operands must have the same reduction dimension K")
    out = gemm_triton(a_op, b_op, spec, bias)
    return out.reshape(*a_shape[:-1], b_op.rows)


__all__ = ["gemm_triton", "gemm", "exact_fallbacks", "wait_timeouts", "exact_tile_steps", "resolve_scale_apply", "check_headroom", "get_format"]
