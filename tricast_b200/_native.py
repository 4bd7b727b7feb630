"""ctypes binding of the C ABI in ``include/tricast_b200.h`` (library ``_lib/libtricast_b200.so``).

Structures below mirror the header field for field. The library is the only compute path: if it
cannot be loaded the import fails; there is no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

from .formats import get_format
from .rounding import rounding_code

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtricast_b200.so"

TC_OK, TC_INVALID_ARGUMENT, TC_UNSUPPORTED, TC_CUDA_ERROR, TC_WORKSPACE_TOO_SMALL, TC_NONFINITE = range(6)
TC_F32, TC_BF16, TC_F16 = 0, 1, 2
SPECIAL_CODES = {"ieee": 0, "fn": 1, "fnuz": 2, "none": 3}
GRANULARITY_CODES = {"tensor": 0, "row": 1, "group": 2, "block": 3}
METHOD_CODES = {"absmax": 0, "pow2_floor": 1, "pow2_ceil": 2, "mse": 3, "percentile": 4}
ZERO_POINT_CODES = {"none": 0, "int": 1, "float": 2}
ALGORITHM_CODES = {"cofda": 0, "gdfs": 1, "fp32_fma": 2, "fp64": 3, "int_exact": 4}
APPLY_CODES = {"epilogue": 0, "product": 1, "group": 2, "promote": 3, "operand": 4}
SCALE_KIND_CODES = {"none": 0, "tensor": 1, "row": 2, "k": 3}


class TcFormat(C.Structure):
    _fields_ = [("kind", C.c_int32), ("ebits", C.c_int32), ("mbits", C.c_int32), ("bias", C.c_int32),
                ("special", C.c_int32), ("is_signed", C.c_int32), ("subnormals", C.c_int32),
                ("bits", C.c_int32), ("symmetric", C.c_int32), ("frac_bits", C.c_int32)]


class TcQuantSpec(C.Structure):
    _fields_ = [("format", TcFormat), ("granularity", C.c_int32), ("group_size", C.c_int32),
                ("block_rows", C.c_int32), ("block_cols", C.c_int32), ("has_scale", C.c_int32),
                ("scale_format", TcFormat), ("scale_method", C.c_int32), ("scale_rounding", C.c_int32),
                ("two_level", C.c_int32), ("zero_point", C.c_int32), ("rounding", C.c_int32),
                ("sr_bits", C.c_int32), ("saturate", C.c_int32), ("percentile", C.c_float),
                ("n_search", C.c_int32), ("mse_search", C.POINTER(C.c_float))]


class TcQuantOut(C.Structure):
    _fields_ = [("values", C.c_void_p), ("values_dtype", C.c_int32), ("scale", C.c_void_p),
                ("zero_point", C.c_void_p), ("global_scale", C.c_void_p), ("codes", C.c_void_p),
                ("scale_codes", C.c_void_p), ("dequant", C.c_void_p)]


class TcOperand(C.Structure):
    _fields_ = [("values", C.c_void_p), ("values_dtype", C.c_int32), ("rows", C.c_int64), ("K", C.c_int64),
                ("fmt", TcFormat), ("scale", C.c_void_p), ("scale_kind", C.c_int32), ("has_scale_fmt", C.c_int32),
                ("scale_fmt", TcFormat), ("k_domain", C.c_int32), ("alpha", C.c_void_p)]


class TcMmaSpec(C.Structure):
    _fields_ = [("algorithm", C.c_int32), ("f_bits", C.c_int32), ("chunk_size", C.c_int32), ("c_mode", C.c_int32),
                ("f2_bits", C.c_int32), ("g_bits", C.c_int32), ("group_size", C.c_int32), ("k_tile", C.c_int32),
                ("norm_rounding", C.c_int32), ("scale_apply", C.c_int32), ("promote_interval", C.c_int32),
                ("out_format", TcFormat), ("out_dtype", C.c_int32)]


EXPORTS = {
    "tc_cast": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.POINTER(TcFormat), C.c_int32, C.c_int32,
                          C.c_int32, C.c_void_p]),
    "tc_quantize_workspace": (C.c_size_t, [C.c_int64, C.c_int64, C.POINTER(TcQuantSpec)]),
    "tc_quantize": (C.c_int, [C.c_void_p, C.c_int32, C.c_int64, C.c_int64, C.POINTER(TcQuantSpec), C.c_void_p,
                              C.c_void_p, C.c_void_p, C.POINTER(TcQuantOut), C.c_void_p, C.c_size_t, C.c_void_p]),
    "tc_gemm_workspace": (C.c_size_t, [C.POINTER(TcOperand), C.POINTER(TcOperand), C.POINTER(TcMmaSpec)]),
    "tc_gemm": (C.c_int, [C.POINTER(TcOperand), C.POINTER(TcOperand), C.POINTER(TcMmaSpec), C.c_void_p, C.c_void_p,
                          C.c_void_p, C.c_size_t, C.c_void_p]),
    "tc_encode_b_bytes": (C.c_size_t, [C.POINTER(TcOperand), C.POINTER(TcOperand), C.POINTER(TcMmaSpec)]),
    "tc_encode_b": (C.c_int, [C.POINTER(TcOperand), C.POINTER(TcOperand), C.POINTER(TcMmaSpec), C.c_void_p, C.c_size_t,
                              C.c_void_p]),
    "tc_gemm_encoded": (C.c_int, [C.POINTER(TcOperand), C.POINTER(TcOperand), C.c_void_p, C.c_size_t,
                                  C.POINTER(TcMmaSpec), C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "tc_gemm_noalloc": (C.c_int, [C.POINTER(TcOperand), C.POINTER(TcOperand), C.POINTER(TcMmaSpec), C.c_void_p,
                                  C.c_void_p, C.c_void_p]),
    "tc_any_nonfinite": (C.c_int, [C.c_void_p, C.c_int32, C.c_int64, C.c_void_p, C.c_void_p]),
    "tc_error_stats": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_int64, C.c_void_p, C.c_void_p]),
    "tc_last_error": (C.c_char_p, []),
    "tc_version": (C.c_char_p, []),
    "tc_launch_count": (C.c_uint64, []),
    "tc_exact_fallbacks": (C.c_int, [C.POINTER(C.c_uint64)]),
    "tc_wait_timeouts": (C.c_int, [C.POINTER(C.c_uint64)]),
    "tc_tensor_amax_bits": (C.c_int, [C.c_void_p, C.c_int32, C.c_int64, C.c_void_p, C.c_void_p]),
    "tc_exact_tile_steps": (C.c_int, [C.POINTER(C.c_uint64)]),
    "tc_set_wait_limit": (C.c_int, [C.c_int32]),
    "tc_probe_mma_fp8": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int32, C.c_void_p,
                                   C.c_void_p, C.c_void_p]),
    "tc_probe_mma_fp4": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                   C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
}

_lib = None
_lock = threading.Lock()


def lib():
    """The loaded library (built first if the in-tree .so is missing or older than its sources)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                from . import build as _build

                try:
                    if _build.stale():
                        _build.build()
                except Exception as exc:  # the .so might still exist and be usable
                    if not LIB_PATH.exists():
                        raise ImportError(f"tricast_b200: cannot build {LIB_PATH}: {exc}") from exc
                handle = C.CDLL(str(LIB_PATH))
                for name, (res, args) in EXPORTS.items():
                    fn = getattr(handle, name)
                    fn.restype, fn.argtypes = res, args
                _lib = handle
    return _lib


class NativeError(RuntimeError):
    pass


def check(status: int, what: str) -> None:
    if status == TC_OK:
        return
    msg = lib().tc_last_error().decode()
    if status == TC_INVALID_ARGUMENT:
        raise ValueError(msg or what)
    if status == TC_UNSUPPORTED:
        raise NotImplementedError(msg or what)
    raise NativeError(f"{what}: {msg} (status {status})")


def tc_format(fmt) -> TcFormat:
    f = get_format(fmt)
    out = TcFormat()
    if f.kind == "float":
        out.kind, out.ebits, out.mbits, out.bias = 0, f.ebits, f.mbits, f.bias
        out.special, out.is_signed, out.subnormals = SPECIAL_CODES[f.special], int(f.signed), int(f.subnormals)
    elif f.kind == "int":
        out.kind, out.bits, out.is_signed = 1, f.bits, int(f.signed)
        out.symmetric, out.frac_bits = int(f.symmetric), f.frac_bits
    else:
        out.kind, out.ebits, out.bias = 2, f.ebits, f.bias
    return out


def dtype_code(dtype) -> int:
    import torch

    codes = {torch.float32: TC_F32, torch.bfloat16: TC_BF16, torch.float16: TC_F16}
    if dtype not in codes:
        raise ValueError(f"unsupported tensor dtype {dtype} (fp32, bf16 or fp16)")
    return codes[dtype]


def stream_of(device) -> C.c_void_p:
    import torch

    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr(t) -> C.c_void_p:
    return C.c_void_p(0 if t is None else t.data_ptr())


__all__ = ["lib", "check", "tc_format", "rounding_code", "dtype_code", "stream_of", "ptr"]
