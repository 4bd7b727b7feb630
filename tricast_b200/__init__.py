"""tricast_b200 — a B200-native (sm_100a) backend for TriCast's emulation hot path.

Public surface (TriCast's GPU backend API, ``src/tricast/kernels``):

* ``round_to_format_triton(x, fmt, rounding, *, saturate, noise, sr_bits)`` — casts;
* ``quantize_triton(x, spec, *, amax, noise, seed, scale_noise)`` — quantization to a QTensor;
* ``gemm_triton(a, b, spec, bias)`` — the emulated MMA/GEMM of every TriCast accumulation model;
* ``metrics.ErrorStats`` — per-layer MSE/SQNR/cosine sums;
* ``install()`` — register this package as TriCast's GPU backend module (``tricast.kernels``), so
  ``tricast.quantize``/``tricast.gemm`` with ``backend="auto"`` or ``"triton"``, recipes,
  ``patch_model``, the CLI and the app run on it unchanged.

All compute runs in ``_lib/libtricast_b200.so`` (C ABI: ``include/tricast_b200.h``); importing this
package does not load it until the first call.
"""

from . import formats, rounding, spec  # noqa: F401
from .formats import get_format  # noqa: F401
from .mma import gemm, gemm_triton  # noqa: F401
from .operand import Operand, QTensor, as_operand  # noqa: F401
from .quantize import QuantizePlan, quantize, quantize_into, quantize_triton, round_to_format_triton  # noqa: F401
from .spec import PRESETS, SCHEMES, MMASpec, QuantSpec, ScaleSpec, get_preset, get_scheme  # noqa: F401

__version__ = "0.1.0"


def install():
    """Register as TriCast's ``tricast.kernels`` backend (see ``backend.install``)."""
    from .backend import install as _install

    return _install()
