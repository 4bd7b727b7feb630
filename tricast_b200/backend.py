"""Registration shim: serve TriCast's GPU backend slot without Triton.

TriCast's dispatchers pick their GPU backend by importing ``tricast.kernels`` (``quant/api.py:26-30``)
and then call ``tricast.kernels.quantize.quantize_triton`` / ``round_to_format_triton``
(``quant/api.py:50``) and ``tricast.kernels.mma.gemm_triton`` (``mma/api.py:94``). ``install()``
places modules with exactly those names and functions in ``sys.modules``, backed by this package,
so every caller above the API — ``tricast.quantize``, ``tricast.gemm``, ``fake_quant``,
``EmuLinear``/``patch_model`` with ``backend: auto`` or ``triton``, the CLI and the app — runs on the
B200 library with no edit to TriCast. The backend string stays ``"triton"``/``"auto"`` because
TriCast's schema and validators hard-code that enum.
"""

from __future__ import annotations

import sys
import types


def install():
    """Install the shim modules; returns the ``tricast.kernels`` module. Needs TriCast importable."""
    import tricast  # noqa: F401  (the host package must exist)

    from .mma import gemm_triton, resolve_scale_apply
    from .quantize import quantize_triton, round_to_format_triton

    pkg = types.ModuleType("tricast.kernels")
    pkg.__path__ = []
    pkg.__doc__ = "TriCast GPU backend served by tricast_b200 (sm_100a CUDA, no Triton)."
    qmod = types.ModuleType("tricast.kernels.quantize")
    qmod.round_to_format_triton = round_to_format_triton
    qmod.quantize_triton = quantize_triton
    mmod = types.ModuleType("tricast.kernels.mma")
    mmod.gemm_triton = gemm_triton
    mmod.resolve_scale_apply = resolve_scale_apply
    pkg.quantize, pkg.mma = qmod, mmod
    sys.modules["tricast.kernels"] = pkg
    sys.modules["tricast.kernels.quantize"] = qmod
    sys.modules["tricast.kernels.mma"] = mmod
    import tricast as host

    host.kernels = pkg
    return pkg


def installed() -> bool:
    mod = sys.modules.get("tricast.kernels")
    return mod is not None and getattr(getattr(mod, "quantize", None), "quantize_triton", None) is not None and \
        "tricast_b200" in (mod.__doc__ or "")
