"""CPU checks of the host-side mirror of TriCast's interface: format vocabulary, specs, scale
policy resolution and validation messages (TriCast ``tests/test_mma_invariants.py`` /
``tests/test_golden.py`` style), and the registration shim."""

from __future__ import annotations

import sys
from types import SimpleNamespace

import pytest
import torch

from tricast_b200 import formats as F
from tricast_b200.mma import check_headroom, resolve_scale_apply
from tricast_b200.quantize import layout
from tricast_b200.spec import PRESETS, SCHEMES, MMASpec, QuantSpec, ScaleSpec, get_scheme


def test_format_grids():
    assert F.FP8_E4M3.max_normal == 448 and F.FP8_E4M3.emin == -6
    assert F.FP4_E2M1.max_normal == 6 and F.FP4_E2M1.min_subnormal == 0.5
    assert F.UE4M3.max_normal == 448 and not F.UE4M3.signed
    assert F.E8M0.emin == -127 and F.E8M0.emax == 127
    assert F.INT4.qmin == -7 and F.INT4.qmax == 7 and F.UINT4.qmax == 15
    assert F.get_format("int8:full").qmin == -128
    assert F.get_format("e3m4:nosub").subnormals is False
    assert F.get_format("e5m0:bias=20").kind == "pow2"
    with pytest.raises(ValueError):
        F.get_format("e9m2")
    assert F.container_dtype(F.FP4_E2M1) == torch.bfloat16
    assert F.container_dtype(F.FP16) == torch.float16
    assert F.container_dtype(F.FP32) == torch.float32
    assert F.container_dtype(F.get_format("int24")) == torch.float32


def test_specs_match_reference_registry():
    ref = pytest.importorskip("tricast.quant.spec") if "tricast" in sys.modules else None
    assert set(PRESETS) == {"nvidia_ada_fp8", "nvidia_hopper_fp8", "nvidia_blackwell_fp8", "nvidia_blackwell_fp4",
                            "deepseek_fp8_promote128", "fp32_fma", "fp64", "int_exact"}
    assert SCHEMES["nvfp4"].scale.two_level and SCHEMES["mxfp4"].scale.method == "pow2_floor"
    assert get_scheme("bfp8_b16").group_size == 16
    del ref


def test_spec_validation_messages():
    with pytest.raises(ValueError, match="zero points need an integer element format"):
        QuantSpec("fp8", "group", group_size=8, zero_point="int", mma_input="dequant")
    with pytest.raises(ValueError, match="promote_interval must be a multiple"):
        MMASpec(promote_interval=48, chunk_size=32)
    with pytest.raises(ValueError, match="groups per tile"):
        MMASpec("gdfs", group_size=4, k_tile=64)
    with pytest.raises(ValueError, match="power-of-two scale format"):
        ScaleSpec("e8m0", "absmax")


def _op(kind, K=64, kd=0, fmt=F.FP8_E4M3, scale_fmt=None):
    return SimpleNamespace(scale_kind=kind, K=K, k_domain=kd, fmt=fmt, scale_fmt=scale_fmt)


def test_resolve_scale_apply():
    assert resolve_scale_apply(PRESETS["nvidia_hopper_fp8"], _op("tensor"), _op("tensor")) == "epilogue"
    assert resolve_scale_apply(PRESETS["nvidia_blackwell_fp4"], _op("k", kd=16), _op("k", kd=16)) == "group"
    assert resolve_scale_apply(PRESETS["nvidia_hopper_fp8"], _op("k", kd=32), _op("none")) == "product"
    assert resolve_scale_apply(PRESETS["deepseek_fp8_promote128"], _op("k", K=256, kd=128), _op("none")) == "promote"
    with pytest.raises(ValueError, match="crosses K scale domain"):
        resolve_scale_apply(PRESETS["deepseek_fp8_promote128"], _op("k", K=256, kd=32), _op("none"))
    with pytest.raises(ValueError, match="cannot be applied in the epilogue"):
        resolve_scale_apply(PRESETS["int_exact"], _op("k", kd=32), _op("none"))


def test_scale_domain_crossing_matches_full_scan():
    """resolve_scale_apply decides domain crossings from one period of lcm(span, k_domain); the
    decision equals the reference's scan over every interval."""
    def full(K, span, kd):
        return any(s // kd != (min(s + span, K) - 1) // kd for s in range(0, K, span))

    for K in (1, 7, 16, 64, 100, 1000, 4096):
        for span in (1, 3, 16, 24, 32, 128):
            for kd in (1, 5, 16, 32, 48, 128):
                op = SimpleNamespace(scale_kind="k", K=K, k_domain=kd)
                spec = MMASpec("cofda", f_bits=13, chunk_size=1, promote_interval=span)
                try:
                    resolve_scale_apply(spec, op, SimpleNamespace(scale_kind="none"))
                    raised = False
                except ValueError:
                    raised = True
                assert raised == full(K, span, kd), (K, span, kd)


def test_headroom():
    int8 = F.INT8
    a = _op("none", fmt=int8)
    check_headroom(a, a, MMASpec("cofda", f_bits=23, chunk_size=32), "epilogue")
    with pytest.raises(ValueError, match="headroom"):
        check_headroom(a, a, MMASpec("cofda", f_bits=48, chunk_size=4096), "epilogue")


def test_layouts():
    assert layout(SCHEMES["mxfp4"], 3, 70) == (3, 3)
    assert layout(SCHEMES["fp8_tensor"], 3, 70) == ()
    assert layout(SCHEMES["int8_row"], 3, 70) == (3, 1)
    assert layout(SCHEMES["fp8_block128"], 300, 70) == (3, 1)


def test_install_shim_registers_backend_modules(monkeypatch):
    tricast = pytest.importorskip("tricast")  # TriCast itself is optional for this package
    from tricast_b200 import backend

    for name in ("tricast.kernels", "tricast.kernels.quantize", "tricast.kernels.mma"):
        monkeypatch.delitem(sys.modules, name, raising=False)
    pkg = backend.install()
    assert backend.installed()
    from tricast.kernels.mma import gemm_triton
    from tricast.kernels.quantize import quantize_triton, round_to_format_triton

    import tricast_b200

    assert quantize_triton is tricast_b200.quantize_triton
    assert round_to_format_triton is tricast_b200.round_to_format_triton
    assert gemm_triton is tricast_b200.gemm_triton
    from tricast.quant.api import resolve_backend

    assert resolve_backend("auto") == "reference"  # CPU tensors still use TriCast's reference
    assert pkg is tricast.kernels
