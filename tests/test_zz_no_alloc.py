"""tc_gemm_noalloc: the GEMM entry point for callers that cannot allocate device memory.

Some hosts reach this library only through a plain C FFI and own no CUDA allocator, or reserve all
device memory up front, so they cannot pass tc_gemm a workspace. tc_gemm_noalloc takes its scratch
from a fixed array inside the library instead. These tests call it through the C ABI and require
its results to equal tc_gemm's bit for bit (the tolerance of every GEMM test here), on consecutive
calls that reuse the shared scratch. The file sorts last so that a run stopping at the first failure
has already run every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import pytest
import torch

from tests.conftest import bits_equal
from tricast_b200 import _native as N
from tricast_b200 import as_operand, gemm_triton, quantize_triton
from tricast_b200.mma import _Prepared, exact_fallbacks, mma_spec_struct, resolve_scale_apply
from tricast_b200.spec import PRESETS, SCHEMES, MMASpec

pytestmark = pytest.mark.gpu


def _operand(scheme, rows, k, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, k, generator=g) * scale
    return as_operand(quantize_triton(x.bfloat16().cuda(), SCHEMES[scheme]))


def _noalloc(a, b, spec, bias=None):
    """Direct C-ABI call of tc_gemm_noalloc (no workspace argument)."""
    pa, pb = _Prepared(a), _Prepared(b)
    ms = mma_spec_struct(spec, resolve_scale_apply(spec, a, b))
    from tricast_b200.formats import container_dtype

    dev = a.values.device
    with torch.cuda.device(dev):  # the fixed scratch array used is the current device's
        out = torch.empty((a.rows, b.rows), device=dev, dtype=container_dtype(spec.out_format))
        bias_t = None if bias is None else bias.float().contiguous()
        N.check(N.lib().tc_gemm_noalloc(pa.desc, pb.desc, ms, N.ptr(bias_t), N.ptr(out), N.stream_of(dev)),
                "tc_gemm_noalloc")
    return out


def _launches(fn):
    """(result, kernels the library launched for it, exact fallbacks it caused)."""
    torch.cuda.synchronize()
    l0, f0 = N.lib().tc_launch_count(), exact_fallbacks()
    out = fn()
    torch.cuda.synchronize()
    return out, N.lib().tc_launch_count() - l0, exact_fallbacks() - f0


def test_noalloc_equals_tc_gemm_on_consecutive_calls():
    spec = PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32")
    cases = [(_operand("nvfp4", 192, 1024, 1), _operand("nvfp4", 320, 1024, 2, 0.02)),
             (_operand("mxfp4", 130, 1040, 3), _operand("mxfp4", 65, 1040, 4)),
             (_operand("nvfp4", 192, 1024, 1), _operand("nvfp4", 320, 1024, 2, 0.02))]
    for a, b in cases:
        first, n_first, fb_first = _launches(lambda: _noalloc(a, b, spec))
        second = _noalloc(a, b, spec)  # the scratch now holds this call's own leftovers
        want, n_want, _ = _launches(lambda: gemm_triton(a, b, spec))
        assert bits_equal(first.cpu().numpy(), want.cpu().numpy())
        assert bits_equal(second.cpu().numpy(), want.cpu().numpy())
        # The same fast kernels ran on the fixed array (tc_gemm's launch count, no exact fallback).
        assert fb_first == 0 and n_first == n_want


def test_noalloc_fp64_and_fp32_fma_take_the_fast_kernel():
    """fp64 / fp32_fma need no scratch at all; they still run tc_gemm's FMA-chain kernel, not the
    generic exact one."""
    a, b = _operand("nvfp4", 96, 512, 11), _operand("nvfp4", 80, 512, 12, 0.02)
    for spec in (MMASpec("fp64", out_format="fp32"), MMASpec("fp32_fma", out_format="fp32")):
        want, n_want, _ = _launches(lambda: gemm_triton(a, b, spec))
        for _ in range(2):
            got, n_got, fb = _launches(lambda: _noalloc(a, b, spec))
            assert bits_equal(got.cpu().numpy(), want.cpu().numpy())
            assert fb == 0 and n_got == n_want == 1


def test_noalloc_without_fast_path_and_with_bias():
    a, b = _operand("fp8_tensor", 40, 256, 5), _operand("fp8_tensor", 24, 256, 6, 0.02)
    spec = PRESETS["nvidia_hopper_fp8"].with_(out_format="bf16")
    bias = torch.randn(24, generator=torch.Generator().manual_seed(7)).cuda()
    for _ in range(2):
        got = _noalloc(a, b, spec, bias)
        assert bits_equal(got.float().cpu().numpy(), gemm_triton(a, b, spec, bias).float().cpu().numpy())


def test_noalloc_rejects_operands_beyond_the_fixed_scratch():
    a, b = _operand("nvfp4", 8192, 2048, 8), _operand("nvfp4", 8192, 2048, 9)
    spec = PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32")
    with pytest.raises(ValueError, match="fixed 33554432-byte array"):
        _noalloc(a, b, spec)
