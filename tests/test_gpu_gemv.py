"""Bit-exact GPU parity of the small-M (decode) GEMM kernels (TriCast ``tests/gpu/test_triton_gemv.py``):
GDFS-FP4 and CoFDA-FP8 products with at most 16 rows of A, through the C ABI, against the oracle.
Covers every row count class (1, a few, a power of two, 16), ragged N and K (partial groups, tiles,
chunks and steps, K not a multiple of 16 so B rows lose their 16-byte alignment), bf16 and fp32
containers, promote intervals, wide (fp64) radices, and operands that force the exact fallback."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from tests.conftest import bits_equal, first_mismatch
from tricast_b200 import gemm_triton, quantize_triton
from tricast_b200.mma import exact_fallbacks
from tricast_b200.operand import Operand, as_operand
from tricast_b200.spec import PRESETS, SCHEMES, MMASpec

pytestmark = pytest.mark.gpu


def _quantized(scheme, rows, K, seed, scale=1.0, outliers=0, compact=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, K, generator=g) * scale
    if outliers:
        x[:, torch.randperm(K, generator=g)[:outliers]] *= 20
    return as_operand(quantize_triton(x.bfloat16().cuda(), SCHEMES[scheme]), compact=compact)


def _check(a: Operand, b: Operand, spec, label="", fast=True):
    """Bit-exact against the oracle; with ``fast`` the small-M kernel itself must have produced the
    result (the exact generic kernel behind it did not run)."""
    before = exact_fallbacks()
    got = gemm_triton(a, b, spec).float().cpu().numpy()
    ran_exact = exact_fallbacks() > before
    want = oracle.gemm_reference(a, b, spec)
    assert bits_equal(got, want), f"{label} {spec}: {first_mismatch(got, want)}"
    assert ran_exact != fast, f"{label} {spec}: exact fallback {'ran' if ran_exact else 'did not run'}"


FP4_SPECS = [
    PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32"),
    PRESETS["nvidia_blackwell_fp4"].with_(out_format="bf16", norm_rounding="rne"),
    PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32", k_tile=128),
    PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32", k_tile=16, f_bits=24),
]


@pytest.mark.parametrize("scheme", ["nvfp4", "mxfp4"])
@pytest.mark.parametrize("shape", [(1, 300, 1024), (3, 40, 520), (16, 130, 2048), (5, 1, 16), (2, 33, 7),
                                   (7, 64, 1001), (1, 17, 4096)])
@pytest.mark.parametrize("compact", [False, True])
def test_gdfs_fp4_gemv_vs_oracle(scheme, shape, compact):
    m, n, k = shape
    a = _quantized(scheme, m, k, 101, outliers=min(3, k), compact=compact)
    b = _quantized(scheme, n, k, 102, scale=0.02, compact=compact)
    for spec in FP4_SPECS:
        _check(a, b, spec, f"{scheme} {shape}")


@pytest.mark.parametrize("case", ["wide_tile_scales", "cancel_then_large", "tiny_running_nvfp4", "zero_rows"])
def test_gdfs_fp4_gemv_exact_fallback(case):
    """Tiles that fail the single-pass bounds (scale spreads, cancelling running values, subnormal
    running values, zero rows) take the exact per-output step inside the small-M kernel."""
    from tests.test_gpu_gemm import E2M1_GRID, _fp4_operand

    rng = np.random.default_rng(len(case) * 104729)
    M, N, K = 12, 40, 512
    kd, sfmt = (16, "ue4m3") if case == "tiny_running_nvfp4" else (32, "e8m0")
    va = E2M1_GRID[rng.integers(0, 8, (M, K))] * rng.choice([-1.0, 1.0], (M, K)).astype(np.float32)
    vb = E2M1_GRID[rng.integers(0, 8, (N, K))] * rng.choice([-1.0, 1.0], (N, K)).astype(np.float32)
    lim = 4 if sfmt == "e8m0" else 6
    ea = rng.integers(-lim, lim + 1, (M, K // kd))
    eb = rng.integers(-lim, lim + 1, (N, K // kd))
    if case == "wide_tile_scales":
        ea[::3] += rng.integers(-50, 51, ea[::3].shape)
    if case in ("cancel_then_large", "tiny_running_nvfp4"):
        vb[:, 64:128] = vb[:, 0:64]
        eb[:, 64 // kd:128 // kd] = eb[:, 0:64 // kd]
        va[::2, 64:128] = -va[::2, 0:64]
        ea[::2, 64 // kd:128 // kd] = ea[::2, 0:64 // kd]
        va[::4, 64 + 5] = np.where(va[::4, 64 + 5] == 0, 0.5, va[::4, 64 + 5])
        ea[:, 128 // kd:] += 20 if sfmt == "e8m0" else 6
    if case == "zero_rows":
        va[5] = 0.0
        vb[7, :256] = 0.0
    if sfmt == "e8m0":
        sa = np.exp2(np.clip(ea, -127, 127)).astype(np.float32)
        sb = np.exp2(np.clip(eb, -127, 127)).astype(np.float32)
    else:
        sa = ((8 + rng.integers(0, 8, ea.shape)) / 8.0 * np.exp2(np.clip(ea, -6, 7))).astype(np.float32)
        sb = ((8 + rng.integers(0, 8, eb.shape)) / 8.0 * np.exp2(np.clip(eb, -6, 7))).astype(np.float32)
    a, b = _fp4_operand(va, sa, sfmt, kd), _fp4_operand(vb, sb, sfmt, kd)
    for spec in FP4_SPECS[:2]:
        _check(a, b, spec, case)


def test_gdfs_fp4_gemv_flags():
    """Non-finite B values or scales (found inside the small-M kernel) and A values (found by its
    encoder) send the product to the exact generic kernel; zero-scale groups stay on the fast path."""
    spec = PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32")
    a = _quantized("nvfp4", 4, 256, 111)
    b = _quantized("nvfp4", 50, 256, 112, scale=0.02)
    bv = b.values.clone()
    bv[9, 40] = float("nan")
    _check(a, Operand(bv, b.fmt, b.scale, b.scale_fmt, b.scale_kind, b.k_domain, b.alpha), spec, "nan in B",
           fast=False)
    bv = b.values.clone()
    bv[3, 7] = float("-inf")
    _check(a, Operand(bv, b.fmt, b.scale, b.scale_fmt, b.scale_kind, b.k_domain, b.alpha), spec, "inf in B",
           fast=False)
    bs = b.scale.clone()
    bs[2, 1] = float("nan")
    _check(a, Operand(b.values, b.fmt, bs, b.scale_fmt, b.scale_kind, b.k_domain, b.alpha), spec, "nan B scale",
           fast=False)
    av = a.values.clone()
    av[1, 3] = float("inf")
    _check(Operand(av, a.fmt, a.scale, a.scale_fmt, a.scale_kind, a.k_domain, a.alpha), b, spec, "inf in A",
           fast=False)
    g = torch.Generator().manual_seed(113)
    x = torch.randn(3, 256, generator=g)
    x[1, 32:48] = 0
    _check(as_operand(quantize_triton(x.cuda(), SCHEMES["mxfp4"])), _quantized("mxfp4", 20, 256, 114), spec,
           "zero group")


COFDA_CASES = [
    ("nvidia_hopper_fp8", "fp8_tensor"), ("nvidia_ada_fp8", "fp8_tensor"), ("nvidia_hopper_fp8", "mxfp8_e4m3"),
    ("deepseek_fp8_promote128", "fp8_group128"), ("nvidia_hopper_fp8", "mxfp8_e5m2"),
    ("nvidia_blackwell_fp8", "fp8_tensor"), ("nvidia_blackwell_fp8", "mxfp8_e4m3"),
]


@pytest.mark.parametrize("preset,scheme", COFDA_CASES)
@pytest.mark.parametrize("shape", [(1, 300, 1024), (4, 33, 520), (5, 70, 1000), (16, 130, 2048), (2, 1, 5),
                                   (9, 64, 4096)])
def test_cofda_gemv_vs_oracle(preset, scheme, shape):
    m, n, k = shape
    if preset.startswith("deepseek") and k % 128:
        k = (k // 128 + 1) * 128
    a = _quantized(scheme, m, k, 121, outliers=min(3, k))
    b = _quantized(scheme, n, k, 122, scale=0.02, compact=True)
    for spec in (PRESETS[preset].with_(out_format="fp32"), PRESETS[preset].with_(norm_rounding="rne", f_bits=9),
                 PRESETS[preset].with_(chunk_size=8, out_format="bf16")):
        _check(a, b, spec, f"{scheme} {shape}")


def test_cofda_gemv_wide_radix_and_flags():
    a = _quantized("fp8_tensor", 6, 700, 131, outliers=5)
    b = _quantized("fp8_tensor", 45, 700, 132, scale=0.02)
    for spec in (MMASpec("cofda", f_bits=40, chunk_size=8, out_format="fp32", norm_rounding="rne"),
                 MMASpec("cofda", f_bits=30, chunk_size=16, out_format="bf16")):
        _check(a, b, spec, "wide")
    spec = PRESETS["nvidia_hopper_fp8"].with_(out_format="fp32")
    bv = b.values.clone()
    bv[4, 100] = float("inf")
    _check(a, Operand(bv, b.fmt, b.scale, b.scale_fmt, b.scale_kind, b.k_domain, b.alpha), spec, "inf in B",
           fast=False)
    av = a.values.clone()
    av[0, 1] = float("nan")
    _check(Operand(av, a.fmt, a.scale, a.scale_fmt, a.scale_kind, a.k_domain, a.alpha), b, spec, "nan in A",
           fast=False)
