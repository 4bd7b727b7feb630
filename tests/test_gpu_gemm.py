"""Bit-exact GPU parity of the emulated GEMM (TriCast ``tests/gpu/test_triton_mma.py``) against the
golden fixtures, all 1,716 NADPE vectors, and the oracle at larger sizes, through the C ABI."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from tests.conftest import bits_equal, first_mismatch
from tests.golden_cases import bf16_bits, load, mma_operand, mspec, nadpe_cases
from tricast_b200 import gemm_triton, quantize_triton
from tricast_b200.mma import exact_fallbacks
from tricast_b200.formats import FP16, IntFormat
from tricast_b200.operand import Operand, as_operand
from tricast_b200.spec import PRESETS, SCHEMES, MMASpec

pytestmark = pytest.mark.gpu


def _t(a):
    return None if a is None else torch.from_numpy(np.array(a, np.float32)).cuda()  # keeps 0-d shapes


def cuda_operand(ns) -> Operand:
    return Operand(_t(ns.values), ns.fmt, _t(ns.scale), ns.scale_fmt, ns.scale_kind, ns.k_domain,
                   None if ns.alpha is None else _t(np.asarray(ns.alpha, np.float32).reshape(())))


@pytest.mark.parametrize("case", load("mma")[0], ids=lambda c: c["id"])
def test_gemm_golden(case):
    _, arrays = load("mma")
    a, b = mma_operand(case, arrays, "a"), mma_operand(case, arrays, "b")
    spec = mspec(case["spec"])
    bias = arrays.get(f"{case['id']}|bias")
    if case["error"] is not None:
        with pytest.raises(ValueError):
            gemm_triton(cuda_operand(a), cuda_operand(b), spec, _t(bias))
        return
    got = gemm_triton(cuda_operand(a), cuda_operand(b), spec, _t(bias)).float().cpu().numpy()
    want = arrays[f"{case['id']}|out"]
    assert got.shape == want.shape
    assert bits_equal(got, want), f"{spec}: {first_mismatch(got, want)}"


def _nadpe_groups():
    cases = nadpe_cases()
    return [(k, [c for c in cases if c[0] == k]) for k in sorted({c[0] for c in cases})]


@pytest.mark.parametrize("key,cases", _nadpe_groups(), ids=lambda v: v if isinstance(v, str) else "")
def test_nadpe_vectors_gpu(key, cases):
    for _, index, a, b, spec, expected in cases:
        got = gemm_triton(cuda_operand(a), cuda_operand(b), spec)
        bits = got.contiguous().view(torch.int16).cpu().numpy()
        assert np.array_equal(bits, expected), f"{key} case {index}: {spec}"


def _quantized(scheme, rows, K, seed, scale=1.0, outliers=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, K, generator=g) * scale
    if outliers:
        x[:, torch.randperm(K, generator=g)[:outliers]] *= 20
    return as_operand(quantize_triton(x.bfloat16().cuda(), SCHEMES[scheme]))


def _oracle_gemm(a: Operand, b: Operand, spec):
    return oracle.gemm_reference(a, b, spec)


@pytest.mark.parametrize("scheme,preset", [
    ("nvfp4", "nvidia_blackwell_fp4"), ("mxfp4", "nvidia_blackwell_fp4"), ("fp8_tensor", "nvidia_hopper_fp8"),
    ("fp8_tensor", "nvidia_blackwell_fp8"), ("mxfp8_e4m3", "nvidia_hopper_fp8"), ("fp8_tensor", "nvidia_ada_fp8"),
])
@pytest.mark.parametrize("out", ["fp32", "bf16"])
def test_preset_configs_vs_oracle(scheme, preset, out):
    """Benchmark-config formats and presets at 64x96x1024 against the oracle."""
    a = _quantized(scheme, 64, 1024, 1, outliers=4)
    b = _quantized(scheme, 96, 1024, 2, scale=0.02)
    spec = PRESETS[preset].with_(out_format=out)
    before = exact_fallbacks()
    got = gemm_triton(a, b, spec).float().cpu().numpy()
    assert exact_fallbacks() == before, "the fast kernel declined benchmark-config operands"
    want = _oracle_gemm(a, b, spec)
    assert bits_equal(got, want), first_mismatch(got, want)


@pytest.mark.parametrize("compact", [False, True])
def test_cfg4_mapping_vs_oracle(compact):
    """INT8 row-scaled activations x INT4 g128 asymmetric weights, CoFDA F=23 promoted every 128; the
    activations also in bf16 containers, as the benchmark passes them."""
    g = torch.Generator().manual_seed(4)
    x = torch.randn(48, 1024, generator=g)
    w = torch.randn(80, 1024, generator=g) * 0.02
    qa = quantize_triton(x.cuda(), SCHEMES["int8_row"])
    qw = quantize_triton(w.cuda(), SCHEMES["int4_g128_zp"])
    z = qw.zero_point.repeat_interleave(128, dim=1)[:, :1024]
    a = as_operand(qa, compact=compact)
    b = Operand(qw.values.float() - z, IntFormat("int5", 5), qw.scale, FP16, "k", 128)
    spec = MMASpec("cofda", f_bits=23, chunk_size=32, promote_interval=128, out_format="fp32")
    got = gemm_triton(a, b, spec).cpu().numpy()
    want = _oracle_gemm(a, b, spec)
    assert bits_equal(got, want), first_mismatch(got, want)


def test_fp64_reference_gemm_vs_oracle():
    g = torch.Generator().manual_seed(5)
    a = as_operand(torch.randn(32, 1024, generator=g).bfloat16().cuda())
    b = as_operand((torch.randn(40, 1024, generator=g) * 0.02).bfloat16().cuda())
    spec = MMASpec("fp64", out_format="fp32")
    got = gemm_triton(a, b, spec).cpu().numpy()
    assert bits_equal(got, _oracle_gemm(a, b, spec))


def test_errors():
    a = Operand(torch.ones(2, 4, device="cuda"), IntFormat("int8", 8))
    b = Operand(torch.tensor([[float("nan"), 1, 1, 1]], device="cuda"), IntFormat("int8", 8))
    with pytest.raises(ValueError, match="finite"):
        gemm_triton(a, b, MMASpec("int_exact"))
    c = Operand(torch.ones(2, 5, device="cuda"), IntFormat("int8", 8))
    with pytest.raises(ValueError, match="same K"):
        gemm_triton(a, c, MMASpec("int_exact"))
    wide = MMASpec("cofda", f_bits=48, chunk_size=2 ** 14)
    with pytest.raises(ValueError, match="headroom"):
        gemm_triton(a, Operand(torch.ones(3, 4, device="cuda"), IntFormat("int8", 8)), wide)


@pytest.mark.parametrize("scheme", ["nvfp4", "mxfp4"])
@pytest.mark.parametrize("shape", [(37, 70, 200), (1, 1, 16), (130, 65, 1040), (64, 64, 64)])
def test_fp4_fast_path_ragged_shapes(scheme, shape):
    """The fast GDFS kernel with partial CTA tiles, partial K tiles and partial groups."""
    m, n, k = shape
    a = _quantized(scheme, m, k, 11, outliers=min(3, k))
    b = _quantized(scheme, n, k, 12, scale=0.02)
    for preset in (PRESETS["nvidia_blackwell_fp4"], PRESETS["nvidia_blackwell_fp4"].with_(g_bits=9, f_bits=13),
                   PRESETS["nvidia_blackwell_fp4"].with_(k_tile=128, norm_rounding="rne")):
        spec = preset.with_(out_format="fp32")
        got = gemm_triton(a, b, spec).cpu().numpy()
        want = _oracle_gemm(a, b, spec)
        assert bits_equal(got, want), f"{spec}: {first_mismatch(got, want)}"


def test_fp4_fast_path_falls_back_on_specials():
    """NaN operands and NaN / zero scales: the encoder flags them and the generic kernel runs."""
    g = torch.Generator().manual_seed(9)
    x = torch.randn(40, 256, generator=g)
    x[3, 17] = float("nan")
    a = as_operand(quantize_triton(x.cuda(), SCHEMES["nvfp4"]))
    b = _quantized("nvfp4", 50, 256, 10, scale=0.02)
    spec = PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32")
    got = gemm_triton(a, b, spec).cpu().numpy()
    assert bits_equal(got, _oracle_gemm(a, b, spec))
    # A zero scale group (all-zero block) stays on the fast path and must act as a zero term.
    x = torch.randn(40, 256, generator=g)
    x[5, 32:48] = 0
    a = as_operand(quantize_triton(x.cuda(), SCHEMES["mxfp4"]))
    b = _quantized("mxfp4", 50, 256, 13)
    got = gemm_triton(a, b, spec).cpu().numpy()
    assert bits_equal(got, _oracle_gemm(a, b, spec))


E2M1_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)


def _fp4_operand(values: np.ndarray, scales: np.ndarray, scale_fmt: str, kd: int) -> Operand:
    from tricast_b200.formats import get_format

    return Operand(torch.from_numpy(values).cuda(), get_format("fp4_e2m1"), torch.from_numpy(scales).cuda(),
                   get_format(scale_fmt), "k", kd)


@pytest.mark.parametrize("case", ["wide_tile_scales", "cancel_then_large", "tiny_running_nvfp4", "zero_rows"])
def test_fp4_single_pass_and_exact_fallback(case):
    """The fp64 single pass of the GDFS FP4 kernel and its exact two-pass fallback: K-tiles whose group
    scales span more than the radix allows, running values that cancel to (almost) nothing before far
    larger terms arrive (the reference truncates the running value then), and all-zero rows."""
    rng = np.random.default_rng(len(case) * 7919)
    M, N, K = 48, 40, 512
    kd, sfmt = (16, "ue4m3") if case == "tiny_running_nvfp4" else (32, "e8m0")
    va = E2M1_GRID[rng.integers(0, 8, (M, K))] * rng.choice([-1.0, 1.0], (M, K)).astype(np.float32)
    vb = E2M1_GRID[rng.integers(0, 8, (N, K))] * rng.choice([-1.0, 1.0], (N, K)).astype(np.float32)
    ga, gb = K // kd, K // kd
    if sfmt == "e8m0":
        ea = rng.integers(-4, 5, (M, ga))
        eb = rng.integers(-4, 5, (N, gb))
    else:
        ea = rng.integers(-6, 7, (M, ga))
        eb = rng.integers(-6, 7, (N, gb))
    if case == "wide_tile_scales":
        ea[::3] += rng.integers(-50, 51, ea[::3].shape)   # > 40 binades inside a 64-wide tile
    if case in ("cancel_then_large", "tiny_running_nvfp4"):
        # Tile 1 repeats tile 0 with the sign flipped on half the rows (B repeats too): the running
        # value returns to (almost) zero; a few elements of tile 1 differ by one grid step so that
        # some outputs keep a tiny remainder; later tiles carry far larger scales.
        vb[:, 64:128] = vb[:, 0:64]
        eb[:, 64 // kd:128 // kd] = eb[:, 0:64 // kd]
        va[::2, 64:128] = -va[::2, 0:64]
        ea[::2, 64 // kd:128 // kd] = ea[::2, 0:64 // kd]
        va[::4, 64 + 5] = np.where(va[::4, 64 + 5] == 0, 0.5, va[::4, 64 + 5])
        big = 20 if sfmt == "e8m0" else 6
        ea[:, 128 // kd:] += big
    if case == "zero_rows":
        va[5] = 0.0
        vb[7, :256] = 0.0
    if sfmt == "e8m0":
        sa = np.exp2(np.clip(ea, -127, 127)).astype(np.float32)
        sb = np.exp2(np.clip(eb, -127, 127)).astype(np.float32)
    else:  # UE4M3 grid: m/8 * 2**e with m in 8..15, e in [-6, 7] (max_normal 448)
        sa = ((8 + rng.integers(0, 8, ea.shape)) / 8.0 * np.exp2(np.clip(ea, -6, 7))).astype(np.float32)
        sb = ((8 + rng.integers(0, 8, eb.shape)) / 8.0 * np.exp2(np.clip(eb, -6, 7))).astype(np.float32)
    a, b = _fp4_operand(va, sa, sfmt, kd), _fp4_operand(vb, sb, sfmt, kd)
    for spec in (PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32"),
                 PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32", norm_rounding="rne")):
        got = gemm_triton(a, b, spec).cpu().numpy()
        want = _oracle_gemm(a, b, spec)
        assert bits_equal(got, want), f"{case} {spec.norm_rounding}: {first_mismatch(got, want)}"


@pytest.mark.parametrize("shape", [(37, 70, 200), (1, 1, 5), (130, 65, 1040), (64, 64, 8192)])
@pytest.mark.parametrize("preset,scheme", [
    ("nvidia_hopper_fp8", "fp8_tensor"), ("nvidia_ada_fp8", "fp8_tensor"), ("nvidia_hopper_fp8", "mxfp8_e4m3"),
    ("deepseek_fp8_promote128", "fp8_group128"), ("nvidia_hopper_fp8", "mxfp8_e5m2"),
    ("nvidia_blackwell_fp8", "fp8_tensor"), ("nvidia_blackwell_fp8", "mxfp8_e4m3"),
])
def test_cofda_fast_path_vs_oracle(shape, preset, scheme):
    """The fast CoFDA kernel (epilogue, pow2 product and promoted scales) on ragged shapes."""
    m, n, k = shape
    if preset.startswith("deepseek") and k % 128:
        k = (k // 128 + 1) * 128
    a = _quantized(scheme, m, k, 21, outliers=min(3, k))
    b = _quantized(scheme, n, k, 22, scale=0.02)
    for spec in (PRESETS[preset].with_(out_format="fp32"), PRESETS[preset].with_(norm_rounding="rne", f_bits=9)):
        before = exact_fallbacks()
        got = gemm_triton(a, b, spec).float().cpu().numpy()
        assert exact_fallbacks() == before, f"{spec}: the fast kernel declined finite on-grid operands"
        want = _oracle_gemm(a, b, spec)
        assert bits_equal(got, want), f"{spec}: {first_mismatch(got, want)}"


def test_cofda_wide_radix_fp64_path():
    """Radices beyond fp32's exact range (F + 2 + log2(CS + 1) > 24) take the fp64 CoFDA kernel."""
    a = _quantized("fp8_tensor", 70, 700, 41, outliers=5)
    b = _quantized("fp8_tensor", 45, 700, 42, scale=0.02)
    for spec in (MMASpec("cofda", f_bits=25, chunk_size=32, out_format="fp32"),
                 MMASpec("cofda", f_bits=40, chunk_size=8, out_format="fp32", norm_rounding="rne"),
                 MMASpec("cofda", f_bits=30, chunk_size=16, out_format="bf16")):
        got = gemm_triton(a, b, spec).float().cpu().numpy()
        want = _oracle_gemm(a, b, spec)
        assert bits_equal(got, want), f"{spec}: {first_mismatch(got, want)}"


def test_cofda_chunk8_and_fallback_on_nan():
    a = _quantized("fp8_tensor", 40, 300, 31)
    b = _quantized("fp8_tensor", 33, 300, 32, scale=0.02)
    spec = MMASpec("cofda", f_bits=13, chunk_size=8, out_format="fp32")
    assert bits_equal(gemm_triton(a, b, spec).cpu().numpy(), _oracle_gemm(a, b, spec))
    g = torch.Generator().manual_seed(33)
    x = torch.randn(40, 300, generator=g)
    x[7, 100] = float("inf")
    a = as_operand(quantize_triton(x.cuda(), SCHEMES["fp8_row"]))
    spec = PRESETS["nvidia_hopper_fp8"].with_(out_format="fp32")
    assert bits_equal(gemm_triton(a, b, spec).cpu().numpy(), _oracle_gemm(a, b, spec))


@pytest.mark.parametrize("shape", [(200, 150, 2048), (3, 129, 256)])
def test_int_promote_fast_path_vs_oracle(shape):
    """cfg4 mapping (INT8 row x INT5 (uint4 - zero point), F=23 promoted every 128) at larger sizes."""
    m, n, k = shape
    g = torch.Generator().manual_seed(40 + m)
    qa = quantize_triton(torch.randn(m, k, generator=g).cuda(), SCHEMES["int8_row"])
    qw = quantize_triton((torch.randn(n, k, generator=g) * 0.02).cuda(), SCHEMES["int4_g128_zp"])
    z = qw.zero_point.repeat_interleave(128, dim=1)[:, :k]
    a = as_operand(qa)
    b = Operand(qw.values.float() - z, IntFormat("int5", 5), qw.scale, FP16, "k", 128)
    spec = MMASpec("cofda", f_bits=23, chunk_size=32, promote_interval=128, out_format="fp32")
    got = gemm_triton(a, b, spec).cpu().numpy()
    assert bits_equal(got, _oracle_gemm(a, b, spec))
    # int_exact on int8 x int8 with row scales (the int8_row_w8a8 recipe's arithmetic)
    a8 = as_operand(qa)
    b8 = as_operand(quantize_triton(torch.randn(n, k, generator=g).cuda(), SCHEMES["int8_row"]))
    spec = MMASpec("int_exact", out_format="fp32")
    assert bits_equal(gemm_triton(a8, b8, spec).cpu().numpy(), _oracle_gemm(a8, b8, spec))


@pytest.mark.parametrize("scheme,preset", [("fp8_tensor", "nvidia_hopper_fp8"), ("fp8_tensor", "nvidia_blackwell_fp8"),
                                           ("mxfp8_e4m3", "nvidia_ada_fp8")])
def test_cofda_compact_bf16_operands(scheme, preset):
    """The tiled CoFDA kernel on operands in bf16 containers (as cfg3 passes them), fp32 and fp64
    accumulation, a ragged K: bit-exact against the oracle, produced by the fast kernel."""
    g = torch.Generator().manual_seed(7)
    xa = torch.randn(130, 1000, generator=g)
    xb = torch.randn(72, 1000, generator=g) * 0.02
    a = as_operand(quantize_triton(xa.bfloat16().cuda(), SCHEMES[scheme]), compact=True)
    b = as_operand(quantize_triton(xb.bfloat16().cuda(), SCHEMES[scheme]), compact=True)
    assert a.values.dtype == torch.bfloat16 and b.values.dtype == torch.bfloat16
    spec = PRESETS[preset].with_(out_format="fp32")
    before = exact_fallbacks()
    got = gemm_triton(a, b, spec).float().cpu().numpy()
    assert exact_fallbacks() == before, "the fast kernel declined compact on-grid operands"
    want = _oracle_gemm(a, b, spec)
    assert bits_equal(got, want), first_mismatch(got, want)


@pytest.mark.parametrize("scheme", ["nvfp4", "mxfp4"])
@pytest.mark.parametrize("shape", [(130, 64, 1024), (40, 200, 1000)])
def test_gdfs_fp4_compact_bf16_operands(scheme, shape):
    """Operands in bf16 containers (``as_operand(..., compact=True)``, as the benchmark passes them) on
    the tiled kernel: whole groups are encoded four elements at a time from their bit patterns, and a
    ragged K leaves the last group to the per-element path. Bit-exact against the oracle with the fast
    kernel producing the result; a NaN inside a bf16 group must hand the product to the exact kernel,
    which is bit-exact too."""
    m, n, k = shape
    g = torch.Generator().manual_seed(m + n + k)
    xa = torch.randn(m, k, generator=g)
    xa[:, torch.randperm(k, generator=g)[:4]] *= 20
    xb = torch.randn(n, k, generator=g) * 0.02
    a = as_operand(quantize_triton(xa.bfloat16().cuda(), SCHEMES[scheme]), compact=True)
    b = as_operand(quantize_triton(xb.bfloat16().cuda(), SCHEMES[scheme]), compact=True)
    assert a.values.dtype == torch.bfloat16 and b.values.dtype == torch.bfloat16
    spec = PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32")
    before = exact_fallbacks()
    got = gemm_triton(a, b, spec).float().cpu().numpy()
    assert exact_fallbacks() == before, "the fast kernel declined compact on-grid operands"
    want = _oracle_gemm(a, b, spec)
    assert bits_equal(got, want), first_mismatch(got, want)
    b.values[7, 37] = float("nan")
    before = exact_fallbacks()
    got = gemm_triton(a, b, spec).float().cpu().numpy()
    assert exact_fallbacks() > before, "a NaN element did not reach the exact kernel"
    want = _oracle_gemm(a, b, spec)
    assert bits_equal(got, want), first_mismatch(got, want)


@pytest.mark.parametrize("rows", [40, 3])  # tiled kernel and small-M kernel
def test_cofda_tiny_folded_scales(rows):
    """Power-of-two product scales that fold into tiny values: labels down to -50 stay on the fast
    kernels (exact scale powers, a chunk of zero products with a tiny running value), lower ones go
    to the exact kernel."""
    a = _quantized("mxfp8_e4m3", rows, 512, 51)
    b = _quantized("mxfp8_e4m3", 33, 512, 52, scale=0.02)
    spec = PRESETS["nvidia_hopper_fp8"].with_(out_format="fp32")
    for exp_a, exp_b, fast in ((-40, -3, True), (-44, -40, True), (-58, 0, False)):
        sa = torch.full_like(a.scale, 2.0 ** exp_a)
        sb = torch.full_like(b.scale, 2.0 ** exp_b)
        sb[:, 3] = 2.0 ** -127  # E8M0 code 0, a zero scale: a chunk of zero products after the first
        ta = Operand(a.values, a.fmt, sa, a.scale_fmt, a.scale_kind, a.k_domain, a.alpha)
        tb = Operand(b.values, b.fmt, sb, b.scale_fmt, b.scale_kind, b.k_domain, b.alpha)
        before = exact_fallbacks()
        got = gemm_triton(ta, tb, spec).cpu().numpy()
        assert (exact_fallbacks() == before) == fast, (exp_a, exp_b)
        want = _oracle_gemm(ta, tb, spec)
        assert bits_equal(got, want), f"{exp_a} {exp_b}: {first_mismatch(got, want)}"


@pytest.mark.parametrize("rows", [40, 3])  # tiled kernel and small-M kernel
@pytest.mark.parametrize("f_bits,f2_bits,chunk", [(13, 23, 32), (13, 13, 16), (21, 35, 8), (25, 48, 32), (9, 5, 32)])
def test_cofda_decoupled_fast_path(rows, f_bits, f2_bits, chunk):
    """Decoupled CoFDA: each chunk normalised at F from zero, then merged into the running value at
    F2, on the fast kernels (fp32 or fp64 chunk sums, fp64 merge)."""
    a = _quantized("fp8_tensor", rows, 1000, 61, outliers=5)
    b = _quantized("fp8_tensor", 37, 1000, 62, scale=0.02)
    for spec in (MMASpec("cofda", f_bits=f_bits, chunk_size=chunk, c_mode="decoupled", f2_bits=f2_bits,
                         out_format="fp32"),
                 MMASpec("cofda", f_bits=f_bits, chunk_size=chunk, c_mode="decoupled", f2_bits=f2_bits,
                         out_format="bf16", norm_rounding="rne")):
        before = exact_fallbacks()
        got = gemm_triton(a, b, spec).float().cpu().numpy()
        assert exact_fallbacks() == before, f"{spec}: the fast kernel declined the operands"
        want = _oracle_gemm(a, b, spec)
        assert bits_equal(got, want), f"{spec}: {first_mismatch(got, want)}"
    mx_a = _quantized("mxfp8_e4m3", rows, 512, 63)
    mx_b = _quantized("mxfp8_e4m3", 29, 512, 64, scale=0.02)
    spec = MMASpec("cofda", f_bits=f_bits, chunk_size=chunk, c_mode="decoupled", f2_bits=f2_bits, out_format="fp32")
    got = gemm_triton(mx_a, mx_b, spec).cpu().numpy()
    assert bits_equal(got, _oracle_gemm(mx_a, mx_b, spec))


@pytest.mark.parametrize("shape", [(130, 260, 384), (1, 1, 128), (128, 128, 128), (257, 129, 1000)])
def test_int_tensor_core_path(shape):
    """Integer operands on the tcgen05 kind::i8 kernel: promoted CoFDA intervals (INT8 row-scaled x
    INT5 with FP16 K scales per 128) and int_exact, ragged tiles and spans, bit-exact and without the
    exact fallback."""
    m, n, k = shape
    g = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(m, k, generator=g)
    w = torch.randn(n, k, generator=g) * 0.02
    qa = quantize_triton(x.cuda(), SCHEMES["int8_row"])
    qw = quantize_triton(w.cuda(), SCHEMES["int4_g128_zp"])
    z = qw.zero_point.repeat_interleave(128, dim=1)[:, :k]
    a = as_operand(qa)
    b = Operand(qw.values.float() - z, IntFormat("int5", 5), qw.scale, FP16, "k", 128)
    spec = MMASpec("cofda", f_bits=23, chunk_size=32, promote_interval=128, out_format="fp32")
    before = exact_fallbacks()
    got = gemm_triton(a, b, spec).cpu().numpy()
    assert exact_fallbacks() == before, "the tensor-core kernel declined or timed out"
    want = _oracle_gemm(a, b, spec)
    assert bits_equal(got, want), first_mismatch(got, want)
    ia = Operand(qa.values.float(), IntFormat("int8", 8))
    ib = Operand(qw.values.float() - z, IntFormat("int5", 5))
    spec = MMASpec("int_exact", out_format="fp32")
    before = exact_fallbacks()
    got = gemm_triton(ia, ib, spec).cpu().numpy()
    assert exact_fallbacks() == before, "the tensor-core kernel declined or timed out"
    want = _oracle_gemm(ia, ib, spec)
    assert bits_equal(got, want), first_mismatch(got, want)


# ---------------------------------------------------------------- GDFS on narrow float grids
GDFS_NARROW = [
    # TriCast's own benchmark row (scripts/bench/bench_mma_vs_nadpe.py:31-32)
    dict(f_bits=25, g_bits=32, group_size=16, k_tile=32),
    dict(f_bits=25, g_bits=32, group_size=16, k_tile=64),
    dict(f_bits=23, g_bits=10, group_size=16, k_tile=16),
    dict(f_bits=13, g_bits=8, group_size=8, k_tile=32),       # precision below fp32's: F < 23
    dict(f_bits=35, g_bits=24, group_size=32, k_tile=64, norm_rounding="rne"),
]


@pytest.mark.parametrize("kw", GDFS_NARROW, ids=lambda kw: "-".join(f"{k[0]}{v}" for k, v in kw.items()))
@pytest.mark.parametrize("scheme,shape", [("fp8_tensor", (70, 50, 160)), ("fp8_row", (33, 65, 96)),
                                          ("mxfp8_e4m3", (64, 64, 256)), ("mxfp8_e5m2", (40, 72, 128))])
def test_gdfs_narrow_kernel_matches_oracle(kw, scheme, shape):
    """The fast GDFS kernel for narrow float grids (tc_gemm_gdfs.cu) on FP8 E4M3 / E5M2 operands with
    tensor, row and E8M0 group scales, ragged shapes and K tails, bit for bit with the oracle, and
    without falling back to the exact generic kernel."""
    if scheme not in SCHEMES:
        pytest.skip(f"{scheme} is not a registered scheme")
    m, n, k = shape
    spec = MMASpec("gdfs", out_format="fp32", **kw)
    if scheme == "mxfp8_e4m3" and kw["group_size"] > 32:
        pytest.skip("a GDFS group may not cross a 32-wide E8M0 scale domain")
    a = _quantized(scheme, m, k, 1, outliers=3)
    b = _quantized(scheme, n, k, 2, scale=0.02)
    before = exact_fallbacks()
    got = gemm_triton(a, b, spec).cpu().numpy()
    assert exact_fallbacks() == before, "the fast GDFS kernel declined finite on-grid operands"
    want = _oracle_gemm(a, b, spec)
    assert bits_equal(got, want), f"{spec}: {first_mismatch(got, want)}"


def test_gdfs_narrow_kernel_cancelling_groups():
    """A group whose aligned sum cancels to exactly zero takes no part in the tile's FDA. Here the
    third group of 16 (k 32..47) has the largest products but pairs every product with its negation,
    so it sets the tile's provisional exponent and then drops out: those outputs redo their tile step
    with the exponent of the remaining terms."""
    g = torch.Generator().manual_seed(3)

    def fp8(x):
        return x.to(torch.float8_e4m3fn).float()

    m, n = 8, 16
    a = fp8(torch.randn(m, 64, generator=g) * 2)
    b = fp8(torch.randn(n, 64, generator=g) * 2)
    half_a = fp8(torch.randn(m, 8, generator=g) * 64)
    half_b = fp8(torch.randn(n, 8, generator=g) * 64)
    a[:, 32:48] = torch.cat([half_a, half_a], dim=1)
    b[:, 32:48] = torch.cat([half_b, -half_b], dim=1)
    b[:, 48:64] *= 0.01  # the group that remains after the cancellation is small
    b = fp8(b)
    from tricast_b200.formats import FP32, get_format

    one = torch.ones((), device="cuda")
    opa = Operand(a.cuda(), get_format("fp8_e4m3"), one, FP32, "tensor")
    opb = Operand(b.cuda(), get_format("fp8_e4m3"), one, FP32, "tensor")
    for kt in (32, 64):
        spec = MMASpec("gdfs", f_bits=25, g_bits=32, group_size=16, k_tile=kt, out_format="fp32")
        before = exact_fallbacks()
        got = gemm_triton(opa, opb, spec).cpu().numpy()
        assert exact_fallbacks() == before
        want = _oracle_gemm(opa, opb, spec)
        assert bits_equal(got, want), f"k_tile={kt}: {first_mismatch(got, want)}"


def test_gdfs_narrow_kernel_wide_label_spread():
    """Groups whose products span more than G - ma - mb binades truncate their smallest products at
    radix G, so the kernel's exact-sum shortcut must not take them: rows and columns mixing the
    largest E4M3 magnitudes with subnormals (labels 8 and -9 on each side), next to ordinary rows in
    the same warps, bit for bit with the oracle for G = 32 (span 26) and G = 20 (span 14)."""
    g = torch.Generator().manual_seed(11)

    def fp8(x):
        return x.to(torch.float8_e4m3fn).float()

    m, n, k = 40, 48, 128
    a = fp8(torch.randn(m, k, generator=g) * 2)
    b = fp8(torch.randn(n, k, generator=g) * 2)
    for r in range(0, m, 5):
        a[r, r % 16::16] = 448.0
        a[r, (r + 3) % 16::16] = 2.0 ** -9
    for c in range(0, n, 7):
        b[c, (c + 1) % 16::16] = -448.0
        b[c, (c + 5) % 16::16] = 2.0 ** -8
    from tricast_b200.formats import FP32, get_format

    one = torch.ones((), device="cuda")
    opa = Operand(a.cuda(), get_format("fp8_e4m3"), one, FP32, "tensor")
    opb = Operand(b.cuda(), get_format("fp8_e4m3"), one, FP32, "tensor")
    for g_bits in (32, 20):
        spec = MMASpec("gdfs", f_bits=25, g_bits=g_bits, group_size=16, k_tile=32, out_format="fp32")
        before = exact_fallbacks()
        got = gemm_triton(opa, opb, spec).cpu().numpy()
        assert exact_fallbacks() == before
        want = _oracle_gemm(opa, opb, spec)
        assert bits_equal(got, want), f"g_bits={g_bits}: {first_mismatch(got, want)}"


@pytest.mark.parametrize("m,n,k", [(3, 2, 0), (40, 70, 0), (0, 6, 64), (5, 0, 64)])
@pytest.mark.parametrize("fmt,spec", [
    ("fp8_e4m3", MMASpec("cofda", f_bits=13, chunk_size=32, out_format="fp32")),
    ("fp8_e4m3", MMASpec("gdfs", f_bits=25, g_bits=32, group_size=16, k_tile=32, out_format="fp32")),
    ("fp4_e2m1", MMASpec("gdfs", f_bits=35, g_bits=6, group_size=16, k_tile=64, out_format="bf16")),
    ("fp8_e4m3", MMASpec("fp64", out_format="fp32")),
    ("fp8_e4m3", MMASpec("fp32_fma", out_format="fp32")),
    ("int8", MMASpec("int_exact", out_format="fp32")),
], ids=lambda x: getattr(x, "algorithm", x))
def test_empty_shapes(m, n, k, fmt, spec):
    """Empty products as TriCast's reference treats them: no rows or columns give an empty output, and
    K = 0 gives each output the epilogue of a zero sum (the bias here)."""
    from tricast_b200.formats import FP32, get_format

    f = get_format(fmt)
    one = torch.ones((), device="cuda")
    a = Operand(torch.zeros(m, k, device="cuda"), f, one, FP32, "tensor")
    b = Operand(torch.zeros(n, k, device="cuda"), f, one, FP32, "tensor")
    bias = torch.linspace(-2, 3, n, device="cuda") if n else None
    got = gemm_triton(a, b, spec, bias=bias)
    assert tuple(got.shape) == (m, n)
    want = oracle.gemm_reference(a, b, spec, bias=bias)
    assert bits_equal(got.float().cpu().numpy(), np.asarray(want).reshape(m, n))
