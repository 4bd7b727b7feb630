"""Bit-exact GPU parity of casts and quantization against the golden fixtures and the oracle
(the case matrix of TriCast ``tests/gpu/test_triton_quantize.py``), through the C ABI."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from oracle.quantize import dequantize as oracle_dequantize
from oracle.quantize import quantize_reference as oracle_quantize
from tests.conftest import bits_equal, first_mismatch
from tests.golden_cases import load, qspec
from tricast_b200 import quantize_into, quantize_triton, round_to_format_triton
from tricast_b200.formats import REGISTRY, container_dtype, get_format
from tricast_b200.spec import SCHEMES, QuantSpec, ScaleSpec

pytestmark = pytest.mark.gpu


def _cast_entries():
    meta, _ = load("cast")
    return [m for m in meta if "sr_bits" not in m]


@pytest.mark.parametrize("entry", _cast_entries(), ids=lambda m: m["key"])
def test_cast_golden(entry):
    _, arrays = load("cast")
    fmt = get_format(entry["format"])
    key = entry["key"]
    x = torch.from_numpy(arrays[f"x|{key}"]).cuda()
    noise = torch.from_numpy(arrays[f"noise|{key}"].astype(np.int64)).cuda()
    for r in ("rne", "rna", "rtz", "rup", "rdn", "sr"):
        for sat in (0, 1):
            name = f"y|{key}|{r}|{sat}"
            if name not in arrays:
                with pytest.raises(ValueError, match="stochastic rounding"):
                    round_to_format_triton(x, fmt, r, saturate=bool(sat), noise=noise)
                continue
            got = round_to_format_triton(x, fmt, r, saturate=bool(sat), noise=noise).cpu().numpy()
            assert bits_equal(got, arrays[name]), f"{key} {r} sat={sat}: {first_mismatch(got, arrays[name])}"


def test_cast_sr_bits_golden():
    meta, arrays = load("cast")
    for entry in (m for m in meta if "sr_bits" in m):
        _, name, bits = entry["key"].split("|")
        x = torch.from_numpy(arrays[f"srx|{name}|{bits}"]).cuda()
        noise = torch.from_numpy(arrays[f"srn|{name}|{bits}"].astype(np.int64)).cuda()
        got = round_to_format_triton(x, get_format(entry["format"]), "sr", noise=noise, sr_bits=int(bits))
        assert bits_equal(got.cpu().numpy(), arrays[f"sry|{name}|{bits}"]), entry["key"]


@pytest.mark.parametrize("fmt", list(REGISTRY.values()), ids=list(REGISTRY))
def test_cast_random_vs_oracle(fmt):
    """Wide random bit patterns with random noise, checked against the CPU oracle."""
    g = np.random.default_rng(7)
    bits = g.integers(0, 2 ** 32, 200_003, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    noise = g.integers(0, 2 ** 32, x.shape, dtype=np.uint64).astype(np.int64)
    for r in ("rne", "rtz", "rup", "sr"):
        if fmt.kind == "pow2" and r == "sr":
            continue
        want = oracle.round_to_format(x, fmt, r, saturate=False, noise=noise)
        got = round_to_format_triton(torch.from_numpy(x).cuda(), fmt, r, saturate=False,
                                     noise=torch.from_numpy(noise).cuda()).cpu().numpy()
        assert bits_equal(got, want), f"{fmt.name} {r}: {first_mismatch(got, want)}"


def _assert_qtensor(actual, case, arrays):
    cid = case["id"]
    for field in ("values", "scale", "zero_point", "global_scale"):
        want = arrays.get(f"{cid}|{field}")
        value = getattr(actual, field)
        if want is None:
            assert value is None, field
            continue
        assert value is not None, field
        assert tuple(value.shape) == want.shape, (field, tuple(value.shape), want.shape)
        got = value.float().cpu().numpy()
        assert bits_equal(got, want), f"{field}: {first_mismatch(got, want)}"


def _quantize_cases():
    meta, _ = load("quantize")
    return meta


@pytest.mark.parametrize("case", _quantize_cases(), ids=lambda c: c["id"])
def test_quantize_golden(case):
    _, arrays = load("quantize")
    cid = case["id"]
    spec = qspec(case["spec"])
    x = torch.from_numpy(arrays[f"{cid}|x"]).cuda()
    kwargs = {}
    if f"{cid}|noise" in arrays:
        kwargs["noise"] = torch.from_numpy(arrays[f"{cid}|noise"].astype(np.int64)).cuda()
    if f"{cid}|scale_noise" in arrays:
        kwargs["scale_noise"] = torch.from_numpy(arrays[f"{cid}|scale_noise"].astype(np.int64)).cuda()
    if case["amax"] is not None:
        kwargs["amax"] = torch.tensor(case["amax"], dtype=torch.float32).cuda()
    q, extras = quantize_into(x, spec, want_dequant=True, **kwargs)
    _assert_qtensor(q, case, arrays)
    assert q.values.dtype == container_dtype(spec.format)
    assert bits_equal(extras.dequant.reshape(x.shape).cpu().numpy(), arrays[f"{cid}|dequant"])


@pytest.mark.parametrize("name", ["mxfp4", "nvfp4", "mxfp8_e4m3", "fp8_tensor", "int4_g128_zp", "int8_row",
                                  "mxint8", "kivi4", "fp8_block128"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_quantize_random_vs_oracle(name, dtype):
    """Larger random tensors (both the fused group pass and the general pass) against the oracle."""
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(96, 512, generator=g) * 3).to(dtype)
    x.view(-1)[torch.randperm(x.numel(), generator=g)[:50]] *= 40
    spec = SCHEMES[name]
    want = oracle_quantize(x.float().numpy(), spec)
    got, extras = quantize_into(x.cuda(), spec, want_dequant=True)
    for field in ("values", "scale", "zero_point", "global_scale"):
        w, v = getattr(want, field), getattr(got, field)
        assert (w is None) == (v is None), field
        if w is not None:
            assert bits_equal(v.float().cpu().numpy(), np.asarray(w)), f"{field}: {first_mismatch(v.float().cpu().numpy(), w)}"
    assert bits_equal(extras.dequant.cpu().numpy(), oracle_dequantize(want))


E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
                       np.float32)


def test_mxfp4_codes_decode_to_values():
    """Packed E2M1 nibbles (low nibble = even element) and E8M0 bytes decode to the QTensor fields."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(64, 1024, generator=g)
    q, ex = quantize_into(x.cuda(), SCHEMES["mxfp4"], want_codes=True, want_scale_codes=True, want_dequant=True)
    codes = ex.codes.cpu().numpy()
    lo, hi = codes & 0xF, codes >> 4
    nib = np.stack((lo, hi), axis=1).reshape(-1)
    assert bits_equal(E2M1_VALUES[nib], q.values.float().cpu().numpy().reshape(-1))
    sc = ex.scale_codes.cpu().numpy().astype(np.int64)
    assert np.array_equal(np.ldexp(1.0, sc - 127).astype(np.float32), q.scale.cpu().numpy())


def test_nvfp4_scale_codes_are_ue4m3():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(32, 256, generator=g)
    q, ex = quantize_into(x.cuda(), SCHEMES["nvfp4"], want_scale_codes=True)
    decoded = torch.from_numpy(ex.scale_codes.cpu().numpy()).view(torch.float8_e4m3fn).float().numpy()
    assert bits_equal(decoded, q.scale.cpu().numpy())


def test_cfg1_full_size_vs_oracle():
    """The benchmark workload (4096x4096 MXFP4, 0.1% x50 outliers, seed 0) against the oracle."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, 4096, generator=g)
    idx = torch.randperm(4096 * 4096, generator=g)[:16777]
    x.view(-1)[idx] *= 50
    want = oracle_quantize(x.numpy(), SCHEMES["mxfp4"])
    got, ex = quantize_into(x.cuda(), SCHEMES["mxfp4"], want_dequant=True, want_codes=True)
    assert bits_equal(got.values.float().cpu().numpy(), want.values)
    assert bits_equal(got.scale.cpu().numpy(), want.scale)
    assert bits_equal(ex.dequant.cpu().numpy(), oracle_dequantize(want))


def test_errors_match_reference_messages():
    x = torch.ones(4, 4, device="cuda")
    with pytest.raises(ValueError, match="nonempty"):
        quantize_triton(torch.ones(0, 4, device="cuda"), SCHEMES["mxfp4"])
    with pytest.raises(ValueError, match="amax override requires tensor granularity"):
        quantize_triton(x, SCHEMES["mxfp4"], amax=torch.tensor(1.0, device="cuda"))
    spec = QuantSpec("fp4", "row", scale=ScaleSpec("fp16", rounding="sr"))
    with pytest.raises(ValueError, match="scale_noise"):
        quantize_triton(x, spec)
    with pytest.raises(ValueError, match="stochastic rounding"):
        round_to_format_triton(x, "e8m0", "sr", noise=torch.zeros(4, 4, dtype=torch.int64, device="cuda"))
    with pytest.raises(ValueError, match="CUDA"):
        round_to_format_triton(torch.ones(3), "fp8")


def test_seeded_sr_is_repeatable():
    spec = SCHEMES["mxfp4"].with_(rounding="sr")
    x = torch.linspace(-1.5, 1.5, 1024, device="cuda")
    a = quantize_triton(x, spec, seed=42)
    b = quantize_triton(x, spec, seed=42)
    c = quantize_triton(x, spec, seed=43)
    assert torch.equal(a.values, b.values)
    assert not torch.equal(a.values, c.values)


def test_noncontiguous_and_amax_override():
    g = torch.Generator().manual_seed(42)
    x = torch.randn((7, 3), generator=g).cuda().T
    amax = torch.tensor(8.0, device="cuda")
    got = quantize_triton(x, SCHEMES["fp8_tensor"], amax=amax)
    want = oracle_quantize(x.cpu().numpy(), SCHEMES["fp8_tensor"], amax=np.float32(8.0))
    assert bits_equal(got.values.float().cpu().numpy(), want.values)
    assert bits_equal(got.scale.cpu().numpy(), want.scale)


@pytest.mark.parametrize("name", ["mxfp4", "nvfp4", "fp8_tensor", "int8_row", "int4_g128_zp"])
def test_extras_without_values_match(name):
    """Skipping the QTensor values leaves every other output unchanged (all dispatch paths)."""
    g = torch.Generator().manual_seed(21)
    x = torch.randn(64, 256, generator=g).cuda()
    want_codes = name in ("mxfp4", "nvfp4", "fp8_tensor", "int8_row")
    q1, e1 = quantize_into(x, SCHEMES[name], want_dequant=True, want_codes=want_codes)
    q2, e2 = quantize_into(x, SCHEMES[name], want_dequant=True, want_codes=want_codes, want_values=False)
    assert q2.values is None
    assert torch.equal(q1.scale, q2.scale)
    assert bits_equal(e1.dequant.cpu().numpy(), e2.dequant.cpu().numpy())
    if want_codes:
        assert torch.equal(e1.codes, e2.codes)
