"""Group-quantize stress against the oracle over the whole matrix the streaming kernels dispatch on:
float element formats (narrow, ieee / fn / none specials, plus fnuz and no-subnormal formats that
take the generic pass), every element rounding, saturating and not, absmax / pow2_floor / pow2_ceil /
two-level scales in several scale formats, group sizes 8..128, fp32 and bf16 inputs. Values span
fp32's whole exponent range per group (subnormal results, clamped and overflowing scales) and some
groups hold zeros, signed zeros, Inf and NaN. Values, scales, global scale, dequant and the element
and scale codes are all compared bit for bit."""

from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

from oracle.quantize import dequantize as oracle_dequantize
from oracle.quantize import quantize_reference as oracle_quantize
from tests.conftest import bits_equal, first_mismatch
from tricast_b200 import quantize_into
from tricast_b200.formats import get_format
from tricast_b200.spec import QuantSpec, ScaleSpec

pytestmark = pytest.mark.gpu

ELEMENTS = ["fp4_e2m1", "fp6_e2m3", "fp6_e3m2", "fp8_e4m3", "fp8_e5m2", "e4m3:ieee", "e3m4", "fp16",
            "fp8_e4m3fnuz", "e4m3:nosub"]
SCALES = {
    "e8m0_floor": lambda: ScaleSpec("e8m0", "pow2_floor"),
    "e8m0_ceil": lambda: ScaleSpec("e8m0", "pow2_ceil"),
    "fp32_absmax": lambda: ScaleSpec("fp32", "absmax"),
    "ue4m3_two_level": lambda: ScaleSpec("ue4m3", "absmax", two_level=True),
    "bf16_absmax_rtz": lambda: ScaleSpec("bf16", "absmax", rounding="rtz"),
    "fp32_pow2_ceil": lambda: ScaleSpec("fp32", "pow2_ceil"),
}
ROUNDINGS = ["rne", "rtz", "rup", "rdn", "rna"]


def code_table(fmt) -> np.ndarray:
    """Value of every code of a <= 8-bit float format (sign | exponent field | fraction)."""
    e, m = fmt.ebits, fmt.mbits
    n = 1 << (e + m + (1 if fmt.signed else 0))
    out = np.empty(n, np.float64)
    top = (1 << e) - 1
    for c in range(n):
        neg = fmt.signed and (c >> (e + m)) & 1
        field, frac = (c >> m) & top, c & ((1 << m) - 1)
        if fmt.special == "fnuz" and c == 1 << (e + m):
            v, neg = np.nan, False
        elif fmt.special == "ieee" and field == top:
            v = np.inf if frac == 0 else np.nan
        elif fmt.special == "fn" and field == top and frac == (1 << m) - 1:
            v = np.nan
        elif field == 0:
            v = frac * 2.0 ** (1 - fmt.bias - m)
        else:
            v = ((1 << m) + frac) * 2.0 ** (field - fmt.bias - m)
        out[c] = -v if neg else v
    return out.astype(np.float32)


def unpack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    if bits == 4:
        return np.stack((codes & 0xF, codes >> 4), axis=1).reshape(-1)
    return codes.reshape(-1)


def make_input(rng: np.random.Generator, rows: int, K: int, gs: int, dtype: torch.dtype) -> torch.Tensor:
    x = rng.standard_normal((rows, K))
    groups = x.reshape(rows, K // gs, gs)
    groups *= np.exp2(rng.integers(-140, 110, (rows, K // gs, 1)).astype(np.float64))
    flat = x.reshape(-1)
    pick = lambda k: rng.choice(flat.size, k, replace=False)  # noqa: E731
    flat[pick(200)] = 0.0
    flat[pick(200)] = -0.0
    flat[pick(40)] *= 2.0 ** -20
    x = x.astype(np.float32)
    xf = x.reshape(-1)
    xf[pick(6)] = np.inf
    xf[pick(6)] = -np.inf
    xf[pick(6)] = np.nan
    xf[pick(6)] = np.float32(3.3e38)
    t = torch.from_numpy(x)
    return t.to(dtype)


@pytest.mark.parametrize("scale_name", list(SCALES))
@pytest.mark.parametrize("element", ELEMENTS)
def test_group_quantize_matrix(element, scale_name):
    fmt = get_format(element)
    seed = zlib.crc32(f"{element}|{scale_name}".encode())
    rng = np.random.default_rng(seed)
    bits = fmt.ebits + fmt.mbits + 1
    for rounding in ROUNDINGS:
        gs = int(rng.choice([8, 16, 32, 64, 128]))
        dtype = torch.float32 if rng.random() < 0.6 else torch.bfloat16
        saturate = bool(rng.random() < 0.5)
        spec = QuantSpec(fmt, "group", group_size=gs, scale=SCALES[scale_name](), rounding=rounding,
                         saturate=saturate)
        x = make_input(rng, 24, 1024, gs, dtype)
        want = oracle_quantize(x.float().numpy(), spec)
        want_codes = bits <= 8
        got, ex = quantize_into(x.cuda(), spec, want_dequant=True, want_codes=want_codes,
                                want_scale_codes=spec.scale.format.name in ("e8m0", "ue4m3"))
        tag = f"{element} {scale_name} {rounding} gs={gs} sat={saturate} {dtype}"
        for field in ("values", "scale", "global_scale"):
            w, v = getattr(want, field), getattr(got, field)
            assert (w is None) == (v is None), (tag, field)
            if w is not None:
                g = v.float().cpu().numpy()
                assert bits_equal(g, np.asarray(w)), f"{tag} {field}: {first_mismatch(g, np.asarray(w))}"
        dq = ex.dequant.cpu().numpy()
        assert bits_equal(dq, oracle_dequantize(want)), f"{tag} dequant: {first_mismatch(dq, oracle_dequantize(want))}"
        vals = got.values.float().cpu().numpy().reshape(-1)
        if want_codes:
            decoded = code_table(fmt)[unpack_codes(ex.codes.cpu().numpy(), 4 if bits <= 4 else 8)]
            if fmt.special == "none":  # no NaN encoding: a NaN element is written as code 0
                assert not decoded[np.isnan(vals)].any()
                decoded = np.where(np.isnan(vals), vals, decoded)
            assert bits_equal(decoded, vals) or (
                np.array_equal(np.isnan(decoded), np.isnan(vals))
                and bits_equal(np.where(np.isnan(vals), 0, decoded), np.where(np.isnan(vals), 0, vals))
            ), f"{tag} codes: {first_mismatch(decoded, vals)}"
        if ex.scale_codes is not None:
            sc = got.scale.cpu().numpy().reshape(-1)
            codes = ex.scale_codes.cpu().numpy().reshape(-1).astype(np.int64)
            if spec.scale.format.name == "e8m0":
                dec = np.where(codes == 255, np.nan, np.ldexp(1.0, codes - 127)).astype(np.float32)
            else:
                dec = code_table(spec.scale.format)[codes]
            assert np.array_equal(np.isnan(dec), np.isnan(sc)), tag
            ok = ~np.isnan(sc)
            assert bits_equal(dec[ok], sc[ok]), f"{tag} scale codes"


def test_quantize_plan_matches_quantize_into():
    from tricast_b200 import QuantizePlan
    from tricast_b200.spec import SCHEMES

    g = torch.Generator().manual_seed(5)
    for name, dtype in (("mxfp4", torch.float32), ("nvfp4", torch.bfloat16), ("fp8_tensor", torch.bfloat16)):
        plan = QuantizePlan((64, 512), dtype, "cuda", SCHEMES[name], want_codes=name != "fp8_tensor",
                            want_dequant=True)
        for _ in range(2):
            x = (torch.randn(64, 512, generator=g) * 4).to(dtype).cuda()
            q, ex = plan.run(x)
            q2, ex2 = quantize_into(x, SCHEMES[name], want_codes=name != "fp8_tensor", want_dequant=True)
            assert torch.equal(q.values.view(torch.int16), q2.values.view(torch.int16))
            assert torch.equal(q.scale, q2.scale)
            assert torch.equal(ex.dequant, ex2.dequant)
            if name != "fp8_tensor":
                assert torch.equal(ex.codes, ex2.codes)
    with pytest.raises(ValueError, match="planned shape"):
        plan.run(torch.zeros(3, 3, device="cuda"))


@pytest.mark.parametrize("rows,K,gs", [(7, 96, 32), (3, 40, 8), (5, 384, 128), (9, 64, 16), (1, 32, 32),
                                       (13, 1056, 32), (3, 5504, 64), (11, 4112, 16)])
@pytest.mark.parametrize("scale_name", ["e8m0_floor", "ue4m3_two_level", "fp32_absmax"])
def test_group_quantize_ragged_group_counts(rows, K, gs, scale_name):
    """Sizes that split across the TMA-staged chunks (4096 elements), the register-staged kernel
    (whole warp iterations) and the four-elements-per-lane pass (the last few groups)."""
    rng = np.random.default_rng(rows * 1000 + K + gs)
    for element, dtype in (("fp4_e2m1", torch.float32), ("fp8_e4m3", torch.bfloat16)):
        fmt = get_format(element)
        spec = QuantSpec(fmt, "group", group_size=gs, scale=SCALES[scale_name]())
        x = make_input(rng, rows, K, gs, dtype) if rows * K >= 2000 else torch.from_numpy(
            (rng.standard_normal((rows, K)) * 3).astype(np.float32)).to(dtype)
        want = oracle_quantize(x.float().numpy(), spec)
        got, ex = quantize_into(x.cuda(), spec, want_dequant=True, want_codes=True,
                                want_scale_codes=spec.scale.format.name in ("e8m0", "ue4m3"))
        for field in ("values", "scale", "global_scale"):
            w, v = getattr(want, field), getattr(got, field)
            if w is not None:
                assert bits_equal(v.float().cpu().numpy(), np.asarray(w)), (element, field)
        dq = ex.dequant.cpu().numpy()
        assert bits_equal(dq, oracle_dequantize(want)), f"{element} dequant: {first_mismatch(dq, oracle_dequantize(want))}"
        bits = fmt.ebits + fmt.mbits + 1
        decoded = code_table(fmt)[unpack_codes(ex.codes.cpu().numpy(), 4 if bits <= 4 else 8)]
        vals = got.values.float().cpu().numpy().reshape(-1)
        if fmt.special == "none":  # no NaN encoding: a NaN element is written as code 0
            decoded = np.where(np.isnan(vals), vals, decoded)
        assert bits_equal(decoded, vals), f"{element} codes: {first_mismatch(decoded, vals)}"


SEARCH_SPECS = {
    "nvfp4_4o6": lambda: __import__("tricast_b200.spec", fromlist=["SCHEMES"]).SCHEMES["nvfp4_4o6"],
    "fp8_row_mse20": lambda: QuantSpec("fp8_e4m3", "row", scale=ScaleSpec("fp32", "mse", mse_grid=20)),
    "fp4_block_mse8": lambda: QuantSpec("fp4_e2m1", "block", block=(32, 64), scale=ScaleSpec("ue4m3", "mse", mse_grid=8)),
    "fp4_group_mse_sr": lambda: QuantSpec("fp4_e2m1", "group", group_size=32, rounding="sr",
                                          scale=ScaleSpec("ue4m3", "mse", mse_grid=5)),
    "int8_tensor_p999": lambda: QuantSpec("int8", "tensor", scale=ScaleSpec("fp32", "percentile", percentile=99.9)),
    "fp8_group_p99": lambda: QuantSpec("fp8_e4m3", "group", group_size=32,
                                       scale=ScaleSpec("fp32", "percentile", percentile=99.0)),
    "fp4_row_p50_two_level": lambda: QuantSpec("fp4_e2m1", "row",
                                               scale=ScaleSpec("ue4m3", "percentile", percentile=50.0, two_level=True)),
}


@pytest.mark.parametrize("name", list(SEARCH_SPECS))
@pytest.mark.parametrize("shape", [(37, 200), (64, 512)])
def test_mse_and_percentile_scales_vs_oracle(name, shape):
    """MSE candidate search and percentile scales on the GPU (fused group pass and the general
    per-domain pipeline), ragged domains and a NaN row included, against the oracle."""
    spec = SEARCH_SPECS[name]()
    rows, K = shape
    if spec.granularity == "group" and K % spec.group_size:
        K = (K // spec.group_size + 1) * spec.group_size
    rng = np.random.default_rng(zlib.crc32(f"{name}|{rows}".encode()))
    x = rng.standard_normal((rows, K)).astype(np.float32) * 2
    x[:, rng.choice(K, 3, replace=False)] *= 30
    x[3, 7] = np.nan
    kwargs = {}
    if str(getattr(spec.rounding, "name", spec.rounding)).lower() == "sr":
        kwargs["noise"] = rng.integers(0, 2 ** 32, (rows, K), dtype=np.uint64).astype(np.int64)
    want = oracle_quantize(x, spec, **kwargs)
    got, ex = quantize_into(torch.from_numpy(x).cuda(), spec, want_dequant=True,
                            **{k: torch.from_numpy(v).cuda() for k, v in kwargs.items()})
    for field in ("values", "scale", "global_scale"):
        w, v = getattr(want, field), getattr(got, field)
        assert (w is None) == (v is None), field
        if w is not None:
            g = v.float().cpu().numpy()
            assert bits_equal(g, np.asarray(w)), f"{name} {field}: {first_mismatch(g, np.asarray(w))}"
    dq = ex.dequant.cpu().numpy()
    assert bits_equal(dq, oracle_dequantize(want)), f"{name} dequant: {first_mismatch(dq, oracle_dequantize(want))}"


@pytest.mark.parametrize("K", [2048, 4096, 4097])
@pytest.mark.parametrize("spec", [QuantSpec("fp8_e4m3", "row"), QuantSpec("int8", "row"), QuantSpec("fp8_e4m3", "tensor"),
                                  QuantSpec("int4", "row"), QuantSpec("fp4_e2m1", "row"),
                                  QuantSpec("uint4", "row", scale=ScaleSpec("fp16"), zero_point="int", mma_input="dequant")],
                         ids=lambda s: f"{s.format.name}-{s.granularity}{'-zp' if s.zero_point != 'none' else ''}")
def test_single_row_tensors_take_the_grid_wide_pass(spec, K):
    """A decode step's one-row activation is a single scale domain: it runs through the grid-wide
    tensor pipeline (not one block on one row) and must equal the oracle, codes included."""
    g = torch.Generator().manual_seed(K)
    x = torch.randn(1, K, generator=g) * 3
    x[0, 5] = 40.0
    four_bit = spec.format.name in ("int4", "uint4", "fp4_e2m1")
    codes = not (four_bit and K % 2)  # packed 4-bit codes need an even element count
    q, extras = quantize_into(x.cuda(), spec, want_codes=codes, want_dequant=True)
    want = oracle_quantize(x.numpy(), spec)
    assert bits_equal(q.values.float().cpu().numpy(), want.values), first_mismatch(q.values.float().cpu().numpy(), want.values)
    assert bits_equal(q.scale.cpu().numpy().reshape(-1), np.asarray(want.scale, np.float32).reshape(-1))
    if spec.zero_point != "none":
        assert bits_equal(q.zero_point.cpu().numpy().reshape(-1), np.asarray(want.zero_point, np.float32).reshape(-1))
    assert bits_equal(extras.dequant.cpu().numpy(), np.asarray(oracle_dequantize(want)).reshape(extras.dequant.shape))
