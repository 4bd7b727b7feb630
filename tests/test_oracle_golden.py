"""Pin the CPU oracle: it must reproduce every golden fixture made by TriCast's own reference
backend and every NADPE golden vector, bit for bit. (CPU only.)"""

from __future__ import annotations

import hashlib
import json
import math

import numpy as np
import pytest

import oracle
from oracle import metrics as oracle_metrics
from oracle.quantize import dequantize, quantize_reference
from tests.conftest import bits_equal, first_mismatch
from tests.golden_cases import GOLDEN, bf16_bits, load, mma_operand, mspec, nadpe_cases, qspec
from tricast_b200.formats import get_format


def test_manifest_hashes():
    manifest = json.loads((GOLDEN / "MANIFEST.json").read_text())
    assert {"cast.npz", "quantize.npz", "mma.npz", "nadpe.npz", "metrics.json"} <= set(manifest)
    for name, digest in manifest.items():
        assert hashlib.sha256((GOLDEN / name).read_bytes()).hexdigest() == digest, name


def _cast_cases():
    meta, _ = load("cast")
    return [m for m in meta if "sr_bits" not in m]


@pytest.mark.parametrize("entry", _cast_cases(), ids=lambda m: m["key"])
def test_cast_matches_reference(entry):
    _, arrays = load("cast")
    fmt = get_format(entry["format"])
    key = entry["key"]
    x, noise = arrays[f"x|{key}"], arrays[f"noise|{key}"]
    for r in ("rne", "rna", "rtz", "rup", "rdn", "sr"):
        for sat in (0, 1):
            name = f"y|{key}|{r}|{sat}"
            if name not in arrays:
                with pytest.raises(ValueError, match="stochastic rounding"):
                    oracle.round_to_format(x, fmt, r, saturate=bool(sat), noise=noise)
                continue
            got = oracle.round_to_format(x, fmt, r, saturate=bool(sat), noise=noise)
            assert bits_equal(got, arrays[name]), f"{key} {r} sat={sat}: {first_mismatch(got, arrays[name])}"


def test_cast_sr_bits_sweep():
    meta, arrays = load("cast")
    for entry in (m for m in meta if "sr_bits" in m):
        _, name, bits = entry["key"].split("|")
        got = oracle.round_to_format(arrays[f"srx|{name}|{bits}"], get_format(entry["format"]), "sr",
                                     noise=arrays[f"srn|{name}|{bits}"], sr_bits=int(bits))
        assert bits_equal(got, arrays[f"sry|{name}|{bits}"]), entry["key"]


@pytest.mark.parametrize("case", load("quantize")[0], ids=lambda c: c["id"])
def test_quantize_matches_reference(case):
    _, arrays = load("quantize")
    cid = case["id"]
    spec = qspec(case["spec"])
    got = quantize_reference(arrays[f"{cid}|x"], spec, amax=case["amax"], noise=arrays.get(f"{cid}|noise"),
                             scale_noise=arrays.get(f"{cid}|scale_noise"))
    for field in ("values", "scale", "zero_point", "global_scale"):
        want = arrays.get(f"{cid}|{field}")
        value = getattr(got, field)
        if want is None:
            assert value is None, field
            continue
        assert np.shape(value) == want.shape, field
        assert bits_equal(value, want), f"{field}: {first_mismatch(value, want)}"
    assert bits_equal(dequantize(got), arrays[f"{cid}|dequant"])


@pytest.mark.parametrize("case", load("mma")[0], ids=lambda c: c["id"])
def test_gemm_matches_reference(case):
    _, arrays = load("mma")
    a, b = mma_operand(case, arrays, "a"), mma_operand(case, arrays, "b")
    spec = mspec(case["spec"])
    bias = arrays.get(f"{case['id']}|bias")
    if case["error"] is not None:
        with pytest.raises(ValueError):
            oracle.gemm_reference(a, b, spec, bias)
        return
    got = oracle.gemm_reference(a, b, spec, bias)
    want = arrays[f"{case['id']}|out"]
    assert bits_equal(got, want), first_mismatch(got, want)


def _nadpe_groups():
    cases = nadpe_cases()
    keys = sorted({c[0] for c in cases})
    return [(k, [c for c in cases if c[0] == k]) for k in keys]


@pytest.mark.parametrize("key,cases", _nadpe_groups(), ids=lambda v: v if isinstance(v, str) else "")
def test_nadpe_vectors(key, cases):
    """All 1,716 independent NADPE vectors (FP8 GDFS/CoFDA/decoupled, NVFP4, MXFP4)."""
    for _, index, a, b, spec, expected in cases:
        got = bf16_bits(oracle.gemm_reference(a, b, spec))
        assert np.array_equal(got, expected), f"{key} case {index}: {spec}"


def test_error_metrics_match_reference():
    for case in json.loads((GOLDEN / "metrics.json").read_text()):
        got = oracle_metrics.error_metrics(np.float32(case["reference"]), np.float32(case["emulated"]))
        for k, want in case["expected"].items():
            if isinstance(want, str):
                assert got[k] == want, k
            else:
                assert math.isclose(got[k], want, rel_tol=1e-12, abs_tol=0.0), (k, got[k], want)
