"""Pre-encoded B operands: ``gemm_triton`` keeps the fast path's encoding of a weight operand on the
operand object (as TriCast keeps its K-major copy, ``src/tricast/mma/operand.py:66-75``) and reuses it
while the weight's tensors are unchanged. Every result must equal the plain per-call path bit for
bit (the plain path is called through the C ABI directly, so no cache is involved), on the tiled
GDFS-FP4 path and on the small-M CoFDA path, including a B the fast path rejects, a weight edited in
place, and an encoding handed to the wrong kind of GEMM."""

from __future__ import annotations

import pytest
import torch

from tests.conftest import bits_equal
from tricast_b200 import _native as N
from tricast_b200 import as_operand, gemm_triton, quantize_triton
from tricast_b200.mma import _Prepared, exact_fallbacks, mma_spec_struct, resolve_scale_apply
from tricast_b200.spec import PRESETS, SCHEMES
from tricast_b200.formats import container_dtype

pytestmark = pytest.mark.gpu


def plain(a, b, spec):
    """tc_gemm through the C ABI (per-call encoding of both operands)."""
    pa, pb = _Prepared(a), _Prepared(b)
    ms = mma_spec_struct(spec, resolve_scale_apply(spec, a, b))
    out = torch.empty((a.rows, b.rows), device=a.values.device, dtype=container_dtype(spec.out_format))
    lib = N.lib()
    ws = torch.empty(max(lib.tc_gemm_workspace(pa.desc, pb.desc, ms), 1), device=a.values.device, dtype=torch.uint8)
    N.check(lib.tc_gemm(pa.desc, pb.desc, ms, None, N.ptr(out), N.ptr(ws), ws.numel(), N.stream_of(a.values.device)),
            "tc_gemm")
    return out


def operand(scheme, rows, k, seed, scale=1.0, compact=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, k, generator=g) * scale
    return as_operand(quantize_triton(x.bfloat16().cuda(), SCHEMES[scheme]), compact=compact)


def launches(fn):
    torch.cuda.synchronize()
    n0 = N.lib().tc_launch_count()
    out = fn()
    torch.cuda.synchronize()
    return out, N.lib().tc_launch_count() - n0


CASES = [
    # tiled GDFS-FP4 (A of more than 16 rows), tensor-core kernel
    ("nvfp4", "nvidia_blackwell_fp4", 256, 192, 1024, True),
    ("nvfp4", "nvidia_blackwell_fp4", 130, 65, 1040, False),
    ("mxfp4", "nvidia_blackwell_fp4", 200, 320, 512, True),
    # small-M CoFDA (decode shapes)
    ("fp8_tensor", "nvidia_hopper_fp8", 1, 4096, 4096, True),
    ("fp8_tensor", "nvidia_hopper_fp8", 16, 300, 1000, True),
    ("fp8_tensor", "nvidia_ada_fp8", 3, 256, 2048, False),
    ("fp8_tensor", "nvidia_blackwell_fp8", 2, 128, 1024, True),
    ("mxfp8_e4m3", "nvidia_blackwell_fp8", 4, 256, 1024, True),
]


@pytest.mark.parametrize("scheme,preset,m,n,k,compact", CASES)
def test_encoded_b_equals_per_call_path(scheme, preset, m, n, k, compact):
    spec = PRESETS[preset].with_(out_format="fp32")
    a = operand(scheme, m, k, 1, compact=compact)
    b = operand(scheme, n, k, 2, 0.02, compact=compact)
    want = plain(a, b, spec)
    first, n_first = launches(lambda: gemm_triton(a, b, spec))   # encodes B, keeps it
    second, n_second = launches(lambda: gemm_triton(a, b, spec))  # reuses it
    assert "_tc_b_encodings" in b.__dict__ and any(v[1] is not None for v in b._tc_b_encodings.values())
    assert n_second < n_first, "the second call should not encode B again"
    a2 = operand(scheme, m, k, 3, compact=compact)  # another activation against the same weight
    assert bits_equal(first.cpu().numpy(), want.cpu().numpy())
    assert bits_equal(second.cpu().numpy(), want.cpu().numpy())
    assert bits_equal(gemm_triton(a2, b, spec).cpu().numpy(), plain(a2, b, spec).cpu().numpy())


@pytest.mark.parametrize("scheme,preset,m", [("nvfp4", "nvidia_blackwell_fp4", 64),
                                             ("fp8_tensor", "nvidia_hopper_fp8", 2)])
def test_rejected_b_still_goes_to_the_exact_kernel(scheme, preset, m):
    spec = PRESETS[preset].with_(out_format="fp32")
    a = operand(scheme, m, 512, 4, compact=False)
    b = operand(scheme, 96, 512, 5, 0.02, compact=False)
    b.values[7, 100] = float("nan")
    want = plain(a, b, spec)
    f0 = exact_fallbacks()
    for _ in range(2):
        assert bits_equal(gemm_triton(a, b, spec).cpu().numpy(), want.cpu().numpy())
    assert exact_fallbacks() - f0 == 2


def test_weight_edited_in_place_is_encoded_again():
    spec = PRESETS["nvidia_hopper_fp8"].with_(out_format="fp32")
    a, b = operand("fp8_tensor", 4, 1024, 6), operand("fp8_tensor", 128, 1024, 7, 0.02)
    gemm_triton(a, b, spec)
    b.values.mul_(-1)  # still on the grid; bumps the tensor's version
    assert bits_equal(gemm_triton(a, b, spec).cpu().numpy(), plain(a, b, spec).cpu().numpy())


def test_encoding_for_another_kind_of_gemm_is_rejected():
    spec = PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32")
    small, big = operand("nvfp4", 4, 1024, 8), operand("nvfp4", 256, 1024, 9)
    b = operand("nvfp4", 128, 1024, 10, 0.02)
    ms = mma_spec_struct(spec, resolve_scale_apply(spec, big, b))
    pa, pb = _Prepared(big), _Prepared(b)
    lib = N.lib()
    nbytes = lib.tc_encode_b_bytes(pa.desc, pb.desc, ms)
    assert nbytes > 0
    assert lib.tc_encode_b_bytes(_Prepared(small).desc, pb.desc, ms) == 0  # the small-M FP4 path takes none
    enc = torch.empty(nbytes, device="cuda", dtype=torch.uint8)
    N.check(lib.tc_encode_b(pa.desc, pb.desc, ms, N.ptr(enc), nbytes, N.stream_of(enc.device)), "tc_encode_b")
    ps = _Prepared(small)
    out = torch.empty((4, 128), device="cuda")
    ws = torch.empty(max(lib.tc_gemm_workspace(ps.desc, pb.desc, ms), 1), device="cuda", dtype=torch.uint8)
    with pytest.raises(ValueError, match="encoded B was made for another"):
        N.check(lib.tc_gemm_encoded(ps.desc, pb.desc, N.ptr(enc), nbytes, ms, None, N.ptr(out), N.ptr(ws), ws.numel(),
                                    N.stream_of(enc.device)), "tc_gemm_encoded")
