"""The N-column split on one GPU, its ranks emulated one after the other: every slab of the weight is
quantized against the whole tensor's amax (the shards' amax bits reduced into one word, as the NCCL
all-reduce does across GPUs) and must give exactly those rows of the whole tensor's QTensor; every
slab GEMM must give exactly those columns of the whole GEMM."""

from __future__ import annotations

import pytest
import torch

from tricast_b200 import _native as N
from tricast_b200 import as_operand, gemm_triton, quantize_triton
from tricast_b200.quantize import quantize_into
from tricast_b200.shard import column_slab, shard_amax
from tricast_b200.spec import PRESETS, SCHEMES

pytestmark = pytest.mark.gpu


def same_bits(a: torch.Tensor, b: torch.Tensor) -> bool:
    a, b = a.float().contiguous(), b.float().contiguous()
    return a.shape == b.shape and bool(((a.view(torch.int32) == b.view(torch.int32)) | (a.isnan() & b.isnan())).all())


def amax_bits_of_slabs(w: torch.Tensor, slabs) -> torch.Tensor:
    bits = torch.zeros((), dtype=torch.int32, device=w.device)
    for s, e in slabs:
        x = w[s:e].contiguous()
        N.check(N.lib().tc_tensor_amax_bits(N.ptr(x), N.dtype_code(x.dtype), x.numel(), N.ptr(bits),
                                            N.stream_of(w.device)), "tc_tensor_amax_bits")
    return bits


def test_amax_bits_are_the_nan_propagating_amax():
    g = torch.Generator().manual_seed(0)
    for dtype in (torch.float32, torch.bfloat16, torch.float16):
        x = (torch.randn(333, 77, generator=g) * 5).to(dtype).cuda()
        assert shard_amax(x).item() == x.float().abs().max().item()
        x.view(-1)[1234] = float("nan")
        assert torch.isnan(shard_amax(x))
        x.view(-1)[1234] = float("-inf")
        assert shard_amax(x).item() == float("inf")


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("scheme,preset", [("nvfp4", "nvidia_blackwell_fp4"), ("fp8_tensor", "nvidia_hopper_fp8"),
                                           ("mxfp4", "nvidia_blackwell_fp4")])
def test_slabs_equal_the_whole(world, scheme, preset):
    g = torch.Generator().manual_seed(world)
    m, n, k = 192, 1000, 512
    a = torch.randn(m, k, generator=g)
    a[:, :3] *= 20
    a = a.bfloat16().cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).bfloat16().cuda()
    spec, mspec = SCHEMES[scheme], PRESETS[preset].with_(out_format="fp32")
    qa, qw = quantize_triton(a, spec), quantize_triton(w, spec)
    whole = gemm_triton(as_operand(qa, compact=True), as_operand(qw, compact=True), mspec)
    slabs = [column_slab(n, world, r) for r in range(world)]
    amax = amax_bits_of_slabs(w, slabs).view(torch.float32)
    for s, e in slabs:
        if scheme == "nvfp4":
            q = quantize_into(w[s:e], spec, tensor_amax=amax)[0]
        elif scheme == "fp8_tensor":
            q = quantize_into(w[s:e], spec, amax=amax)[0]
        else:
            q = quantize_into(w[s:e], spec)[0]
        assert same_bits(q.values, qw.values[s:e])
        assert same_bits(q.scale.reshape(-1), (qw.scale if qw.scale.dim() == 0 else qw.scale[s:e]).reshape(-1))
        if qw.global_scale is not None:
            assert same_bits(q.global_scale, qw.global_scale)
        part = gemm_triton(as_operand(qa, compact=True), as_operand(q, compact=True), mspec)
        assert same_bits(part, whole[:, s:e]), f"columns {s}..{e} of {n}"


def test_public_quantize_keeps_tricasts_amax_rule():
    x = torch.randn(64, 64).cuda()
    with pytest.raises(ValueError, match="amax override requires tensor granularity"):
        quantize_triton(x, SCHEMES["nvfp4"], amax=torch.tensor(3.0).cuda())
    with pytest.raises(ValueError, match="tensor_amax needs a two-level spec"):
        quantize_into(x, SCHEMES["mxfp4"], tensor_amax=torch.tensor(3.0).cuda())
