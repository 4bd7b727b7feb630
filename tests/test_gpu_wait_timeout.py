"""The bounded waits of the staged GEMM kernels, driven to run out on purpose.

Every pipeline wait on a shared-memory barrier in the TMA-staged kernels is bounded. When one gives
up, the kernel sets its status word, waits for its own copies and MMAs in flight, frees its TMEM and
returns; the exact generic kernel already queued behind it sees the status word and recomputes the
product. ``tc_set_wait_limit(0)`` makes every such wait give up at once (nothing is left waiting on a
flag nobody sets: the limit is a poll count). These tests check that the status word was seen
(``tc_wait_timeouts``), that the result is still bit-identical to the oracle and to the normal run,
and that the context stays usable afterwards.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from tests.conftest import bits_equal, first_mismatch
from tricast_b200 import _native as N
from tricast_b200 import as_operand, gemm_triton, quantize_triton
from tricast_b200.formats import FP16, IntFormat
from tricast_b200.mma import exact_fallbacks, wait_timeouts
from tricast_b200.operand import Operand
from tricast_b200.spec import PRESETS, SCHEMES, MMASpec

pytestmark = pytest.mark.gpu


def _timeouts() -> int:
    return wait_timeouts()


@pytest.fixture
def wait_limit():
    lib = N.lib()

    def set_limit(polls: int) -> None:
        torch.cuda.synchronize()
        N.check(lib.tc_set_wait_limit(polls), "tc_set_wait_limit")

    yield set_limit
    torch.cuda.synchronize()
    lib.tc_set_wait_limit(-1)


def _quantized(scheme, rows, k, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(rows, k, generator=g) * scale).bfloat16().cuda()
    return as_operand(quantize_triton(x, SCHEMES[scheme]), compact=True)


def _cfg4_operands(m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).cuda()
    qa = quantize_triton(x, SCHEMES["int8_row"])
    qw = quantize_triton(w, SCHEMES["int4_g128_zp"])
    bvals = qw.values.float() - qw.zero_point.repeat_interleave(128, dim=1)
    return as_operand(qa, compact=True), Operand(bvals, IntFormat("int5", 5), qw.scale, FP16, "k", 128)


CASES = {
    # tcgen05 GDFS-FP4 kernel (A rows padded to 128): producer, MMA issuer and epilogue warps.
    "gdfs_fp4_tc": lambda: (_quantized("nvfp4", 256, 1024, 1), _quantized("nvfp4", 192, 1024, 2, 0.02),
                            PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32")),
    # CoFDA kernel (all threads wait on the stage barrier).
    "cofda": lambda: (_quantized("fp8_tensor", 130, 512, 3), _quantized("fp8_tensor", 96, 512, 4, 0.02),
                      PRESETS["nvidia_hopper_fp8"].with_(out_format="fp32")),
    # tcgen05 integer kernel with per-128 promotion (the INT4 x INT8 mapping).
    "int_promote_tc": lambda: (*_cfg4_operands(160, 256, 512, 5),
                               MMASpec("cofda", f_bits=23, chunk_size=32, promote_interval=128,
                                       out_format="fp32")),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_wait_that_runs_out_still_gives_the_exact_product(case, wait_limit):
    a, b, spec = CASES[case]()
    want = oracle.gemm_reference(a, b, spec)
    normal = gemm_triton(a, b, spec)
    torch.cuda.synchronize()
    assert bits_equal(normal.cpu().numpy(), want), first_mismatch(normal.cpu().numpy(), want)

    t0, f0 = _timeouts(), exact_fallbacks()
    wait_limit(0)  # every pipeline wait gives up at its first check
    got = gemm_triton(a, b, spec)
    torch.cuda.synchronize()
    assert _timeouts() - t0 == 1, "the fast kernel's status word did not reach the exact kernel"
    assert exact_fallbacks() - f0 == 1
    assert bits_equal(got.cpu().numpy(), want), first_mismatch(got.cpu().numpy(), want)

    # A second call in a row: the status words were cleared at the start of the call.
    again = gemm_triton(a, b, spec)
    torch.cuda.synchronize()
    assert _timeouts() - t0 == 2
    assert bits_equal(again.cpu().numpy(), want)

    # Back to the default limit: the fast kernel completes on its own and the context is usable.
    wait_limit(-1)
    t1 = _timeouts()
    after = gemm_triton(a, b, spec)
    torch.cuda.synchronize()
    assert _timeouts() == t1
    assert bits_equal(after.cpu().numpy(), want)


def test_a_few_polls_give_up_somewhere_in_the_pipeline(wait_limit):
    """With a limit of a few polls a wait may run out anywhere (first stage, a refill, an epilogue
    warp); whichever happens, the output is exact."""
    a, b, spec = CASES["gdfs_fp4_tc"]()
    want = oracle.gemm_reference(a, b, spec)
    for polls in (1, 2, 8):
        wait_limit(polls)
        got = gemm_triton(a, b, spec)
        torch.cuda.synchronize()
        assert bits_equal(got.cpu().numpy(), want), f"polls={polls}: {first_mismatch(got.cpu().numpy(), want)}"
    wait_limit(-1)
    assert np.isfinite(gemm_triton(a, b, spec).cpu().numpy()).all()
