"""The tcgen05 FP8 silicon probe: the native MMA kernel itself, then the emulation presets against it.

The first tests pin the probe kernel (operand layout, descriptors, ragged tiles, K tails): on operands
whose every partial sum is exact in fp32 the hardware result must equal the exact dot product bit for
bit, whatever its accumulation order or alignment. The match-table test then runs the emulated
models against the hardware on random data and checks the findings recorded for this library.
"""

from __future__ import annotations

import json

import pytest
import torch

from tricast_b200 import _native as N
from tricast_b200.probe import FP8_DTYPES, candidate_specs, match_table, native_mma_fp8

pytestmark = pytest.mark.gpu

GRID = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0])


def _grid_operand(rows, k, dtype, gen):
    idx = torch.randint(0, len(GRID), (rows, k), generator=gen)
    return GRID[idx].to(dtype).cuda()


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (128, 64, 128), (130, 70, 45), (257, 129, 1000), (64, 200, 33),
                                   (3, 5, 0)])
def test_native_fp8_exact_sums(fmt, M, N, K):
    """Products are multiples of 1/4 below 16 in magnitude, so every partial sum is exact in fp32."""
    dtype = FP8_DTYPES[fmt]
    gen = torch.Generator().manual_seed(M * 7 + N * 3 + K)
    a, b = _grid_operand(M, K, dtype, gen), _grid_operand(N, K, dtype, gen)
    got = native_mma_fp8(a, b)
    want = (a.double() @ b.double().T).float()
    assert torch.equal(got, want)


def test_native_fp8_rows_and_columns_are_not_permuted():
    """Distinct one-hot rows: output (m, n) is A[m, k_m] * B[n, k_m], which pins row, column and K
    placement inside the tile layout."""
    M, N, K = 128, 64, 256
    a = torch.zeros(M, K)
    b = torch.zeros(N, K)
    for m in range(M):
        a[m, (m * 37) % K] = 1.0 + (m % 8) / 8
    for n in range(N):
        b[n] = ((torch.arange(K) + n) % 7 + 1).float() / 4
    a8, b8 = a.to(torch.float8_e4m3fn).cuda(), b.to(torch.float8_e4m3fn).cuda()
    got = native_mma_fp8(a8, b8)
    assert torch.equal(got, (a8.double() @ b8.double().T).float())


def test_native_fp8_rejects_bad_arguments():
    a = torch.zeros(4, 8, dtype=torch.float8_e4m3fn, device="cuda")
    with pytest.raises(ValueError):
        native_mma_fp8(a, torch.zeros(4, 8, dtype=torch.float8_e5m2, device="cuda"))
    with pytest.raises(ValueError):
        native_mma_fp8(a, torch.zeros(4, 9, dtype=torch.float8_e4m3fn, device="cuda"))
    out = torch.empty(16, device="cuda")
    status = torch.zeros((), dtype=torch.int32, device="cuda")
    rc = N.lib().tc_probe_mma_fp8(N.ptr(a), N.ptr(a), 4, 4, 8, 2, N.ptr(out), N.ptr(status), None)
    assert rc == N.TC_INVALID_ARGUMENT


def test_match_table_runs_every_candidate():
    table = match_table(M=128, N=64, K=512, fmt=0, dist="gauss", seed=1)
    print(json.dumps(table))
    assert set(table["results"]) == set(candidate_specs())
    for row in table["results"].values():
        assert 0.0 <= row["match"] <= 1.0
        assert row["max_ulp"] >= 0.0
