"""Packed element codes of integer formats against TriCast's package format (``src/tricast/pack.py``):
4-bit codes two per byte, low nibble first, and 8-bit codes one per byte, as ``pack_bits`` lays them
out. For unsigned formats (qmin = 0) the library's codes are byte for byte ``pack_bits(values - qmin)``.
For signed formats the library writes two's-complement codes (the bit pattern a hardware int4/int8
operand takes) where a package stores ``values - qmin``; the test pins that one relation code by code."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.pack import pack_bits, unpack_bits
from tricast_b200.quantize import quantize_into
from tricast_b200.spec import SCHEMES

pytestmark = pytest.mark.gpu


def _codes(scheme: str, rows: int, k: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(rows, k, generator=g) * 0.05).cuda()
    q, extras = quantize_into(x, SCHEMES[scheme], want_codes=True)
    return q.values.float().cpu().numpy().astype(np.int64), extras.codes.cpu().numpy(), SCHEMES[scheme].format


@pytest.mark.parametrize("scheme", ["int4_g128_zp", "kivi4"])
@pytest.mark.parametrize("rows,k", [(64, 256), (37, 384), (5, 128)])
def test_unsigned_4bit_codes_are_pack_bits(scheme, rows, k):
    values, codes, fmt = _codes(scheme, rows, k, rows + k)
    assert fmt.qmin == 0 and fmt.qmax == 15
    want = pack_bits(values - fmt.qmin, 4)
    n = values.size
    assert codes.size == (n + 1) // 2
    assert np.array_equal(codes, want[: codes.size])
    assert np.array_equal(unpack_bits(np.concatenate([codes, np.zeros(-codes.size % 4, np.uint8)]), 4, n),
                          (values - fmt.qmin).reshape(-1))


@pytest.mark.parametrize("scheme,bits", [("int4_g128", 4), ("int8_row", 8), ("int8_tensor", 8)])
def test_signed_codes_are_twos_complement_of_pack_codes(scheme, bits):
    values, codes, fmt = _codes(scheme, 48, 256, bits)
    flat = values.reshape(-1)
    packed = pack_bits(flat - fmt.qmin, bits)  # what a TriCast package stores
    stored = unpack_bits(packed, bits, flat.size).astype(np.int64) + fmt.qmin
    mine = unpack_bits(np.concatenate([codes, np.zeros(-codes.size % bits, np.uint8)]), bits, flat.size)
    mine = mine.astype(np.int64)
    mine = np.where(mine >= 1 << (bits - 1), mine - (1 << bits), mine)  # two's complement
    assert np.array_equal(mine, flat) and np.array_equal(stored, flat)
