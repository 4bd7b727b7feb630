"""The oracle's restatement of TriCast's package bit packing, pinned against TriCast's own
``pack_bits`` / ``unpack_bits`` (``src/tricast/pack.py:66-91``) when TriCast is importable."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

from oracle.pack import pack_bits, unpack_bits

_REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _tricast_pack():
    if _REF.is_dir() and str(_REF) not in sys.path:
        sys.path.append(str(_REF))
    try:
        from tricast import pack
    except Exception:  # pragma: no cover - depends on the install
        pytest.skip("TriCast is not installed")
    return pack


@pytest.mark.parametrize("bits", [1, 2, 3, 4, 5, 7, 8])
@pytest.mark.parametrize("count", [0, 1, 7, 8, 9, 64, 1001])
def test_pack_matches_tricast(bits, count):
    import torch

    pack = _tricast_pack()
    codes = np.random.default_rng(bits * 1000 + count).integers(0, 1 << bits, count)
    want = pack.pack_bits(torch.from_numpy(codes), bits).numpy()
    got = pack_bits(codes, bits)
    assert got.dtype == np.uint8 and np.array_equal(got, want)
    assert np.array_equal(unpack_bits(got, bits, count), codes.astype(np.uint8))


def test_four_bit_layout_is_low_nibble_first():
    assert pack_bits([1, 2, 3, 4, 5, 6, 7, 8, 9], 4).tolist() == [0x21, 0x43, 0x65, 0x87, 0x09, 0, 0, 0]


def test_rejects_codes_that_do_not_fit():
    with pytest.raises(ValueError):
        pack_bits([16], 4)
