"""Restatement of TriCast's package bit packing (``src/tricast/pack.py:66-91``), test infrastructure
only: unsigned ``bits``-bit codes as a flat little-endian byte stream, eight codes in ``bits`` bytes,
the last group padded with zeros; a quantized integer value ``v`` is stored as the code ``v - qmin``
(``pack.py:130-133``)."""

from __future__ import annotations

import numpy as np


def pack_bits(codes, bits: int) -> np.ndarray:
    """``pack.py:66-80``: codes (any shape, 0 <= code < 2**bits) -> uint8 stream."""
    if not 1 <= bits <= 8:
        raise ValueError(f"bits must be 1..8, got {bits}")
    flat = np.asarray(codes, dtype=np.int64).reshape(-1)
    if flat.size and (flat.min() < 0 or flat.max() >= 1 << bits):
        raise ValueError(f"codes do not fit in {bits} bits")
    if bits == 8:
        return flat.astype(np.uint8)
    flat = np.concatenate([flat, np.zeros(-flat.size % 8, np.int64)]).reshape(-1, 8)
    word = (flat << (np.arange(8, dtype=np.int64) * bits)).sum(axis=1)
    out = np.stack([(word >> (8 * j)) & 0xFF for j in range(bits)], axis=1)
    return out.reshape(-1).astype(np.uint8)


def unpack_bits(data, bits: int, count: int) -> np.ndarray:
    """``pack.py:83-91``: the first ``count`` codes of a ``pack_bits`` stream."""
    data = np.asarray(data, dtype=np.uint8)
    if bits == 8:
        return data[:count].copy()
    groups = data.astype(np.int64).reshape(-1, bits)
    word = (groups << (np.arange(bits, dtype=np.int64) * 8)).sum(axis=1)
    codes = np.stack([(word >> (bits * i)) & ((1 << bits) - 1) for i in range(8)], axis=1)
    return codes.reshape(-1)[:count].astype(np.uint8)
