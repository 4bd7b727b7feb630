"""Shared pytest setup: the ``gpu`` marker, repo imports and bit-level comparison helpers.

GPU tests need a CUDA device; on a machine without one they are skipped (the CPU suite runs
with ``-m "not gpu"``). On a GPU box they call the C-ABI library and fail loudly if it is missing.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built C-ABI library")
    config.addinivalue_line("markers", "slow: long-running")


def _cuda_ok() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def bits_equal(actual, expected, *, signed_zero: bool = True) -> bool:
    """fp32 equality where every NaN equals every NaN and, by default, the sign of zero counts."""
    a = np.asarray(actual, np.float32).reshape(-1)
    e = np.asarray(expected, np.float32).reshape(-1)
    if a.shape != e.shape:
        return False
    both_nan = np.isnan(a) & np.isnan(e)
    same = a.view(np.uint32) == e.view(np.uint32)
    if not signed_zero:
        same |= (a == 0) & (e == 0)
    return bool((both_nan | same).all())


def first_mismatch(actual, expected) -> str:
    a = np.asarray(actual, np.float32).reshape(-1)
    e = np.asarray(expected, np.float32).reshape(-1)
    bad = ~((np.isnan(a) & np.isnan(e)) | (a.view(np.uint32) == e.view(np.uint32)))
    idx = np.flatnonzero(bad)[:5]
    return ", ".join(f"[{i}] got {a[i]!r} ({a.view(np.uint32)[i]:#010x}) want {e[i]!r} ({e.view(np.uint32)[i]:#010x})"
                     for i in idx)
