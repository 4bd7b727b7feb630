"""Oracle per-layer error statistics (TEST INFRASTRUCTURE ONLY).

Restates ``src/tricast/analysis.py:29-69`` (``_ErrorStats``): fp64 sums of x^2, y^2, (x-y)^2 and
x*y plus max |x-y|, then MSE, SQNR (dB), max abs error, relative Frobenius norm and cosine
similarity (clamped to [-1, 1]); infinite ratios are the strings "inf" / "-inf".
"""

from __future__ import annotations

import math

import numpy as np


def sums(reference, emulated) -> tuple[int, float, float, float, float, float]:
    x = np.asarray(reference, np.float64).reshape(-1)
    y = np.asarray(emulated, np.float64).reshape(-1)
    if x.shape != y.shape or not x.size:
        raise ValueError("error metrics require matching, nonempty tensor shapes")
    if not (np.isfinite(x).all() and np.isfinite(y).all()):
        raise ValueError("error metrics encountered non-finite values")
    d = x - y
    return x.size, float((x * x).sum()), float((y * y).sum()), float((d * d).sum()), float((x * y).sum()), \
        float(np.abs(d).max())


def result(count, signal, estimate, error, dot, maximum) -> dict:
    if not count:
        raise ValueError("no layer activations were observed")
    sqnr = "inf" if not error else "-inf" if not signal else 10.0 * math.log10(signal / error)
    relative = math.sqrt(error / signal) if signal else 0.0 if not error else "inf"
    cosine = (max(-1.0, min(1.0, dot / math.sqrt(signal * estimate))) if signal and estimate
              else float(not signal and not estimate))
    return {"mse": error / count, "sqnr_db": sqnr, "max_abs_error": maximum,
            "relative_frobenius": relative, "cosine": cosine}


def error_metrics(reference, emulated) -> dict:
    return result(*sums(reference, emulated))
