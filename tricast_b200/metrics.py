"""Per-layer error metrics on the device (TriCast ``analysis._ErrorStats``,
``src/tricast/analysis.py:29-69``): the fp64 sums run in ``tc_error_stats``; only the five final
scalars are formed on the host."""

from __future__ import annotations

import math

import torch

from . import _native as N


class ErrorStats:
    """Accumulates fp64 sums over one or more (reference, emulated) pairs on the device."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.sums = torch.zeros(6, dtype=torch.float64, device=self.device)
        self.count = 0

    def update(self, reference: torch.Tensor, emulated: torch.Tensor) -> None:
        if reference.shape != emulated.shape or not reference.numel():
            raise ValueError("error metrics require matching, nonempty tensor shapes")
        r = reference.detach().contiguous()
        e = emulated.detach().contiguous()
        if r.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            r = r.float()
        if e.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            e = e.float()
        with torch.cuda.device(self.device):
            N.check(N.lib().tc_error_stats(N.ptr(r), N.dtype_code(r.dtype), N.ptr(e), N.dtype_code(e.dtype), r.numel(),
                                           N.ptr(self.sums), N.stream_of(self.device)), "tc_error_stats")
        self.count += r.numel()

    def result(self) -> dict:
        if not self.count:
            raise ValueError("no layer activations were observed")
        signal, estimate, error, dot, maximum, bad = self.sums.tolist()
        if bad:
            raise ValueError("error metrics encountered non-finite values")
        return finish(self.count, signal, estimate, error, dot, maximum)


def finish(count, signal, estimate, error, dot, maximum) -> dict:
    """The five metrics from the fp64 sums (``analysis.py:52-62``)."""
    sqnr = "inf" if not error else "-inf" if not signal else 10.0 * math.log10(signal / error)
    relative = math.sqrt(error / signal) if signal else 0.0 if not error else "inf"
    cosine = (max(-1.0, min(1.0, dot / math.sqrt(signal * estimate))) if signal and estimate
              else float(not signal and not estimate))
    return {"mse": error / count, "sqnr_db": sqnr, "max_abs_error": maximum, "relative_frobenius": relative,
            "cosine": cosine}


def error_metrics(reference: torch.Tensor, emulated: torch.Tensor) -> dict:
    stats = ErrorStats(reference.device)
    stats.update(reference, emulated)
    return stats.result()
