"""Seeded synthetic inputs of the five benchmark configurations, shared by ``bench.py`` and the
benchmark-size parity tests, so that the tests compare exactly the tensors the benchmark times.

Every tensor is drawn on the CPU from a ``torch.Generator`` and moved afterwards, so every GPU count
and every process sees identical values (the per-layer sweep tensors, drawn on the device, live in
:mod:`tricast_b200.sweep`).

* cfg1  MXFP4 cast: 4096 x 4096 fp32 N(0,1), seed 0, 0.1 % of entries (16,777) scaled x50.
* cfg2  NVFP4 W4A4 GEMM: A 2048 x 4096 N(0,1) with 8 outlier channels x20 (seed 0); B 4096 x 4096
        N(0,0.02) (seed 1000); both bf16.
* cfg3  FP8 E4M3 W8A8 CoFDA GEMM: A 8192 x 8192 N(0,1), B 8192 x 8192 N(0,0.02), bf16, one seed-0
        stream (A first).
* cfg4  INT4 (g128, asymmetric) x INT8 (per token) GEMM: x 4096 x 4096 N(0,1), W 12288 x 4096
        N(0,0.02), fp32, one seed-0 stream (x first).
"""

from __future__ import annotations

import torch

CFG2_SHAPE = (2048, 4096, 4096)  # M, N, K
CFG3_SHAPE = (8192, 8192, 8192)
CFG4_SHAPE = (4096, 12288, 4096)


def cfg1_input() -> torch.Tensor:
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, 4096, generator=g)
    idx = torch.randperm(4096 * 4096, generator=g)[:16777]
    x.view(-1)[idx] *= 50
    return x


def cfg2_inputs(b_seed: int = 1000) -> tuple[torch.Tensor, torch.Tensor]:
    """(A [2048, 4096], B [4096, 4096]) bf16. ``b_seed`` other than 1000 draws another weight of the
    same distribution (distinct replicas)."""
    m, n, k = CFG2_SHAPE
    g = torch.Generator().manual_seed(0)
    a = torch.randn(m, k, generator=g)
    a[:, torch.randperm(k, generator=g)[:8]] *= 20
    gb = torch.Generator().manual_seed(b_seed)
    b = torch.randn(n, k, generator=gb) * 0.02
    return a.bfloat16(), b.bfloat16()


def cfg3_inputs(size: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """(A, B) bf16, M = N = K = 8192 (or ``size`` for a smaller cube)."""
    m = n = k = size or CFG3_SHAPE[0]
    g = torch.Generator().manual_seed(0)
    a = torch.randn(m, k, generator=g).bfloat16()
    b = (torch.randn(n, k, generator=g) * 0.02).bfloat16()
    return a, b


def cfg4_inputs() -> tuple[torch.Tensor, torch.Tensor]:
    """(x [4096, 4096], W [12288, 4096]) fp32."""
    m, n, k = CFG4_SHAPE
    g = torch.Generator().manual_seed(0)
    x = torch.randn(m, k, generator=g)
    w = torch.randn(n, k, generator=g) * 0.02
    return x, w


def cfg4_operands(qa, qw):
    """The INT4 x INT8 operand mapping: A = the INT8 per-token QTensor (row scale into the epilogue);
    B = the INT4 codes minus their zero points as an int5 grid with the fp16 group-128 scales applied
    at each promotion (``tricast.mma.operand.Operand`` semantics)."""
    from .formats import FP16, IntFormat
    from .operand import Operand, as_operand

    bvals = qw.values.float() - qw.zero_point.repeat_interleave(128, dim=1)[:, : qw.values.shape[1]]
    return as_operand(qa, compact=True), Operand(bvals, IntFormat("int5", 5), qw.scale, FP16, "k", 128)


def cfg4_spec():
    """CoFDA F=23 CS=32 promoted every 128 (exact INT32 sums per group, fp32 FMA promotion), fp32 out."""
    from .spec import MMASpec

    return MMASpec("cofda", f_bits=23, chunk_size=32, promote_interval=128, out_format="fp32")
