"""Silicon probe: does an emulated accumulation model reproduce the B200's own FP8 tensor-core MMA?

``native_mma_fp8`` runs ``tcgen05.mma kind::f8f6f4`` (fp32 accumulator in TMEM, K issued 32 at a time in
order, no scales) on E4M3 / E5M2 codes; ``match_table`` runs the same products through this library's
emulation under each candidate ``MMASpec`` with an fp32 output and counts the outputs that agree bit
for bit. The presets under test are TriCast's ``nvidia_*_fp8`` models (``tricast/mma/spec.py:223-330``);
the sweep adds neighbouring CoFDA models (fraction bits, chunk size, normalisation rounding) so that a
mismatch says which way the hardware differs.

``python -m tricast_b200.probe`` prints the table as one JSON object (needs a CUDA device).
"""

from __future__ import annotations

import json

import torch

from . import _native as N
from .formats import FP32, get_format
from .mma import gemm_triton
from .operand import Operand
from .spec import PRESETS, MMASpec

FP8_DTYPES = {0: torch.float8_e4m3fn, 1: torch.float8_e5m2}


def native_mma_fp8(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a @ b.T`` in fp32 by the tensor core's FP8 MMA; ``a`` [M, K] and ``b`` [N, K] are CUDA tensors of
    the same float8 dtype (``float8_e4m3fn`` or ``float8_e5m2``)."""
    if a.dtype != b.dtype or a.dtype not in FP8_DTYPES.values():
        raise ValueError("operands must share a float8_e4m3fn or float8_e5m2 dtype")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError("operands must be [M, K] and [N, K]")
    if not a.is_cuda or a.device != b.device:
        raise ValueError("operands must be on the same CUDA device")
    fmt = 0 if a.dtype == torch.float8_e4m3fn else 1
    a8, b8 = a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8)
    M, K = a8.shape
    out = torch.empty((M, b8.shape[0]), device=a.device, dtype=torch.float32)
    status = torch.zeros((), device=a.device, dtype=torch.int32)
    with torch.cuda.device(a.device):
        N.check(N.lib().tc_probe_mma_fp8(N.ptr(a8), N.ptr(b8), M, b8.shape[0], K, fmt, N.ptr(out), N.ptr(status),
                                         N.stream_of(a.device)), "tc_probe_mma_fp8")
    if int(status.item()) != 0:
        raise N.NativeError("tc_probe_mma_fp8: a wait inside the kernel ran out")
    return out


def random_fp8(rows: int, K: int, dtype: torch.dtype, dist: str, gen: torch.Generator, device) -> torch.Tensor:
    """Seeded fp8 operands: ``"gauss"`` = N(0, 1) rounded to the format (clustered exponents),
    ``"codes"`` = uniform over the finite codes (the full exponent range, subnormals and signed zeros)."""
    if dist == "gauss":
        return torch.randn(rows, K, generator=gen).to(dtype).to(device)
    if dist != "codes":
        raise ValueError(f"unknown distribution {dist!r}")
    codes = torch.randint(0, 256, (rows, K), generator=gen, dtype=torch.int32).to(torch.uint8)
    x = codes.view(dtype)
    finite = torch.isfinite(x.to(torch.float32))
    x = torch.where(finite, x.to(torch.float32), torch.zeros(())).to(dtype)
    return x.to(device)


def candidate_specs() -> dict[str, MMASpec]:
    """The FP8 presets, fp32 FMA / fp64, and a sweep of CoFDA models around the Blackwell preset."""
    specs = {name: PRESETS[name] for name in ("nvidia_blackwell_fp8", "nvidia_hopper_fp8", "nvidia_ada_fp8",
                                              "fp32_fma", "fp64")}
    for f in (23, 24, 25, 26, 27, 28):
        for cs in (16, 32, 64, 128):
            for rnd in ("rtz", "rne"):
                specs[f"cofda_f{f}_cs{cs}_{rnd}"] = MMASpec("cofda", f_bits=f, chunk_size=cs, norm_rounding=rnd)
    return specs


def match_table(M: int = 256, N: int = 128, K: int = 1024, *, fmt: int = 0, dist: str = "gauss", seed: int = 0,
                specs: dict[str, MMASpec] | None = None, device="cuda") -> dict:
    """Fraction of the M x N outputs on which each candidate model equals the hardware bit for bit
    (``+0`` and ``-0`` counted equal), with the largest difference in fp32 ulps of the native result."""
    dtype = FP8_DTYPES[fmt]
    gen = torch.Generator().manual_seed(seed)
    a = random_fp8(M, K, dtype, dist, gen, device)
    b = random_fp8(N, K, dtype, dist, gen, device)
    native = native_mma_fp8(a, b)
    nbits = native.view(torch.int32)
    fmt_obj = get_format("fp8_e4m3" if fmt == 0 else "fp8_e5m2")
    oa, ob = Operand(a.to(torch.float32), fmt_obj), Operand(b.to(torch.float32), fmt_obj)
    rows = {}
    for name, spec in (specs or candidate_specs()).items():
        emu = gemm_triton(oa, ob, spec.with_(out_format=FP32))
        same = (emu.view(torch.int32) == nbits) | ((emu == 0) & (native == 0))
        ulp = torch.ldexp(torch.ones_like(native, dtype=torch.float64), (torch.frexp(native)[1] - 24).clamp_min(-149))
        diff = ((emu.double() - native.double()).abs() / ulp).max()
        rows[name] = {"match": round(float(same.double().mean()), 6), "max_ulp": round(float(diff), 3)}
    return {"M": M, "N": N, "K": K, "fmt": fmt_obj.name, "dist": dist, "seed": seed, "results": rows}


def main() -> None:
    out = []
    for fmt in (0, 1):
        for dist in ("gauss", "codes"):
            out.append(match_table(fmt=fmt, dist=dist))
    print(json.dumps(out))


if __name__ == "__main__":
    main()
