"""Silicon probe: does an emulated accumulation model reproduce the B200's own tensor-core MMA?

``native_mma_fp8`` runs ``tcgen05.mma kind::f8f6f4`` (fp32 accumulator in TMEM, K issued 32 at a time in
order, no scales) on E4M3 / E5M2 codes; ``native_mma_fp4`` runs the block-scaled
``kind::mxf4nvf4`` on E2M1 codes with UE4M3 scales per 16 (NVFP4) or E8M0 scales per 32 (MXFP4).
``match_table`` / ``match_table_fp4`` run the same products through this library's emulation under
each candidate ``MMASpec`` with an fp32 output and count the outputs that agree bit for bit. The
presets under test are TriCast's ``nvidia_*_fp8`` and ``nvidia_blackwell_fp4`` models
(``tricast/mma/spec.py:223-330``); the sweeps add neighbouring models (fraction bits, chunk or group
size, normalisation rounding) so that a mismatch says which way the hardware differs.

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


E2M1_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])
FP4_BLOCK = {0: 16, 1: 32}  # scale_fmt -> elements per scale


def native_mma_fp4(a_codes: torch.Tensor, b_codes: torch.Tensor, sfa: torch.Tensor, sfb: torch.Tensor,
                   scale_fmt: int) -> torch.Tensor:
    """Block-scaled ``a @ b.T`` in fp32 by the tensor core. ``a_codes`` [M, K] and ``b_codes`` [N, K] are
    uint8 E2M1 codes (0..15, one a byte; packed two a byte here), ``sfa`` [M, K / V] and ``sfb``
    [N, K / V] uint8 scale codes: ``scale_fmt`` 0 = UE4M3 with V = 16, 1 = E8M0 with V = 32."""
    if scale_fmt not in FP4_BLOCK:
        raise ValueError("scale_fmt must be 0 (UE4M3 per 16) or 1 (E8M0 per 32)")
    V = FP4_BLOCK[scale_fmt]
    M, K = a_codes.shape
    Nr = b_codes.shape[0]
    if b_codes.shape[1] != K or K % 64:
        raise ValueError("operands must be [M, K] and [N, K] with K a multiple of 64")
    if tuple(sfa.shape) != (M, K // V) or tuple(sfb.shape) != (Nr, K // V):
        raise ValueError("scales must be [rows, K / V]")
    dev = a_codes.device

    def pack(c):
        c = c.to(torch.uint8)
        return ((c[:, 0::2] & 15) | ((c[:, 1::2] & 15) << 4)).contiguous()

    pa, pb = pack(a_codes), pack(b_codes)
    sa, sb = sfa.to(torch.uint8).contiguous(), sfb.to(torch.uint8).contiguous()
    out = torch.empty((M, Nr), device=dev, dtype=torch.float32)
    status = torch.zeros((), device=dev, dtype=torch.int32)
    with torch.cuda.device(dev):
        N.check(N.lib().tc_probe_mma_fp4(N.ptr(pa), N.ptr(pb), N.ptr(sa), N.ptr(sb), M, Nr, K, scale_fmt, N.ptr(out),
                                         N.ptr(status), N.stream_of(dev)), "tc_probe_mma_fp4")
    if int(status.item()) != 0:
        raise N.NativeError("tc_probe_mma_fp4: a wait inside the kernel ran out")
    return out


def scale_values(codes: torch.Tensor, scale_fmt: int) -> torch.Tensor:
    """fp32 values of UE4M3 (scale_fmt 0) or E8M0 (1) scale codes."""
    if scale_fmt == 0:
        return codes.to(torch.uint8).view(torch.float8_e4m3fn).to(torch.float32)
    return torch.ldexp(torch.ones(codes.shape, dtype=torch.float32, device=codes.device), codes.to(torch.int32) - 127)


def random_fp4(rows: int, K: int, scale_fmt: int, dist: str, gen: torch.Generator, e8m0_span: int = 30):
    """Seeded E2M1 codes and scale codes. ``"gauss"``: codes of N(0, 2) rounded to the E2M1 grid, scales
    within 2^-3 .. 2^3; ``"codes"``: uniform codes, scales over a wide range (UE4M3: every finite
    non-zero code; E8M0: 2^-e8m0_span .. 2^e8m0_span)."""
    V = FP4_BLOCK[scale_fmt]
    if dist == "gauss":
        x = torch.randn(rows, K, generator=gen) * 2
        codes = (x.unsqueeze(-1) - E2M1_VALUES[:8].unsqueeze(0) * torch.sign(x).unsqueeze(-1)).abs()[..., :8].argmin(-1)
        codes = torch.where(x < 0, codes + 8, codes)
        if scale_fmt == 0:  # UE4M3 codes with exponent field 4..10: 2^-3 .. 2^3
            sc = torch.randint(4 << 3, 11 << 3, (rows, K // V), generator=gen)
        else:
            sc = torch.randint(124, 131, (rows, K // V), generator=gen)
    elif dist == "codes":
        codes = torch.randint(0, 16, (rows, K), generator=gen)
        if scale_fmt == 0:
            sc = torch.randint(1, 0x7F, (rows, K // V), generator=gen)
        else:
            sc = torch.randint(127 - e8m0_span, 128 + e8m0_span, (rows, K // V), generator=gen)
    else:
        raise ValueError(f"unknown distribution {dist!r}")
    return codes.to(torch.uint8), sc.to(torch.uint8)


def candidate_specs_fp4() -> dict[str, MMASpec]:
    """The FP4 preset, fp32 FMA / fp64, and GDFS / CoFDA models around it."""
    specs = {name: PRESETS[name] for name in ("nvidia_blackwell_fp4", "nvidia_blackwell_fp8", "fp32_fma", "fp64")}
    for f in (25, 30, 35, 40, 48):
        for g in (6, 8):
            for kt in (32, 64, 128):
                specs[f"gdfs_f{f}_g{g}_gs16_kt{kt}"] = MMASpec("gdfs", f_bits=f, g_bits=g, group_size=16, k_tile=kt)
    for f in (25, 35):
        specs[f"gdfs_f{f}_g6_gs16_kt64_rne"] = MMASpec("gdfs", f_bits=f, g_bits=6, group_size=16, k_tile=64,
                                                       norm_rounding="rne")
        specs[f"gdfs_f{f}_g6_gs32_kt64"] = MMASpec("gdfs", f_bits=f, g_bits=6, group_size=32, k_tile=64)
    for f in (25, 35):
        for cs in (16, 32, 64):
            specs[f"cofda_f{f}_cs{cs}_rtz"] = MMASpec("cofda", f_bits=f, chunk_size=cs)
    return specs


def match_table_fp4(M: int = 256, N: int = 128, K: int = 1024, *, scale_fmt: int = 0, dist: str = "gauss",
                    seed: int = 0, specs: dict[str, MMASpec] | None = None, device="cuda",
                    e8m0_span: int = 30) -> dict:
    """``match_table`` for the block-scaled FP4 MMA: each candidate model on the same E2M1 codes and
    per-block scales (the operands TriCast builds for NVFP4 / MXFP4 weights and activations)."""
    from .formats import get_format as fmt_of

    V = FP4_BLOCK[scale_fmt]
    gen = torch.Generator().manual_seed(seed)
    ac, sa = random_fp4(M, K, scale_fmt, dist, gen, e8m0_span)
    bc, sb = random_fp4(N, K, scale_fmt, dist, gen, e8m0_span)
    ac, sa, bc, sb = (t.to(device) for t in (ac, sa, bc, sb))
    native = native_mma_fp4(ac, bc, sa, sb, scale_fmt)
    nbits = native.view(torch.int32)
    e2m1 = E2M1_VALUES.to(device)
    sfmt = fmt_of("ue4m3" if scale_fmt == 0 else "e8m0")
    oa = Operand(e2m1[ac.long()], fmt_of("fp4_e2m1"), scale_values(sa, scale_fmt), sfmt, "k", V)
    ob = Operand(e2m1[bc.long()], fmt_of("fp4_e2m1"), scale_values(sb, scale_fmt), sfmt, "k", V)
    rows = {}
    for name, spec in (specs or candidate_specs_fp4()).items():
        try:
            emu = gemm_triton(oa, ob, spec.with_(out_format=FP32))
        except ValueError as exc:  # the model cannot take these operands (e.g. a group across a scale block)
            rows[name] = {"match": None, "max_ulp": None, "inapplicable": str(exc)}
            continue
        same = (emu.view(torch.int32) == nbits) | ((emu == 0) & (native == 0)) | (emu.isnan() & native.isnan())
        ulp = torch.ldexp(torch.ones_like(native, dtype=torch.float64), (torch.frexp(native)[1] - 24).clamp_min(-149))
        diff = ((emu.double() - native.double()).abs() / ulp).nan_to_num(0.0).max()
        rows[name] = {"match": round(float(same.double().mean()), 6), "max_ulp": round(float(diff), 3)}
    table = {"M": M, "N": N, "K": K, "scale": sfmt.name, "block": V, "dist": dist, "seed": seed, "results": rows}
    if scale_fmt == 1 and dist == "codes":
        table["e8m0_span"] = e8m0_span
    return table


def main() -> None:
    out = []
    for fmt in (0, 1):
        for dist in ("gauss", "codes"):
            out.append(match_table(fmt=fmt, dist=dist))
    for scale_fmt in (0, 1):
        for dist in ("gauss", "codes"):
            out.append(match_table_fp4(scale_fmt=scale_fmt, dist=dist))
    print(json.dumps(out))


if __name__ == "__main__":
    main()
