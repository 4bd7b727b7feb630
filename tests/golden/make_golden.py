"""Generate the golden fixtures in this folder by running TriCast's own reference backend.

Run once on a machine that has a TriCast checkout, with ``TRICAST_SRC`` set to its ``src``
directory: ``TRICAST_SRC=<checkout>/src python tests/golden/make_golden.py``. The fixtures are committed; nothing at
test time reads the TriCast checkout.

Contents:
* ``cast.npz``      — ``round_to_format`` over every registered and several custom formats ×
                      6 roundings × saturate, on wide random bit patterns plus format boundaries
                      (the case matrix of TriCast ``tests/gpu/test_triton_quantize.py:54-80``);
* ``quantize.*``    — ``quantize_reference`` over all schemes, scale methods × granularities ×
                      roundings, zero points, scale specials, amax overrides, explicit SR streams
                      (``test_triton_quantize.py:109-200,286-420``);
* ``mma.*``         — ``gemm_reference`` over every algorithm × format × scale layout, the
                      adversarial / special / scale-edge / shape cases of
                      ``tests/gpu/test_triton_mma.py:73-209,403-418`` and small instances of the
                      benchmark configurations;
* ``nadpe.*``       — TriCast's 1,716 NADPE golden vectors (``tests/data/nadpe``) converted from
                      ``.pt`` to numpy, decoded with the rules of ``tests/test_golden.py:176-242``;
* ``metrics.json``  — ``analysis._ErrorStats`` on a few pairs;
* ``MANIFEST.json`` — sha256 of every fixture file.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
SRC = os.environ.get("TRICAST_SRC", "")
if not SRC:
    sys.exit("set TRICAST_SRC to the src directory of a TriCast checkout")
sys.path.insert(0, SRC)

from tricast.analysis import error_metrics  # noqa: E402
from tricast.formats import (  # noqa: E402
    BF16, E8M0, FP4_E2M1, FP6_E2M3, FP6_E3M2, FP8_E4M3, FP8_E5M2, FP16, FP32, INT8, MXINT8, REGISTRY, UE4M3,
    FloatFormat, IntFormat, Pow2Format, get_format,
)
from tricast.mma.api import as_operand  # noqa: E402
from tricast.mma.operand import Operand  # noqa: E402
from tricast.mma.spec import MMASpec  # noqa: E402
from tricast.quant.spec import SCHEMES, QuantSpec, ScaleSpec  # noqa: E402
from tricast.reference.cast import round_to_format  # noqa: E402
from tricast.reference.mma import gemm_reference  # noqa: E402
from tricast.reference.quantize import _layout, quantize_reference  # noqa: E402

ROUNDINGS = ("rne", "rna", "rtz", "rup", "rdn", "sr")


def fmt_dict(fmt) -> dict:
    if isinstance(fmt, FloatFormat):
        return {"kind": "float", "name": fmt.name, "ebits": fmt.ebits, "mbits": fmt.mbits, "bias": fmt.bias,
                "special": fmt.special, "signed": fmt.signed, "subnormals": fmt.subnormals}
    if isinstance(fmt, IntFormat):
        return {"kind": "int", "name": fmt.name, "bits": fmt.bits, "signed": fmt.signed,
                "symmetric": fmt.symmetric, "frac_bits": fmt.frac_bits}
    return {"kind": "pow2", "name": fmt.name, "ebits": fmt.ebits, "bias": fmt.bias}


def qspec_dict(spec: QuantSpec) -> dict:
    scale = None
    if spec.scale is not None:
        s = spec.scale
        scale = {"format": fmt_dict(s.format), "method": s.method, "rounding": s.rounding.value,
                 "two_level": s.two_level, "percentile": s.percentile, "mse_grid": s.mse_grid,
                 "search": list(s.search)}
    return {"format": fmt_dict(spec.format), "granularity": spec.granularity, "group_size": spec.group_size,
            "block": list(spec.block), "scale": scale, "zero_point": spec.zero_point,
            "rounding": spec.rounding.value, "sr_bits": spec.sr_bits, "saturate": spec.saturate,
            "mma_input": spec.mma_input, "dequant_format": fmt_dict(spec.dequant_format)}


def mspec_dict(spec: MMASpec) -> dict:
    return {"algorithm": spec.algorithm, "f_bits": spec.f_bits, "chunk_size": spec.chunk_size,
            "c_mode": spec.c_mode, "f2_bits": spec.f2_bits, "g_bits": spec.g_bits, "group_size": spec.group_size,
            "k_tile": spec.k_tile, "norm_rounding": spec.norm_rounding, "scale_apply": spec.scale_apply,
            "promote_interval": spec.promote_interval, "out_format": fmt_dict(spec.out_format)}


def wide_fp32(n, gen, lo=0, hi=255):
    sign = torch.randint(0, 2, (n,), generator=gen) << 31
    exp = torch.randint(lo, hi, (n,), generator=gen) << 23
    frac = torch.randint(0, 2 ** 23, (n,), generator=gen)
    return (sign | exp | frac).to(torch.int32).view(torch.float32)


def boundaries(fmt):
    pts = [0.0, -0.0, 2.0 ** -149, 2.0 ** -126, 1.0, 1.5, 2.0, fmt.min_normal, fmt.max_normal]
    q = getattr(fmt, "min_subnormal", fmt.min_normal)
    pts += [q, q / 2, q * 1.5, q * 2.5]
    if isinstance(fmt, FloatFormat):
        pts += [fmt.max_normal + 2.0 ** (fmt.emax - fmt.mbits - 1)]
    elif isinstance(fmt, IntFormat):
        pts += [abs(fmt.qmin) * 2.0 ** -fmt.frac_bits]
    f = torch.tensor(pts, dtype=torch.float64).float()
    f = torch.cat((f, torch.nextafter(f, torch.full_like(f, float("inf"))),
                   torch.nextafter(f, torch.full_like(f, -float("inf")))))
    return torch.cat((f, -f, torch.tensor([float("nan"), -float("inf"), float("inf")])))


def make_cast(arrays: dict, meta: list) -> None:
    gen = torch.Generator().manual_seed(42)
    wide = wide_fp32(3000, gen)
    formats = dict(REGISTRY)
    for name in ("e3m4:nosub", "e8m0:ieee", "int8:full", "int24", "uint24", "int9:frac=130",
                 "e8m23:ieee:bias=127", "ue5m2", "e2m3:fn", "e5m0:bias=20"):
        formats[name] = get_format(name)
    for key, fmt in formats.items():
        x = torch.cat((wide, boundaries(fmt)))
        noise = torch.randint(0, 2 ** 32, x.shape, generator=gen, dtype=torch.int64)
        arrays[f"x|{key}"] = x.numpy()
        arrays[f"noise|{key}"] = noise.numpy().astype(np.uint32)
        for r in ROUNDINGS:
            if isinstance(fmt, Pow2Format) and r == "sr":
                continue
            for sat in (0, 1):
                y = round_to_format(x, fmt, r, saturate=bool(sat), noise=noise)
                arrays[f"y|{key}|{r}|{sat}"] = y.numpy()
        meta.append({"key": key, "format": fmt_dict(fmt)})
    # sr_bits sweep on far-underflow values (test_triton_quantize.py:83-91)
    x = torch.tensor([2.0 ** -149, 2.0 ** -126, 2.0 ** -40, 2.0 ** -25, 0.125, 1.0625])
    x = torch.cat((x, -x))[:, None]
    noise = torch.tensor([0, 1, 255, 65535, 2 ** 23 - 1, 2 ** 31 - 1, 2 ** 31, 2 ** 32 - 1])[None, :]
    x = x.expand(-1, noise.numel()).contiguous()
    for bits in (1, 8, 16, 32):
        for name in ("fp32", "bf16", "fp16", "fp4", "int8"):
            arrays[f"srx|{name}|{bits}"] = x.numpy()
            arrays[f"srn|{name}|{bits}"] = noise.expand_as(x).contiguous().numpy().astype(np.uint32)
            arrays[f"sry|{name}|{bits}"] = round_to_format(x, name, "sr", noise=noise, sr_bits=bits).numpy()
            meta.append({"key": f"sr|{name}|{bits}", "format": fmt_dict(get_format(name)), "sr_bits": bits})


def make_quantize(arrays: dict, meta: list) -> None:
    def add(cid, x, spec, noise=None, scale_noise=None, amax=None):
        q = quantize_reference(x, spec, amax=amax, noise=noise, scale_noise=scale_noise)
        arrays[f"{cid}|x"] = x.numpy()
        if noise is not None:
            arrays[f"{cid}|noise"] = torch.broadcast_to(noise, x.shape).contiguous().numpy().astype(np.uint32)
        if scale_noise is not None:
            arrays[f"{cid}|scale_noise"] = scale_noise.numpy().astype(np.uint32)
        for f in ("values", "scale", "zero_point", "global_scale"):
            v = getattr(q, f)
            if v is not None:
                arrays[f"{cid}|{f}"] = v.float().numpy()
        arrays[f"{cid}|dequant"] = q.dequantize().numpy()
        meta.append({"id": cid, "spec": qspec_dict(spec), "shape": list(x.shape),
                     "amax": None if amax is None else float(amax),
                     "fields": [f for f in ("values", "scale", "zero_point", "global_scale")
                                if getattr(q, f) is not None],
                     "values_dtype": str(q.values.dtype).replace("torch.", "")})

    for name, spec in SCHEMES.items():
        if spec.observer is not None:
            continue
        for shape in ((37,), (3, 35), (2, 3, 129), (129, 7)):
            x = torch.randn(shape, generator=torch.Generator().manual_seed(42)) * 3.25
            x.reshape(-1)[0] = 0
            add(f"scheme-{name}-{'x'.join(map(str, shape))}", x, spec)
    for method in ("absmax", "pow2_floor", "pow2_ceil", "mse", "percentile"):
        for gran in ("tensor", "row", "group", "block"):
            for r in ROUNDINGS:
                spec = QuantSpec("fp4", gran, group_size=7, block=(2, 5), rounding=r,
                                 scale=ScaleSpec("e8m0" if method.startswith("pow2") else "fp16", method, mse_grid=3))
                x = torch.randn((3, 17), generator=torch.Generator().manual_seed(42))
                noise = torch.randint(0, 2 ** 32, x.shape, generator=torch.Generator().manual_seed(42), dtype=torch.int64)
                add(f"method-{method}-{gran}-{r}", x, spec, noise=noise)
    for zp in ("int", "float"):
        for r in ROUNDINGS:
            spec = QuantSpec("uint4", "group", group_size=5, zero_point=zp, mma_input="dequant",
                             scale=ScaleSpec("fp16"), rounding=r)
            x = torch.tensor([[-3.1, -1.25, -0.1, 0.0, 7.3, 0.125, 2.75]])
            noise = torch.tensor([0, 1, 2 ** 31, 2 ** 32 - 1, 17, 31, 255])
            add(f"zp-{zp}-{r}", x, spec, noise=noise)
    for name in ("kivi2", "kivi4"):
        for r in ROUNDINGS:
            spec = SCHEMES[name].with_(group_size=4, rounding=r)
            x = torch.tensor([[-1., .1, .5, 2., 2., 2., 2.], [2., 2.25, 3.5, 5., -2., -2., -2.],
                              [-5., -4., -3., -2., 0., 0., 0.]])
            noise = torch.tensor([0, 2 ** 30 - 1, 2 ** 30, 2 ** 32 - 1, 0, 1, 2 ** 31])
            add(f"kivi-{name}-{r}", x, spec, noise=noise)
    for sign in (-1.0, 1.0):
        spec = SCHEMES["kivi2"].with_(scale=ScaleSpec("fp32"), dequant_format="fp32")
        add(f"kivi-subnormal-{int(sign)}", torch.tensor([[sign * k * 2. ** -149 for k in (1, 2, 3, 4)]]), spec)
    add("kivi-subtract-first", torch.tensor([[-2. ** -24, 1., 6.]]), SCHEMES["kivi2"])
    for seed in (2, 3, 4, 7):
        bits = torch.randint(0, 2, (17, 33), generator=torch.Generator().manual_seed(seed)) * -(2 ** 31)
        add(f"zp-signed-zero-{seed}", bits.int().view(torch.float32),
            QuantSpec("uint4", "block", block=(16, 16), zero_point="float", mma_input="dequant"))
    for name in ("mxfp4", "nvfp4", "fp8_tensor", "int4_g128", "int8_row", "mxfp8_e4m3"):
        for value in (0.0, 2.0 ** -149, 2.0 ** -126, float("inf"), float("nan"), -float("inf")):
            add(f"special-{name}-{value}", torch.full((2, 35), value), SCHEMES[name])
    for method in ("pow2_floor", "pow2_ceil"):
        for sfmt in ("ue4m3", "e8m0"):
            spec = QuantSpec("fp4_e2m1", "group", group_size=16, scale=ScaleSpec(sfmt, method, two_level=True))
            x = torch.cat((wide_fp32(4096, torch.Generator().manual_seed(42), 110, 140), torch.tensor([6.0] * 32)))
            add(f"two-level-{method}-{sfmt}", x.reshape(-1, 32), spec)
    x = torch.randn((7, 3), generator=torch.Generator().manual_seed(42)).T.contiguous()
    add("amax-override", x, SCHEMES["fp8_tensor"], amax=torch.tensor(8.0))
    for method in ("absmax", "pow2_floor", "pow2_ceil"):
        spec = QuantSpec("fp4", scale=ScaleSpec("e8m0" if method.startswith("pow2") else "fp32", method))
        add(f"negzero-amax-{method}", torch.zeros((2, 7)), spec, amax=torch.tensor(-0.0))
    for gran in ("tensor", "row", "group", "block"):
        for two_level in (False, True):
            g = torch.Generator().manual_seed(42)
            x = torch.randn((5, 19), generator=g) * 7
            spec = QuantSpec("fp4", gran, group_size=7, block=(2, 5), rounding="sr",
                             scale=ScaleSpec("fp16", rounding="sr", two_level=two_level))
            noise = torch.randint(0, 2 ** 32, (1, 19), generator=g, dtype=torch.int64)
            sn = torch.randint(0, 2 ** 32, _layout(spec, *x.shape), generator=torch.Generator().manual_seed(43),
                               dtype=torch.int64)
            add(f"scale-sr-{gran}-{int(two_level)}", x, spec, noise=noise, scale_noise=sn)
    x = torch.tensor([[.15, 1.05, 6.003], [.15, 1.05, 6.003]])
    add("scale-sr-separate", x, QuantSpec("fp4", "row", rounding="sr", scale=ScaleSpec("fp16", rounding="sr")),
        noise=torch.zeros_like(x, dtype=torch.int64), scale_noise=torch.tensor([[0], [2 ** 32 - 1]]))
    # Small instances of the benchmark configurations.
    g = torch.Generator().manual_seed(0)
    x = torch.randn(64, 256, generator=g)
    x.view(-1)[torch.randperm(x.numel(), generator=g)[:40]] *= 50
    add("cfg1-mxfp4", x, SCHEMES["mxfp4"])
    add("cfg2-nvfp4", torch.randn(64, 256, generator=g).bfloat16().float(), SCHEMES["nvfp4"])
    add("cfg3-fp8", (torch.randn(64, 256, generator=g) * 0.02).bfloat16().float(), SCHEMES["fp8_tensor"])
    add("cfg4-w", (torch.randn(48, 256, generator=g) * 0.02).bfloat16().float(), SCHEMES["int4_g128_zp"])
    add("cfg4-x", torch.randn(32, 256, generator=g), SCHEMES["int8_row"])


def _operand(rows, k, fmt, layout, gen):
    values = round_to_format(torch.randn(rows, k, generator=gen) * 2, fmt)
    if layout == "none":
        return Operand(values, fmt)
    if layout in ("tensor", "row"):
        shape = () if layout == "tensor" else (rows, 1)
        return Operand(values, fmt, 0.5 + torch.rand(shape, generator=gen), FP32, layout)
    domain = 64 if layout == "block" else 32
    domains = (k + domain - 1) // domain
    srows = (rows + 3) // 4 if layout == "block" else rows
    raw = 0.25 + torch.rand((srows, domains), generator=gen) * 2
    sfmt = E8M0 if layout == "mx" else UE4M3 if layout == "nv" else FP32
    scales = round_to_format(raw, sfmt)
    if layout == "block":
        scales = scales.repeat_interleave(4, dim=0)[:rows]
    alpha = torch.tensor(1.001234) if layout == "nv" else None
    return Operand(values, fmt, scales, sfmt, "k", domain, alpha)


def make_mma(arrays: dict, meta: list) -> None:
    def put_op(cid, side, op):
        arrays[f"{cid}|{side}|values"] = op.values.float().numpy()
        if op.scale is not None:
            arrays[f"{cid}|{side}|scale"] = op.scale.float().numpy()
        if op.alpha is not None:
            arrays[f"{cid}|{side}|alpha"] = op.alpha.float().reshape(()).numpy()
        return {"fmt": fmt_dict(op.fmt), "scale_fmt": None if op.scale_fmt is None else fmt_dict(op.scale_fmt),
                "scale_kind": op.scale_kind, "k_domain": op.k_domain, "has_alpha": op.alpha is not None}

    def add(cid, a, b, spec, bias=None):
        try:
            out = gemm_reference(a, b, spec, bias)
            error = None
        except ValueError as exc:
            out, error = None, str(exc)
        entry = {"id": cid, "a": put_op(cid, "a", a), "b": put_op(cid, "b", b), "spec": mspec_dict(spec),
                 "has_bias": bias is not None, "error": error}
        if bias is not None:
            arrays[f"{cid}|bias"] = bias.float().numpy()
        if out is not None:
            arrays[f"{cid}|out"] = out.float().numpy()
            entry["out_dtype"] = str(out.dtype).replace("torch.", "")
        meta.append(entry)

    formats = (FP8_E4M3, FP8_E5M2, FP6_E3M2, FP6_E2M3, FP4_E2M1, BF16, FP16, INT8, MXINT8)
    layouts = ("none", "tensor", "row", "mx", "nv", "block", "mixed")
    for ai, algorithm in enumerate(("cofda", "gdfs", "fp32_fma", "fp64")):
        for fi, fmt in enumerate(formats):
            for variation in range(2):
                i = fi * 2 + variation
                layout = layouts[(i + ai) % len(layouts)]
                cs = (8, 16, 32)[i % 3]
                pi = 32 if algorithm == "cofda" and i % 4 == 0 else 0
                spec = MMASpec(algorithm, f_bits=(3, 7, 13, 23, 25, 35)[i % 6], chunk_size=cs,
                               c_mode="decoupled" if variation else "fused", f2_bits=(7, 23, 35)[fi % 3],
                               g_bits=16, group_size=8 if variation else 16, k_tile=64,
                               norm_rounding="rne" if variation else "rtz", promote_interval=pi,
                               out_format=(FP32, BF16, FP16, FP8_E4M3, FP6_E3M2, FP4_E2M1)[(i + ai) % 6])
                index = i + ai * 18
                gen = torch.Generator().manual_seed(42)
                sg = torch.Generator().manual_seed(42 + index)
                m, n = torch.randint(1, 20, (2,), generator=sg).tolist()
                k = int(torch.randint(1, 100, (), generator=sg))
                la, lb = ("row", "mx") if layout == "mixed" else (layout, layout)
                a, b = _operand(m, k, fmt, la, gen), _operand(n, k, fmt, lb, gen)
                bias = torch.randn(n, generator=gen) / 7
                add(f"mode-{algorithm}-{fmt.name}-{layout}-{i}", a, b, spec, bias)
    for fmt in (INT8, MXINT8):
        for layout in ("none", "tensor", "row"):
            gen = torch.Generator().manual_seed(42)
            sg = torch.Generator().manual_seed(42)
            m, n = torch.randint(1, 20, (2,), generator=sg).tolist()
            k = int(torch.randint(1, 100, (), generator=sg))
            a, b = _operand(m, k, fmt, layout, gen), _operand(n, k, fmt, layout, gen)
            add(f"int_exact-{fmt.name}-{layout}", a, b, MMASpec("int_exact", out_format=FP32),
                torch.randn(n, generator=gen) / 7)
    adv = {"subnormal": ([2.0 ** -149, -2.0 ** -148, 2.0 ** -126, 2.0 ** -130, 0.0], [1.0, 1.5, 0.125, 0.375, -0.0]),
           "special": ([float("inf"), -float("inf"), float("nan"), 0.0, 1.0], [0.0, 1.0, -1.0, float("inf"), 1.0]),
           "cancel": ([1.125, -1.125, 0.0, -0.0, 1.0], [1.0, 1.0, -0.0, 0.0, 0.0]),
           "wide_alignment": ([2.0 ** 127, 2.0 ** 64, 2.0 ** 63, 2.0 ** 62, 2.0 ** -149], [1.0] * 5)}
    for algorithm in ("cofda", "gdfs", "fp32_fma", "fp64"):
        spec = MMASpec(algorithm, f_bits=25, chunk_size=8, g_bits=25, group_size=8, k_tile=32, out_format=FP32)
        for case, (av, bv) in adv.items():
            a = Operand(torch.tensor([av]), FP32)
            b = Operand(torch.cat((torch.tensor([bv]), torch.diag(torch.tensor(bv)))), FP32)
            add(f"adversarial-{algorithm}-{case}", a, b, spec)
        a = Operand(torch.tensor([[-float("inf")], [float("inf")], [float("nan")], [0.0], [-0.0], [1.0]]), FP32)
        b = Operand(torch.tensor([[-float("inf")], [0.0], [float("inf")], [1.0], [-1.0]]), FP32)
        add(f"singletons-{algorithm}", a, b, spec)
    for f_bits in (3, 7, 13, 23, 25, 35):
        add(f"short-promote-{f_bits}", Operand(torch.tensor([[1.5 * 2.0 ** -65]]), BF16),
            Operand(torch.tensor([[1.421875 * 2.0 ** -65]]), BF16),
            MMASpec(f_bits=f_bits, chunk_size=8, promote_interval=32, out_format=FP32))
    for algorithm in ("cofda", "gdfs"):
        spec = MMASpec(algorithm, f_bits=35, chunk_size=8, g_bits=35, group_size=8, k_tile=32, out_format=FP32)
        edges = {"wide_product": (torch.tensor([[1.9999998807907104, -1.5, 0.25, 1.125, -0.5]]),
                                  torch.tensor([[1.9999998807907104]]), FP32),
                 "scale_subnormal": (torch.tensor([[2.0 ** 60, 2.0 ** 59, -2.0 ** 60, 2.0 ** 57, 0.0]]),
                                     torch.tensor([[2.0 ** -127]]), BF16),
                 "zero_nan": (torch.zeros(1, 5), torch.tensor([[float("nan")]]), FP32),
                 "zero_inf": (torch.zeros(1, 5), torch.tensor([[float("inf")]]), FP32),
                 "inf_zero": (torch.full((1, 5), float("inf")), torch.zeros(1, 1), FP32),
                 "e8m0_field0": (torch.full((1, 5), 2.0 ** 64), torch.tensor([[2.0 ** -127]]), E8M0)}
        for case, (values, scale, fmt) in edges.items():
            add(f"scale-edge-{algorithm}-{case}", Operand(values, FP32, scale, fmt, "k", 8),
                Operand(values, FP32, torch.ones_like(scale), fmt, "k", 8), spec)
        for side in ("a", "b"):
            for fname in ("e8m0", "e8m0:bias=128", "e7m0:bias=127"):
                for exponent in (-127, -126):
                    values = torch.ones((1, 8))
                    so = Operand(values, FP4_E2M1, torch.tensor([[2.0 ** exponent]]), get_format(fname), "k", 8)
                    uo = Operand(values, FP4_E2M1)
                    a, b = (so, uo) if side == "a" else (uo, so)
                    add(f"field0-{algorithm}-{side}-{fname}-{exponent}", a, b,
                        MMASpec(algorithm, f_bits=25, chunk_size=8, g_bits=6, group_size=8, k_tile=8, out_format=FP32))
        add(f"e8m0-nan-{algorithm}", Operand(torch.ones(1, 1), FP4_E2M1, torch.tensor([[float("nan")]]), E8M0, "k", 8),
            Operand(torch.ones(1, 1), FP4_E2M1),
            MMASpec(algorithm, f_bits=13, chunk_size=8, group_size=8, k_tile=32, out_format=FP32))
    for shape in ((0, 7, 3), (3, 0, 7), (3, 5, 0), (67, 81, 511)):
        gen = torch.Generator().manual_seed(42)
        m, n, k = shape
        add(f"shape-{m}x{n}x{k}", _operand(m, k, FP8_E4M3, "none", gen), _operand(n, k, FP8_E4M3, "none", gen),
            MMASpec(f_bits=13, chunk_size=32, out_format=FP32))
    fmt = IntFormat("fixed_subnormal", 8, frac_bits=75)
    add("int-exact-subnormal", Operand(torch.tensor([[3 * 2.0 ** -75]]), fmt), Operand(torch.tensor([[2.0 ** -75]]), fmt),
        MMASpec("int_exact", out_format=FP32))
    for algorithm in ("cofda", "gdfs", "fp32_fma", "fp64", "int_exact"):
        gen = torch.Generator().manual_seed(42)
        fmt = INT8 if algorithm == "int_exact" else BF16
        add(f"tile-{algorithm}", _operand(33, 37, fmt, "none", gen), _operand(35, 37, fmt, "none", gen),
            MMASpec(algorithm, f_bits=13, chunk_size=8, g_bits=13, group_size=8, k_tile=32, out_format=FP32))
    # Benchmark configurations at small size, through the public quantize/as_operand path.
    from tricast.quant.api import quantize
    g = torch.Generator().manual_seed(0)
    presets = {"cfg2": ("nvfp4", {"preset": "nvidia_blackwell_fp4", "out_format": "fp32"}),
               "cfg3": ("fp8_tensor", {"preset": "nvidia_hopper_fp8", "out_format": "fp32"}),
               "mxfp4": ("mxfp4", {"preset": "nvidia_blackwell_fp4", "out_format": "fp32"}),
               "mxfp4-bf16": ("mxfp4", {"preset": "nvidia_blackwell_fp4"}),
               "fp8-bf16": ("fp8_tensor", {"preset": "nvidia_hopper_fp8"}),
               "bw-fp8": ("fp8_tensor", {"preset": "nvidia_blackwell_fp8", "out_format": "fp32"}),
               "ada-fp8": ("fp8_tensor", {"preset": "nvidia_ada_fp8", "out_format": "fp32"}),
               "mxfp8-promote": ("mxfp8_e4m3", {"preset": "nvidia_hopper_fp8", "out_format": "fp32"})}
    for name, (scheme, mspec) in presets.items():
        xa = torch.randn(40, 512, generator=g)
        xa[:, torch.randperm(512, generator=g)[:3]] *= 20
        xb = torch.randn(24, 512, generator=g) * 0.02
        a = as_operand(quantize(xa.bfloat16().float(), scheme, backend="reference"))
        b = as_operand(quantize(xb.bfloat16().float(), scheme, backend="reference"))
        add(f"cfg-{name}", a, b, MMASpec.from_dict(mspec))
    xa = torch.randn(40, 512, generator=g)
    w = torch.randn(24, 512, generator=g) * 0.02
    qa = quantize(xa, "int8_row", backend="reference")
    qw = quantize(w, "int4_g128_zp", backend="reference")
    z = qw.zero_point.repeat_interleave(128, dim=1)[:, :512]
    b = Operand(qw.values.float() - z, IntFormat("int5", 5), qw.scale, FP16, "k", 128)
    add("cfg-cfg4", as_operand(qa), b,
        MMASpec("cofda", f_bits=23, chunk_size=32, promote_interval=128, out_format="fp32"))
    wb = (torch.randn(24, 512, generator=g) * 0.02).bfloat16()
    add("cfg-fp64-ref", as_operand(xa.bfloat16()), as_operand(wb), MMASpec("fp64", out_format="fp32"))


def make_nadpe(arrays: dict, meta: list) -> None:
    root = Path(SRC).parent / "tests" / "data" / "nadpe"
    e2m1 = torch.tensor((0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0))
    for path in sorted(root.glob("fp8_*.pt")):
        v = torch.load(path, map_location="cpu", weights_only=True)
        key = path.stem
        arrays[f"{key}|a"] = v["a_codes"].contiguous().view(torch.float8_e4m3fn).float().numpy()
        arrays[f"{key}|b"] = v["w_codes"].contiguous().view(torch.float8_e4m3fn).float().numpy()
        cases = []
        for i, c in enumerate(v["cases"]):
            arrays[f"{key}|out|{i}"] = c["out_bits"].numpy()
            cases.append({k: int(c[k]) for k in ("algorithm", "f_bits", "g_bits", "group_size", "chunk_size")})
        meta.append({"key": key, "kind": "fp8", "scale_a": float(v["scale_a"]), "scale_b": float(v["scale_b"]),
                     "cases": cases})
    for path in sorted(root.glob("fp4_*.pt")):
        v = torch.load(path, map_location="cpu", weights_only=True)
        key = path.stem
        for side in ("a", "w"):
            arrays[f"{key}|{side}"] = e2m1[v[f"{side}_codes"].to(torch.int64)].numpy()
            codes = v[f"{side}_scale_codes"]
            if v["scale_format"] == "ue4m3":
                scale = (codes & 0x7F).contiguous().view(torch.float8_e4m3fn).float()
            else:
                scale = torch.ldexp(torch.ones(codes.shape), codes.to(torch.int64) - 127).float()
            arrays[f"{key}|{side}_scale"] = scale.numpy()
        cases = []
        for i, c in enumerate(v["cases"]):
            arrays[f"{key}|out|{i}"] = c["out_bits"].numpy()
            cases.append({k: int(c[k]) for k in ("algorithm", "f_bits", "g_bits", "group_size", "chunk_size")})
        meta.append({"key": key, "kind": "fp4", "block": int(v["block_size"]), "alpha": float(v["alpha"]),
                     "scale_format": v["scale_format"], "cases": cases})


def make_metrics() -> list:
    out = []
    g = torch.Generator().manual_seed(5)
    for n in (1, 17, 4096):
        x = torch.randn(n, generator=g).double()
        y = (x + torch.randn(n, generator=g) * 1e-2).float()
        out.append({"reference": x.float().tolist(), "emulated": y.tolist(), "expected": error_metrics(x.float(), y)})
    z = torch.zeros(8)
    out.append({"reference": z.tolist(), "emulated": z.tolist(), "expected": error_metrics(z, z)})
    return out


def main() -> None:
    HERE.mkdir(parents=True, exist_ok=True)
    for name, maker in (("cast", make_cast), ("quantize", make_quantize), ("mma", make_mma), ("nadpe", make_nadpe)):
        arrays, meta = {}, []
        maker(arrays, meta)
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
        (HERE / f"{name}.json").write_text(json.dumps(meta, indent=0))
        print(name, len(meta), "cases")
    (HERE / "metrics.json").write_text(json.dumps(make_metrics()))
    files = sorted(p.name for p in HERE.iterdir() if p.suffix in (".npz", ".json") and p.name != "MANIFEST.json")
    manifest = {f: hashlib.sha256((HERE / f).read_bytes()).hexdigest() for f in files}
    (HERE / "MANIFEST.json").write_text(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    main()
