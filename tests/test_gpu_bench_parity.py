"""Bit-exact parity at benchmark size, on the benchmark's own seeded tensors.

``bench.py`` times configs 2-5 on the tensors of :mod:`tricast_b200.workloads` and
:func:`tricast_b200.sweep.make_layer`. These tests build the same tensors, run the same public calls
(``quantize_triton`` + ``gemm_triton`` on compact operands) at full size, and compare them bit for bit
with TriCast's own pure-PyTorch reference backend (``tricast.quantize`` / ``tricast.gemm`` with
``backend="reference"``, ``src/tricast/reference/{quantize,mma}.py``) run on the same GPU. The
reference gives the same bits on CUDA as on the CPU (TriCast's ``tests/gpu/test_reference_cuda.py``);
its GEMM keeps ``[rows, N, chunk]`` integer intermediates, so it runs on row slabs of A with all of B
and the whole K (every output is computed independently, ``reference/mma.py:340``).

* cfg2: every one of the 2048 x 4096 outputs.
* cfg3 and cfg4: row slabs spread over M (first, middle, last rows), full N and K.
* cfg5: one full-size layer (2048 tokens) of each of the five distinct Linear shapes, under all four
  formats, plus the fp64 reference output and the error sums.

Quantized operands are compared at full size first (values, scales, tensor scales). The exact-path
counters are reported: whole-GEMM fallbacks must not happen on these finite on-grid operands, and the
tensor-core GDFS kernel's exact tile steps (rare outputs whose K tile fails the single-pass bounds)
are counted; those outputs are part of the bit comparison like every other.

TriCast comes from ``baseline/_ref`` (installed offline with ``pip --target``); without it the tests
fall back to the numpy oracle on a few short row slabs.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from tricast_b200 import as_operand, gemm_triton, quantize_triton, workloads
from tricast_b200.mma import exact_fallbacks, exact_tile_steps
from tricast_b200.spec import PRESETS, SCHEMES

_REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
if _REF.is_dir() and str(_REF) not in sys.path:
    sys.path.append(str(_REF))
try:
    import tricast  # noqa: F401

    HAVE_TRICAST = True
except ImportError:  # pragma: no cover - depends on the box
    HAVE_TRICAST = False

pytestmark = pytest.mark.gpu


def mismatches(got: torch.Tensor, want: torch.Tensor) -> int:
    """Outputs whose bits differ (NaN equals NaN; the sign of zero counts), compared on the device."""
    got, want = got.float().contiguous(), want.to(got.device).float().contiguous()
    assert got.shape == want.shape, (got.shape, want.shape)
    same = (got.view(torch.int32) == want.view(torch.int32)) | (torch.isnan(got) & torch.isnan(want))
    return int((~same).sum().item())


def first_bad(got: torch.Tensor, want: torch.Tensor) -> str:
    got, want = got.float(), want.to(got.device).float()
    bad = ~((got.view(torch.int32) == want.view(torch.int32)) | (torch.isnan(got) & torch.isnan(want)))
    idx = bad.nonzero()[:3].tolist()
    return "; ".join(f"{tuple(i)}: got {got[tuple(i)].item()!r} want {want[tuple(i)].item()!r}" for i in idx)


def assert_qtensor_equal(ours, ref, what: str) -> None:
    assert mismatches(ours.values.float(), ref.values.float()) == 0, f"{what}: quantized values differ"
    for field in ("scale", "zero_point", "global_scale"):
        a, b = getattr(ours, field, None), getattr(ref, field, None)
        assert (a is None) == (b is None), f"{what}: {field} presence differs"
        if a is not None:
            assert mismatches(a.float().reshape(b.shape), b.float()) == 0, f"{what}: {field} differs"


# ----------------------------------------------------------------------------- reference side
def t_rows(op, r0: int, r1: int):
    """Rows r0..r1 of a TriCast Operand (values and per-row / K scales sliced, the rest shared)."""
    from tricast.mma.operand import Operand

    scale = op.scale
    if scale is not None and op.scale_kind in ("row", "k"):
        scale = scale[r0:r1]
    return Operand(op.values[r0:r1], op.fmt, scale, op.scale_fmt, op.scale_kind, op.k_domain, op.alpha)


def ref_gemm_rows(ta, tb, spec, r0: int, r1: int, step: int) -> torch.Tensor:
    from tricast.mma.api import gemm

    parts = [gemm(t_rows(ta, s, min(s + step, r1)), tb, spec, backend="reference") for s in range(r0, r1, step)]
    return torch.cat(parts)


def check_rows(out: torch.Tensor, ta, tb, spec, slabs, step: int, what: str) -> None:
    for r0, r1 in slabs:
        want = ref_gemm_rows(ta, tb, spec, r0, r1, step)
        bad = mismatches(out[r0:r1], want)
        assert bad == 0, f"{what} rows {r0}..{r1}: {bad} outputs differ ({first_bad(out[r0:r1], want)})"


# ----------------------------------------------------------------------------- oracle fallback
def check_rows_oracle(out: torch.Tensor, a, b, spec, slabs, what: str) -> None:
    import oracle

    class Rows:
        def __init__(self, op, r0, r1):
            self.values = op.values[r0:r1].float().cpu().numpy()
            self.fmt, self.scale_fmt, self.scale_kind, self.k_domain = op.fmt, op.scale_fmt, op.scale_kind, op.k_domain
            s = op.scale
            if s is not None and op.scale_kind in ("row", "k"):
                s = s[r0:r1]
            self.scale = None if s is None else s.float().cpu().numpy()
            self.alpha = None if op.alpha is None else np.float32(op.alpha.item())
            self.rows, self.K = self.values.shape

    bb = Rows(b, 0, b.rows)
    for r0, r1 in slabs:
        want = oracle.gemm_reference(Rows(a, r0, r1), bb, spec)
        got = out[r0:r1].float().cpu().numpy()
        same = (got.view(np.uint32) == want.astype(np.float32).view(np.uint32)) | (np.isnan(got) & np.isnan(want))
        assert same.all(), f"{what} rows {r0}..{r1}: {(~same).sum()} outputs differ from the oracle"


def spread(m: int, rows: int, count: int) -> list[tuple[int, int]]:
    """``count`` slabs of ``rows`` rows: the first, evenly spaced middle ones, the last."""
    starts = sorted({round(i * (m - rows) / (count - 1)) // 8 * 8 for i in range(count)})
    starts[-1] = m - rows
    return [(s, s + rows) for s in starts]


# ----------------------------------------------------------------------------- cfg2
def test_cfg2_every_output_matches_tricast():
    m, n, k = workloads.CFG2_SHAPE
    a_cpu, b_cpu = workloads.cfg2_inputs()
    a, b = a_cpu.cuda(), b_cpu.cuda()
    spec = PRESETS["nvidia_blackwell_fp4"].with_(out_format="fp32")
    qa, qb = quantize_triton(a, SCHEMES["nvfp4"]), quantize_triton(b, SCHEMES["nvfp4"])
    f0, s0 = exact_fallbacks(), exact_tile_steps()
    out = gemm_triton(as_operand(qa, compact=True), as_operand(qb, compact=True), spec)
    torch.cuda.synchronize()
    assert exact_fallbacks() == f0, "the fast kernel declined the benchmark operands"
    steps = exact_tile_steps() - s0
    print(f"cfg2: {steps} of {m * n * (k // 64)} (output, K tile) steps took the exact two-pass step")
    assert out.shape == (m, n)
    if not HAVE_TRICAST:
        check_rows_oracle(out, as_operand(qa), as_operand(qb), spec, spread(m, 4, 3), "cfg2")
        return
    import tricast
    from tricast.mma.api import as_operand as t_as_operand

    ta, tb = tricast.quantize(a, "nvfp4", backend="reference"), tricast.quantize(b, "nvfp4", backend="reference")
    assert_qtensor_equal(qa, ta, "cfg2 A")
    assert_qtensor_equal(qb, tb, "cfg2 B")
    check_rows(out, t_as_operand(ta), t_as_operand(tb), {"preset": "nvidia_blackwell_fp4", "out_format": "fp32"},
               [(0, m)], 128, "cfg2")


# ----------------------------------------------------------------------------- cfg3
def test_cfg3_row_slabs_match_tricast():
    m, n, k = workloads.CFG3_SHAPE
    a_cpu, b_cpu = workloads.cfg3_inputs()
    a, b = a_cpu.cuda(), b_cpu.cuda()
    spec = PRESETS["nvidia_hopper_fp8"].with_(out_format="fp32")
    qa, qb = quantize_triton(a, SCHEMES["fp8_tensor"]), quantize_triton(b, SCHEMES["fp8_tensor"])
    f0 = exact_fallbacks()
    out = gemm_triton(as_operand(qa, compact=True), as_operand(qb, compact=True), spec)
    torch.cuda.synchronize()
    assert exact_fallbacks() == f0
    if not HAVE_TRICAST:
        check_rows_oracle(out, as_operand(qa), as_operand(qb), spec, spread(m, 1, 2), "cfg3")
        return
    import tricast
    from tricast.mma.api import as_operand as t_as_operand

    ta = tricast.quantize(a, "fp8_tensor", backend="reference")
    tb = tricast.quantize(b, "fp8_tensor", backend="reference")
    assert_qtensor_equal(qa, ta, "cfg3 A")
    assert_qtensor_equal(qb, tb, "cfg3 B")
    check_rows(out, t_as_operand(ta), t_as_operand(tb), {"preset": "nvidia_hopper_fp8", "out_format": "fp32"},
               spread(m, 64, 8), 32, "cfg3")


# ----------------------------------------------------------------------------- cfg4
def test_cfg4_row_slabs_match_tricast():
    m, n, k = workloads.CFG4_SHAPE
    x_cpu, w_cpu = workloads.cfg4_inputs()
    x, w = x_cpu.cuda(), w_cpu.cuda()
    qa, qw = quantize_triton(x, SCHEMES["int8_row"]), quantize_triton(w, SCHEMES["int4_g128_zp"])
    opa, opb = workloads.cfg4_operands(qa, qw)
    spec = workloads.cfg4_spec()
    f0 = exact_fallbacks()
    out = gemm_triton(opa, opb, spec)
    torch.cuda.synchronize()
    assert exact_fallbacks() == f0
    if not HAVE_TRICAST:
        check_rows_oracle(out, opa, opb, spec, spread(m, 2, 2), "cfg4")
        return
    import tricast
    from tricast.formats import FP16, IntFormat
    from tricast.mma.api import as_operand as t_as_operand
    from tricast.mma.operand import Operand
    from tricast.mma.spec import MMASpec

    ta = tricast.quantize(x, "int8_row", backend="reference")
    tw = tricast.quantize(w, "int4_g128_zp", backend="reference")
    assert_qtensor_equal(qa, ta, "cfg4 A")
    assert_qtensor_equal(qw, tw, "cfg4 W")
    tb = Operand(tw.values.float() - tw.zero_point.repeat_interleave(128, dim=1), IntFormat("int5", 5), tw.scale,
                 FP16, "k", 128)
    tspec = MMASpec("cofda", f_bits=23, chunk_size=32, promote_interval=128, out_format="fp32")
    check_rows(out, t_as_operand(ta), tb, tspec, spread(m, 128, 8), 32, "cfg4")


# ----------------------------------------------------------------------------- cfg5
# The first layer of each distinct Linear shape of the sweep: q (1024->2048), k (1024->1024),
# o (2048->1024), gate (1024->3072), down (3072->1024); v and up repeat k and gate.
SWEEP_SHAPES = [0, 1, 3, 4, 6]


@pytest.mark.parametrize("index", SWEEP_SHAPES)
def test_cfg5_full_layer_matches_tricast(index):
    from tricast_b200 import sweep

    cfg = sweep.SweepConfig()
    entry = cfg.layers()[index]
    _, name, fin, fout = entry
    dev = torch.device("cuda", torch.cuda.current_device())
    x, w = sweep.make_layer(index, fin, fout, cfg.tokens, dev)
    f0 = exact_fallbacks()
    ours = {fmt: sweep.emulate(x, w, fmt) for fmt in sweep.FORMATS}
    ref64 = sweep.reference(x, w)
    torch.cuda.synchronize()
    assert exact_fallbacks() == f0, f"{name}: a fast kernel declined the sweep operands"
    sums = sweep.run_layers([entry], cfg, dev)[0]  # what the benchmark reduces, [formats, 6]

    if not HAVE_TRICAST:
        import oracle

        want = oracle.gemm_reference(as_operand(x[:2]), as_operand(w), sweep.MMASpec("fp64", out_format="fp32"))
        assert mismatches(ref64[:2], torch.from_numpy(np.ascontiguousarray(want))) == 0
        return
    import tricast
    from tricast.formats import FP16, IntFormat
    from tricast.mma.api import as_operand as t_as_operand
    from tricast.mma.operand import Operand
    from tricast.mma.spec import MMASpec

    t_ref = ref_gemm_rows(t_as_operand(x), t_as_operand(w), MMASpec("fp64", out_format="fp32"), 0, cfg.tokens, 512)
    assert mismatches(ref64, t_ref) == 0, f"{name} fp64 reference: {first_bad(ref64, t_ref)}"
    for col, fmt in enumerate(sweep.FORMATS):
        if fmt == "int4_g128":
            ta = tricast.quantize(x, "int8_row", backend="reference")
            tw = tricast.quantize(w, "int4_g128_zp", backend="reference")
            tb = Operand(tw.values.float() - tw.zero_point.repeat_interleave(128, dim=1)[:, :fin],
                         IntFormat("int5", 5), tw.scale, FP16, "k", 128)
            ta_op, spec, step = t_as_operand(ta), MMASpec("cofda", f_bits=23, chunk_size=32, promote_interval=128,
                                                          out_format="fp32"), 128
        else:
            scheme, preset = {"mxfp4": ("mxfp4", "nvidia_blackwell_fp4"), "nvfp4": ("nvfp4", "nvidia_blackwell_fp4"),
                              "fp8_e4m3": ("fp8_tensor", "nvidia_hopper_fp8")}[fmt]
            ta = tricast.quantize(x, scheme, backend="reference")
            tw = tricast.quantize(w, scheme, backend="reference")
            ta_op, tb, spec, step = t_as_operand(ta), t_as_operand(tw), preset, 128
        want = ref_gemm_rows(ta_op, tb, spec, 0, cfg.tokens, step)
        got = ours[fmt]
        assert got.dtype == want.dtype, (fmt, got.dtype, want.dtype)
        bad = mismatches(got, want)
        assert bad == 0, f"{name} {fmt}: {bad} of {got.numel()} outputs differ ({first_bad(got, want)})"
        # The error sums the sweep reports, against fp64 sums over TriCast's outputs (the reduction
        # order differs, hence the 1e-12 relative bound; the max is exact).
        r, e = t_ref.double(), want.double()
        expect = [float((r * r).sum()), float((e * e).sum()), float(((r - e) ** 2).sum()), float((r * e).sum()),
                  float((r - e).abs().max())]
        for field, (a, b) in enumerate(zip(sums[col, :5].tolist(), expect)):
            assert abs(a - b) <= 1e-12 * max(abs(b), 1e-300), (name, fmt, sweep.METRIC_FIELDS[field], a, b)
        assert sums[col, 5].item() == 0
