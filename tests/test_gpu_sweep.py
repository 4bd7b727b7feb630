"""GPU parity of the per-layer error sweep on a reduced model (1 block, dimensions / 8, 64 tokens):
every emulated layer output bit-exact with the CPU oracle, every metric within 1e-12 relative
(fp64 sums reduced in a different order)."""

from __future__ import annotations

import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle
from oracle import metrics as oracle_metrics
from oracle.quantize import quantize_reference
from tests.conftest import bits_equal
from tricast_b200.formats import BF16, FP16, IntFormat
from tricast_b200.spec import PRESETS, SCHEMES, MMASpec
from tricast_b200.sweep import FORMATS, SweepConfig, emulate, make_layer, reference, run_sweep

pytestmark = pytest.mark.gpu


def _op(q, spec):
    if spec.scale is None:
        return SimpleNamespace(values=q.values, fmt=spec.format, scale=None, scale_fmt=None, scale_kind="none",
                               k_domain=0, alpha=None)
    if spec.granularity == "group":
        return SimpleNamespace(values=q.values, fmt=spec.format, scale=q.scale, scale_fmt=spec.scale.format,
                               scale_kind="k", k_domain=spec.group_size, alpha=q.global_scale)
    kind = "tensor" if spec.granularity == "tensor" else "row"
    return SimpleNamespace(values=q.values, fmt=spec.format, scale=np.asarray(q.scale), scale_fmt=None,
                           scale_kind=kind, k_domain=0, alpha=None)


def oracle_emulate(x: np.ndarray, w: np.ndarray, fmt: str) -> np.ndarray:
    if fmt == "int4_g128":
        qa = quantize_reference(x, SCHEMES["int8_row"])
        qw = quantize_reference(w, SCHEMES["int4_g128_zp"])
        zeros = np.repeat(qw.zero_point, 128, axis=1)[:, : w.shape[1]]
        b = SimpleNamespace(values=(qw.values - zeros).astype(np.float32), fmt=IntFormat("int5", 5), scale=qw.scale,
                            scale_fmt=FP16, scale_kind="k", k_domain=128, alpha=None)
        spec = MMASpec("cofda", f_bits=23, chunk_size=32, promote_interval=128, out_format="fp32")
        return oracle.gemm_reference(_op(qa, SCHEMES["int8_row"]), b, spec)
    scheme, preset = {"mxfp4": ("mxfp4", "nvidia_blackwell_fp4"), "nvfp4": ("nvfp4", "nvidia_blackwell_fp4"),
                      "fp8_e4m3": ("fp8_tensor", "nvidia_hopper_fp8")}[fmt]
    spec = SCHEMES[scheme]
    qa, qw = quantize_reference(x, spec), quantize_reference(w, spec)
    return oracle.gemm_reference(_op(qa, spec), _op(qw, spec), PRESETS[preset])


def test_mini_sweep_matches_oracle():
    cfg = SweepConfig(blocks=1, tokens=64, hidden_scale=8)
    dev = torch.device("cuda", 0)
    for index, _name, fin, fout in cfg.layers():
        x, w = make_layer(index, fin, fout, cfg.tokens, dev)
        xn, wn = x.float().cpu().numpy(), w.float().cpu().numpy()
        ref_dev = reference(x, w).cpu().numpy()
        plain = SimpleNamespace(values=xn, fmt=BF16, scale=None, scale_fmt=None, scale_kind="none", k_domain=0,
                                alpha=None)
        wplain = SimpleNamespace(values=wn, fmt=BF16, scale=None, scale_fmt=None, scale_kind="none", k_domain=0,
                                 alpha=None)
        ref_oracle = oracle.gemm_reference(plain, wplain, MMASpec("fp64", out_format="fp32"))
        assert bits_equal(ref_dev, ref_oracle)
        for fmt in FORMATS:
            got = emulate(x, w, fmt).float().cpu().numpy()
            want = oracle_emulate(xn, wn, fmt)
            assert bits_equal(got, want), (index, fmt)
    records, secs = run_sweep(cfg)
    assert secs > 0 and len(records) == 7
    for rec in records:
        index = rec["layer"]
        _, _, fin, fout = cfg.layers()[index]
        x, w = make_layer(index, fin, fout, cfg.tokens, dev)
        xn, wn = x.float().cpu().numpy(), w.float().cpu().numpy()
        ref = reference(x, w).cpu().numpy()
        for fmt in FORMATS:
            want = oracle_metrics.error_metrics(ref, oracle_emulate(xn, wn, fmt))
            for key, value in want.items():
                got = rec[fmt][key]
                if isinstance(value, str):
                    assert got == value
                else:
                    assert math.isclose(got, value, rel_tol=1e-12, abs_tol=1e-300), (index, fmt, key, got, value)


def test_sweep_resume_skips_recorded_layers(tmp_path):
    cfg = SweepConfig(blocks=1, tokens=32, hidden_scale=8)
    first, _ = run_sweep(cfg, out_dir=str(tmp_path))
    files = sorted(tmp_path.glob("layer_*.json"))
    assert len(files) == 7
    stamp = [f.stat().st_mtime_ns for f in files]
    second, _ = run_sweep(cfg, out_dir=str(tmp_path))
    assert [f.stat().st_mtime_ns for f in files] == stamp  # nothing recomputed or rewritten
    assert first == second


def test_graph_replay_equals_eager_pass():
    """Each layer replayed from its shape's captured graph (static buffers refilled per layer) gives the
    eager pass's sums; layers of one shape share one graph."""
    from tricast_b200.sweep import _GRAPHS, release_graphs, run_layers

    cfg = SweepConfig(blocks=2, tokens=64, hidden_scale=8)
    dev = torch.device("cuda", 0)
    release_graphs()
    graphed = run_layers(cfg.layers(), cfg, dev, graphs=True)
    assert len(_GRAPHS) == 5  # distinct (in, out) shapes of the 14 layers
    eager = run_layers(cfg.layers(), cfg, dev, graphs=False)
    torch.cuda.synchronize()
    assert torch.allclose(graphed, eager, rtol=1e-12, atol=0)
    assert torch.equal(graphed[..., 4], eager[..., 4])  # the max is order-free
    release_graphs()
