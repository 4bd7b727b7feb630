"""TriCast's ``layer_report`` (``src/tricast/analysis.py:275-411``) end to end on a random-init
Qwen3-architecture model, with its per-layer weight / activation / output errors, MMA ULP errors and
model-level KL, top-1 agreement and perplexities: once with the recipe's layers on TriCast's
pure-PyTorch reference backend, once on this library installed as TriCast's GPU backend. The emulated
layers are bit-exact, so every number of the two reports must be identical. The library's launch
counter shows that the second report's layers ran on it.

TriCast itself is needed (installed offline into ``baseline/_ref``); without it these tests are skipped."""

from __future__ import annotations

import copy
import dataclasses
import sys
from pathlib import Path

import pytest
import torch

_REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
if _REF.is_dir() and str(_REF) not in sys.path:
    sys.path.append(str(_REF))
tricast = pytest.importorskip("tricast")
transformers = pytest.importorskip("transformers")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    torch.manual_seed(1)
    cfg = transformers.Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                                   max_position_embeddings=256, tie_word_embeddings=False)
    return transformers.Qwen3ForCausalLM(cfg).eval()


def _strip(report: dict) -> dict:
    """The report without the fields that describe the recipe object (its hash and the patch record
    cover the backend name, which is what differs)."""
    return {k: v for k, v in report.items() if k not in ("recipe_hash", "patch_report")}


@pytest.mark.parametrize("recipe", ["nvfp4_w_a", "mxfp4_w_a", "hopper_fp8_w8a8"])
def test_layer_report_on_library_equals_reference_backend(model, recipe):
    from tricast.analysis import layer_report
    from tricast.recipe import load_recipe

    from tricast_b200 import _native, backend

    backend.install()
    base = load_recipe(recipe)
    ids = torch.randint(0, 512, (1, 2 * 48), generator=torch.Generator().manual_seed(5))
    ref = layer_report(copy.deepcopy(model).cuda(), dataclasses.replace(base, backend="reference"), input_ids=ids,
                       samples=2, seqlen=48)
    launches = _native.lib().tc_launch_count()
    emu = layer_report(copy.deepcopy(model).cuda(), dataclasses.replace(base, backend="triton"), input_ids=ids,
                       samples=2, seqlen=48)
    assert _native.lib().tc_launch_count() - launches >= 2 * 14 * 2, "the report's layers did not run on tricast_b200"
    assert len(emu["layers"]) == 14 and all(e["status"] == "measured" for e in emu["layers"])
    names = lambda report: [name for name, _ in report["patch_report"]["patched"]]  # noqa: E731
    assert names(emu) == names(ref)
    assert _strip(emu) == _strip(ref)
