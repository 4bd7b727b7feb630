"""TriCast's own model flow on this library: ``patch_model`` on a random-init Qwen3-architecture model
with TriCast's shipped recipes, run once on TriCast's pure-PyTorch reference backend and once on
tricast_b200 installed as TriCast's GPU backend (``tricast_b200.install()``); the logits must agree bit
for bit. Every linear layer of the model goes through the library's quantize and GEMM entry points as
TriCast calls them (its EmuLinear, its packed weight operands, its dispatcher). 8 tokens exercise the
small-M kernels, 40 tokens the tiled and tensor-core kernels.

TriCast itself is needed (installed offline into ``baseline/_ref`` with ``pip --target``); without it
these tests are skipped."""

from __future__ import annotations

import copy
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

RECIPES = ["nvfp4_w_a", "mxfp4_w_a", "nvfp4_4o6", "hopper_fp8_w8a8", "ada_fp8_w8a8", "blackwell_fp8_w8a8",
           "fp8_f7_decoupled", "deepseek_fp8_block", "mxfp8_w_a", "int8_row_w8a8"]


@pytest.fixture(scope="module")
def model():
    torch.manual_seed(0)
    cfg = transformers.Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                                   max_position_embeddings=128, tie_word_embeddings=False)
    return transformers.Qwen3ForCausalLM(cfg).eval()


@pytest.mark.parametrize("tokens", [8, 40])
@pytest.mark.parametrize("recipe", RECIPES)
def test_patched_model_matches_reference_backend(model, recipe, tokens):
    from tricast.nn.patch import patch_model

    from tricast_b200 import backend

    backend.install()
    ids = torch.randint(0, 512, (1, tokens), generator=torch.Generator().manual_seed(tokens)).cuda()
    ref = copy.deepcopy(model).cuda()
    report = patch_model(ref, recipe, backend="reference")
    emu = copy.deepcopy(model).cuda()
    patch_model(emu, recipe, backend="triton")  # TriCast's GPU backend slot, served by tricast_b200
    assert len(report.patched) == 14
    from tricast_b200 import _native

    with torch.no_grad():
        want = ref(ids).logits
        launches = _native.lib().tc_launch_count()
        got = emu(ids).logits
    assert _native.lib().tc_launch_count() - launches >= 2 * 14, "the patched layers did not run on tricast_b200"
    assert torch.isfinite(want).all()
    mismatch = (got.view(torch.int32) != want.view(torch.int32)).sum().item()
    assert mismatch == 0, f"{recipe}, {tokens} tokens: {mismatch} of {want.numel()} logits differ"
