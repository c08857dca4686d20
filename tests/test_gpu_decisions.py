"""Calibration to decision directory to load-time apply, on the GPU: GI and IAA scores
collected over random-id batches are written as the reference's decision layout, and the
keep10 archive loads (with the IAA channel statistics found beside it) to the same
model as applying the top-10 % maps of the saved scores in memory."""

from __future__ import annotations

import json

import pytest
import torch

from tests.loader_fixtures import save_checkpoint, tiny_model
from tilequant_b200.apply import apply_tile_maps
from tilequant_b200.calibrate import keep_ids_from_scores
from tilequant_b200.decisions import build_decisions_from_batches, load_npz_map, score_npz_path
from tilequant_b200.loader import ApplyConfig, load_mixed_precision_model_from_masks, make_cfg

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("arch,style", [("llama", "gi"), ("qwen2", "iaa")])
def test_decisions_round_trip(cuda_device, tmp_path, arch, style):
    dense = tiny_model(arch, tie=False)
    ckpt = save_checkpoint(dense, tmp_path / "ckpt", sharded=False)
    calib_model = dense.to(cuda_device)
    gen = torch.Generator().manual_seed(11)
    batches = [{"input_ids": torch.randint(0, 320, (2, 48), generator=gen)} for _ in range(3)]
    ddir = build_decisions_from_batches(calib_model, batches, tmp_path / "dec" / style, quant_style=style,
                                        model_type=arch, model_name_or_path="tiny")
    meta = json.loads((ddir / "decision_meta.json").read_text())
    assert meta["quant_style"] == style and meta["num_targets"] == 14
    assert (ddir / "decision_ready.flag").read_text() == "done\n"
    assert not list(ddir.glob("*progress*.pt"))
    scores = load_npz_map(score_npz_path(ddir, style))
    mtime = score_npz_path(ddir, style).stat().st_mtime_ns
    build_decisions_from_batches(calib_model, batches, ddir, quant_style=style, model_type=arch)  # reuses scores
    assert score_npz_path(ddir, style).stat().st_mtime_ns == mtime
    del calib_model, dense

    ac = ApplyConfig(model_type=arch, dtype_out="bf16", quant_style=style)
    model, _ = load_mixed_precision_model_from_masks(ckpt, ddir / "tile_masks" / "keep10", ac, torch.bfloat16,
                                                     cuda_device)
    from transformers import AutoModelForCausalLM

    ref = AutoModelForCausalLM.from_pretrained(str(ckpt), dtype=torch.bfloat16).to(cuda_device).eval()
    names = [n for n, m in ref.named_modules() if n.replace(".", "_") in scores]
    keep = keep_ids_from_scores({n: torch.from_numpy(scores[n.replace(".", "_")]) for n in names}, 0.10)
    stats = None
    if style == "iaa":
        raw = load_npz_map(ddir / "iaa_channel_mean_abs.npz")
        stats = {n: torch.from_numpy(raw[n.replace(".", "_")]) for n in names}
    apply_tile_maps(ref, keep, make_cfg(ac), model_type=arch, iaa_channel_stats=stats)
    ids = torch.randint(0, 320, (2, 32), generator=torch.Generator().manual_seed(12)).to(cuda_device)
    with torch.inference_mode():
        assert torch.equal(model(input_ids=ids).logits, ref(input_ids=ids).logits)
