"""Decision-directory writing (no GPU): top-k archives per keep fraction in the
reference's layout (src/quantization/decisions.py:174-224), readable by the loader."""

from __future__ import annotations

import json
import math

import numpy as np
import pytest

from tests.loader_fixtures import save_checkpoint, tiny_model
from tilequant_b200.decisions import DEFAULT_KEEP_FRACS, infer_model_type, keep_tag, save_masks, score_npz_path
from tilequant_b200.mask_io import load_fp16_keep_ids_for_layer


def test_keep_tags_and_paths(tmp_path):
    assert [keep_tag(f) for f in DEFAULT_KEEP_FRACS] == ["keep01", "keep02", "keep05", "keep10", "keep20"]
    assert score_npz_path(tmp_path, "iaa").name == "iaa_tile_scores_tile64x64.npz"


def test_save_masks_topk_per_fraction(tmp_path):
    rng = np.random.default_rng(0)
    scores = {"model_layers_0_self_attn_q_proj": rng.random((4, 4)).astype(np.float32),
              "model_layers_0_mlp_down_proj": rng.random((4, 11)).astype(np.float32)}
    dirs = save_masks(tmp_path, scores, DEFAULT_KEEP_FRACS, "tiny", "synthetic", "-", "gi")
    for frac, d in dirs.items():
        meta = json.loads((d / "meta.json").read_text())
        assert meta["keep_frac"] == frac and meta["mask_rule"] == "topk_by_importance" and meta["quant_style"] == "gi"
        for stem, s in scores.items():
            ids, grid = load_fp16_keep_ids_for_layer(d, stem.replace("_", "."))  # stems map back to names
            assert grid == s.shape
            k = max(1, math.ceil(frac * s.size))
            assert ids.numel() == k
            kept = set(ids.tolist())
            flat = s.reshape(-1)
            assert min(flat[list(kept)]) >= max([flat[i] for i in range(s.size) if i not in kept], default=-1.0)


def test_infer_model_type(tmp_path):
    assert infer_model_type(save_checkpoint(tiny_model("llama"), tmp_path / "l", sharded=False)) == "llama"
    assert infer_model_type(save_checkpoint(tiny_model("qwen2"), tmp_path / "q", sharded=False)) == "qwen"
    (tmp_path / "x").mkdir()
    (tmp_path / "x" / "config.json").write_text(json.dumps({"model_type": "gpt2"}))
    with pytest.raises(RuntimeError):
        infer_model_type(tmp_path / "x")


def test_resolve_decision_and_keep_dirs(tmp_path):
    import os
    import time

    from tilequant_b200.decisions import resolve_decision_and_keep_dir, resolve_decision_dir, resolve_keep_dir

    with pytest.raises(RuntimeError, match="Decision directory not found"):
        resolve_decision_dir(tmp_path / "Model-X", "gi", tmp_path / "Decision")
    d = tmp_path / "Decision" / "Model-X" / "gi"
    (d / "tile_masks" / "keep01").mkdir(parents=True)
    (d / "tile_masks" / "keep05").mkdir()
    (d / "tile_masks" / "other").mkdir()
    t = time.time()
    os.utime(d / "tile_masks" / "keep01", (t - 100, t - 100))
    os.utime(d / "tile_masks" / "keep05", (t, t))
    assert resolve_decision_dir(tmp_path / "Model-X", "GI", tmp_path / "Decision") == d.resolve()
    assert resolve_keep_dir(d).name == "keep05"  # the newest keepNN
    assert resolve_keep_dir(d, "keep01").name == "keep01"
    with pytest.raises(RuntimeError, match="Requested keep dir not found"):
        resolve_keep_dir(d, "keep99")
    dd, kd = resolve_decision_and_keep_dir(tmp_path / "Model-X", "gi", "keep01", tmp_path / "Decision")
    assert (dd, kd.name) == (d.resolve(), "keep01")


def test_ensure_decision_artifacts_resolves_or_asks_for_batches(tmp_path):
    from tilequant_b200.decisions import ensure_decision_artifacts

    model_dir = tmp_path / "Model-Y"
    model_dir.mkdir()
    root = tmp_path / "Decision"
    with pytest.raises(RuntimeError, match="no calibration batches"):
        ensure_decision_artifacts(model_dir, "gi", "keep01", root)
    d = root / "Model-Y" / "iaa"
    (d / "tile_masks" / "keep01").mkdir(parents=True)
    with pytest.raises(RuntimeError, match="no calibration batches"):  # IAA needs its channel statistics
        ensure_decision_artifacts(model_dir, "iaa", "keep01", root)
    np.savez(d / "iaa_channel_mean_abs.npz", a=np.ones(2, np.float32))
    md, dd, kd = ensure_decision_artifacts(model_dir, "iaa", "keep01", root)
    assert (md, dd, kd.name) == (model_dir, d.resolve(), "keep01")
    with pytest.raises(RuntimeError, match="no calibration batches"):  # a keep dir that is not there
        ensure_decision_artifacts(model_dir, "iaa", "keep05", root)
