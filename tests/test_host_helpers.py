"""Small host-side helpers of the package (no GPU): padding, target-name filters, tile
grids, archive lookups, the row-major pack check and the CUDA-only guard."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from tilequant_b200 import _native as N
from tilequant_b200.apply import default_cfg, tile_grid
from tilequant_b200.mask_io import archive_path, load_mask_keep_for_layer, load_mask_keep_stem_dict, \
    save_mask_keep_archive
from tilequant_b200.pack import is_row_major_pack
from tilequant_b200.quant_utils import pad_to_multiple
from tilequant_b200.rules import should_quantize_name


def test_pad_to_multiple():
    w = torch.arange(6, dtype=torch.float32).reshape(2, 3)
    p, m, k = pad_to_multiple(w, 4)
    assert (m, k) == (4, 4) and p.shape == (4, 4) and torch.equal(p[:2, :3], w) and float(p[2:].abs().sum()) == 0
    same, m, k = pad_to_multiple(torch.zeros(64, 128), 64)
    assert (m, k) == (64, 128) and same.shape == (64, 128)
    with pytest.raises(ValueError):
        pad_to_multiple(torch.zeros(3), 64)


def test_should_quantize_name_filters():
    assert should_quantize_name("model.layers.0.mlp.down_proj", {"module_filters": []})
    cfg = SimpleNamespace(module_filters=["*.mlp.*"])
    assert should_quantize_name("model.layers.3.mlp.up_proj", cfg)
    assert not should_quantize_name("model.layers.3.self_attn.q_proj", cfg)


def test_tile_grid_rounds_up():
    assert tile_grid(torch.zeros(130, 64), default_cfg()) == (3, 1)
    assert tile_grid(torch.zeros(64, 65), default_cfg()) == (1, 2)


def test_archive_lookups(tmp_path):
    masks = {"model_layers_0_self_attn_q_proj": np.eye(3, dtype=np.uint8),
             "model_layers_0_mlp_down_proj": np.zeros((2, 5), np.uint8)}
    path = save_mask_keep_archive(tmp_path, masks)
    assert path == archive_path(tmp_path) and path.name == "fp16_keep_ids_tile64x64.npz"
    m = load_mask_keep_for_layer(tmp_path, "model.layers.0.self_attn.q_proj")
    assert m.dtype == torch.uint8 and torch.equal(m, torch.eye(3, dtype=torch.uint8))
    d = load_mask_keep_stem_dict(tmp_path)
    assert set(d) == set(masks) and int(d["model_layers_0_mlp_down_proj"].sum()) == 0
    with pytest.raises(ValueError):
        save_mask_keep_archive(tmp_path, {"x": np.full((2, 2), 2, np.uint8)})  # not a 0/1 mask


def test_row_major_pack_check():
    ok = SimpleNamespace(int8_tile_ids=torch.tensor([0, 2, 5]), fp16_tile_ids=torch.tensor([1]))
    bad = SimpleNamespace(int8_tile_ids=torch.tensor([0, 5, 2]), fp16_tile_ids=torch.tensor([], dtype=torch.int32))
    assert is_row_major_pack(ok) and not is_row_major_pack(bad)


def test_cuda_only_guard():
    with pytest.raises(ValueError, match="CUDA"):
        N.require_cuda(torch.zeros(2))
    assert N.require_cuda(None) is None
