"""Host logic of the load-time apply (no GPU): shard resolution, the meta skeleton, the
tile-map coverage checks and tensor installation, against the reference's behaviour
(src/quantization/api.py:63-145)."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from tests.loader_fixtures import keep_archive, save_checkpoint, tiny_model
from tilequant_b200.loader import (ApplyConfig, TileConfig, load_iaa_channel_stats, make_cfg,
                                   parameters_on_meta, resolve_safetensor_shards, set_module_tensor,
                                   validate_fp16_ids_coverage_and_shapes)


def test_apply_config_and_cfg():
    ac = ApplyConfig(model_type="llama", dtype_out="bf16", quant_style="iaa", module_filters=["mlp"])
    cfg = make_cfg(ac)
    assert (cfg.tile_m, cfg.tile_n, cfg.dtype_out, cfg.quant_style, cfg.pad_to_tile) == (64, 64, "bf16", "iaa", True)
    assert cfg.module_filters == ["mlp"] and ac.tile == TileConfig()


def test_resolve_shards(tmp_path):
    model = tiny_model()
    d = save_checkpoint(model, tmp_path / "sharded")
    shards = list(resolve_safetensor_shards(d))
    index = json.loads((d / "model.safetensors.index.json").read_text())
    assert [p.name for p in shards] == sorted(set(index["weight_map"].values())) and len(shards) > 1
    single = save_checkpoint(model, tmp_path / "single", sharded=False)
    assert [p.name for p in resolve_safetensor_shards(single)] == ["model.safetensors"]
    (shards[0]).unlink()
    with pytest.raises(RuntimeError, match="Missing shard"):
        list(resolve_safetensor_shards(d))
    with pytest.raises(RuntimeError, match="No safetensors checkpoint"):
        list(resolve_safetensor_shards(tmp_path))


def test_skeleton_has_meta_parameters_and_host_buffers(tmp_path):
    from transformers import AutoConfig, AutoModelForCausalLM

    d = save_checkpoint(tiny_model(), tmp_path / "ckpt")
    with parameters_on_meta():
        sk = AutoModelForCausalLM.from_config(AutoConfig.from_pretrained(str(d)), dtype=torch.bfloat16)
    assert {p.device.type for p in sk.parameters()} == {"meta"}
    assert {b.device.type for b in sk.buffers()} == {"cpu"}
    # the hook is removed afterwards
    assert torch.nn.Linear(2, 2).weight.device.type == "cpu"
    w = torch.randn(320, 256, dtype=torch.bfloat16)
    set_module_tensor(sk, "model.embed_tokens.weight", "cpu", w)
    assert sk.model.embed_tokens.weight.device.type == "cpu" and torch.equal(sk.model.embed_tokens.weight, w)
    with pytest.raises(KeyError):
        set_module_tensor(sk, "model.embed_tokens.nothing", "cpu", w)


def test_coverage_checks(tmp_path):
    model = tiny_model()
    ids = keep_archive(model, tmp_path / "keep")
    ac = ApplyConfig(model_type="llama", dtype_out="bf16")
    data = validate_fp16_ids_coverage_and_shapes(model, tmp_path / "keep", ac)
    assert set(data) == set(ids)
    for name, (fp16, int8, n_tr, n_tc) in data.items():
        assert torch.equal(fp16, ids[name])
        assert fp16.numel() + int8.numel() == n_tr * n_tc
        assert not set(fp16.tolist()) & set(int8.tolist()) and torch.all(int8[1:] > int8[:-1])
    # an archive whose grid does not match the module
    from tilequant_b200.mask_io import save_mask_keep_archive

    bad = {k.replace(".", "_"): np.zeros((1, 1), np.uint8) for k in ids}
    save_mask_keep_archive(tmp_path / "bad", bad)
    with pytest.raises(RuntimeError, match="shape mismatch"):
        validate_fp16_ids_coverage_and_shapes(model, tmp_path / "bad", ac)
    with pytest.raises(FileNotFoundError):
        validate_fp16_ids_coverage_and_shapes(model, tmp_path / "nowhere", ac)


def test_iaa_stats_location(tmp_path):
    keep = tmp_path / "dec" / "tile_masks" / "keep10"
    keep.mkdir(parents=True)
    ac = ApplyConfig(model_type="llama", quant_style="iaa")
    with pytest.raises(FileNotFoundError):
        load_iaa_channel_stats(keep, ac)
    np.savez(tmp_path / "dec" / "iaa_channel_mean_abs.npz", model_layers_0_mlp_down_proj=np.ones(4, np.float64))
    stats = load_iaa_channel_stats(keep, ac)
    assert stats["model_layers_0_mlp_down_proj"].dtype == torch.float32
    other = tmp_path / "s.npz"
    np.savez(other, a=np.zeros(2, np.float32))
    assert set(load_iaa_channel_stats(keep, ApplyConfig(model_type="llama", iaa_channel_stats_path=str(other)))) == {"a"}
