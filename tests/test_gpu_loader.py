"""Load-time apply on the GPU: a saved checkpoint loaded with its tile-map archive
(``load_mixed_precision_model_from_masks``) equals the dense model with the same maps
applied in memory -- the same packs and therefore the same logits, bit for bit -- for
a tied Llama (sharded checkpoint, GI scales) and a Qwen2 with Q/K/V biases (single
file, IAA scales from the decision directory's channel statistics)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.loader_fixtures import keep_archive, save_checkpoint, tiny_model
from tilequant_b200.apply import apply_tile_maps
from tilequant_b200.loader import ApplyConfig, load_mixed_precision_model_from_masks, make_cfg
from tilequant_b200.mixed_linear import MixedLinear

pytestmark = pytest.mark.gpu

STATS_KEYS = {"num_targets", "num_replaced", "num_replaced_during_load", "num_loaded_non_target_tensors",
              "load_total", "quant_pack_total", "non_target_load_total", "attn_implementation",
              "fused_projection_groups"}


@pytest.mark.parametrize("arch,tie,sharded,style", [("llama", True, True, "gi"), ("qwen2", False, False, "iaa")])
def test_load_time_apply_equals_in_memory_apply(cuda_device, tmp_path, arch, tie, sharded, style):
    from transformers import AutoModelForCausalLM

    dense = tiny_model(arch, tie)
    if arch == "qwen2":
        with torch.no_grad():  # non-zero Q/K/V biases, so the bias path is exercised
            for layer in dense.model.layers:
                for proj in (layer.self_attn.q_proj, layer.self_attn.k_proj, layer.self_attn.v_proj):
                    proj.bias.normal_(0.0, 0.5)
    ckpt = save_checkpoint(dense, tmp_path / "ckpt", sharded=sharded)
    keep_dir = tmp_path / "dec" / "tile_masks" / "keep10"
    ids = keep_archive(dense, keep_dir, 0.1, arch=arch)
    stats = None
    if style == "iaa":
        rng = np.random.default_rng(5)
        stats = {name: rng.random(dense.get_submodule(name).weight.shape[1]).astype(np.float32) + 0.01 for name in ids}
        np.savez(tmp_path / "dec" / "iaa_channel_mean_abs.npz", **{n.replace(".", "_"): v for n, v in stats.items()})
    ac = ApplyConfig(model_type=arch, dtype_out="bf16", quant_style=style)
    model, info = load_mixed_precision_model_from_masks(ckpt, keep_dir, ac, torch.bfloat16, cuda_device,
                                                        attn_implementation="sdpa")
    assert set(info) == STATS_KEYS
    assert info["num_targets"] == info["num_replaced"] == info["num_replaced_during_load"] == len(ids)
    assert all(p.device == cuda_device for p in model.parameters())
    assert all(b.device == cuda_device for b in model.buffers())

    ref = AutoModelForCausalLM.from_pretrained(str(ckpt), dtype=torch.bfloat16, attn_implementation="sdpa")
    ref = ref.to(cuda_device).eval()
    apply_tile_maps(ref, ids, make_cfg(ac), model_type=arch,
                    iaa_channel_stats=None if stats is None else {n: torch.from_numpy(v) for n, v in stats.items()})
    for name, mod in model.named_modules():
        if isinstance(mod, MixedLinear):
            other = ref.get_submodule(name)
            for buf in ("int8_tiles", "int8_scales", "int8_tile_ids", "fp16_tiles", "fp16_tile_ids"):
                assert torch.equal(getattr(mod, buf), getattr(other, buf)), (name, buf)
            assert (mod.bias is None) == (other.bias is None)
            if mod.bias is not None:
                assert torch.equal(mod.bias, other.bias)
    ids_in = torch.randint(0, 320, (2, 40), generator=torch.Generator().manual_seed(7)).to(cuda_device)
    with torch.inference_mode():
        got = model(input_ids=ids_in).logits
        want = ref(input_ids=ids_in).logits
    assert torch.equal(got, want)
