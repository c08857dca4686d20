"""Tiny saved checkpoints with tile-map archives for the load-time apply tests."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch


def tiny_model(arch: str = "llama", tie: bool = True):
    torch.manual_seed(0)
    if arch == "llama":
        from transformers import LlamaConfig as Cfg, LlamaForCausalLM as Model

        cfg = Cfg(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, vocab_size=320, tie_word_embeddings=tie)
    else:
        from transformers import Qwen2Config as Cfg, Qwen2ForCausalLM as Model

        cfg = Cfg(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, vocab_size=320, tie_word_embeddings=tie)
    return Model(cfg).to(torch.bfloat16).eval()


def save_checkpoint(model, out_dir: Path, sharded: bool = True) -> Path:
    out_dir = Path(out_dir)
    model.save_pretrained(str(out_dir), max_shard_size="300KB" if sharded else "10GB")
    return out_dir


def keep_archive(model, keep_dir: Path, frac: float = 0.1, seed: int = 3, arch: str = "llama"):
    """Random kept-tile masks for every target projection, saved in the archive format;
    returns {layer name: kept ids (int32)}."""
    from tilequant_b200.mask_io import layer_name_to_stem, save_mask_keep_archive
    from tilequant_b200.rules import iter_target_linears
    from tilequant_b200.apply import default_cfg

    rng = np.random.default_rng(seed)
    masks, ids = {}, {}
    for _, _, name, lin in iter_target_linears(model, default_cfg(), model_type=arch):
        m, k = lin.weight.shape
        n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
        mask = (rng.random((n_tr, n_tc)) < frac).astype(np.uint8)
        masks[layer_name_to_stem(name)] = mask
        ids[name] = torch.from_numpy(np.flatnonzero(mask.reshape(-1)).astype(np.int32))
    save_mask_keep_archive(keep_dir, masks)
    return ids
