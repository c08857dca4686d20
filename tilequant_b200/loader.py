"""Load-time apply over a safetensors checkpoint: the reference's
``load_mixed_precision_model_from_masks`` (src/quantization/api.py:154-310) and its
helpers, for the released ``Decision/`` tile maps on real checkpoints.

The model skeleton is built from the checkpoint's ``config.json`` with its parameters
on the meta device (no dense weights materialised), then the shards are streamed: a
target projection's weight goes to the GPU and is packed there by the CUDA packer
(quantized straight from the checkpoint tensor, never installed dense), every other
tensor is placed on the device.  The reference packs on the host and imports
``set_module_tensor_to_device`` / ``init_empty_weights`` from transformers or
accelerate, which this environment's transformers (5.5) does not provide; the two
small helpers below stand in for them.  Same arguments, same checks and errors, same
statistics dictionary as the reference.
"""

from __future__ import annotations

import json
import time
from contextlib import contextmanager
from dataclasses import dataclass, field
from pathlib import Path
from types import SimpleNamespace
from typing import Dict, Iterable, Iterator, List, Optional, Tuple

import numpy as np
import torch
import torch.nn as nn

from .mask_io import load_fp16_keep_ids_for_layer
from .mixed_linear import MixedLinear, fuse_projection_groups
from .pack import pack_weight_from_tile_ids
from .rules import iter_target_linears
from .trace import traced


@dataclass(frozen=True)
class TileConfig:
    """src/quantization/types.py:7-10."""

    tile_m: int = 64
    tile_n: int = 64


@dataclass(frozen=True)
class ApplyConfig:
    """src/quantization/types.py:13-20."""

    model_type: str
    dtype_out: str = "fp16"
    tile: TileConfig = field(default_factory=TileConfig)
    module_filters: List[str] = field(default_factory=list)
    quant_style: str = "gi"
    iaa_channel_stats_path: Optional[str] = None


def make_cfg(apply_cfg: ApplyConfig) -> SimpleNamespace:
    """The pack/MixedLinear config of an ApplyConfig (api.py:48-60)."""
    return SimpleNamespace(
        tile_m=int(apply_cfg.tile.tile_m),
        tile_n=int(apply_cfg.tile.tile_n),
        precision_map_source="mask_keep",
        act_quant="per_tensor_absmax",
        weight_quant="per_tile_absmax",
        quant_style=str(getattr(apply_cfg, "quant_style", "gi")),
        dtype_out=str(apply_cfg.dtype_out),
        pad_to_tile=True,
        module_filters=list(apply_cfg.module_filters),
    )


def load_iaa_channel_stats(keep_dir, apply_cfg: ApplyConfig) -> Dict[str, torch.Tensor]:
    """Per-layer IAA channel mean |x| by stem, from ``iaa_channel_stats_path`` or the
    decision directory's ``iaa_channel_mean_abs.npz`` two levels above ``keep_dir``
    (api.py:63-78)."""
    override = getattr(apply_cfg, "iaa_channel_stats_path", None)
    path = Path(str(override)) if override else Path(keep_dir).parent.parent / "iaa_channel_mean_abs.npz"
    if not path.exists():
        raise FileNotFoundError(
            f"IAA channel stats not found: {path}. "
            "Generate via build_decisions.py --quant_style iaa or pass --iaa_channel_stats_path.")
    with np.load(path, allow_pickle=False) as data:
        return {key: torch.from_numpy(np.asarray(data[key], dtype=np.float32)).contiguous() for key in data.files}


def _tile_grid(shape: Iterable[int], tile_m: int, tile_n: int) -> Tuple[int, int]:
    m, k = int(shape[0]), int(shape[1])
    return (m + tile_m - 1) // tile_m, (k + tile_n - 1) // tile_n


def validate_fp16_ids_coverage_and_shapes(model: nn.Module, keep_dir, apply_cfg: ApplyConfig
                                          ) -> Dict[str, Tuple[torch.Tensor, torch.Tensor, int, int]]:
    """For every target projection: its kept 16-bit tile ids from the archive, the INT8
    ids (the complement, ascending) and the tile grid, after checking the archive's grid
    against the module's shape and the ids' range (api.py:81-118)."""
    cfg = make_cfg(apply_cfg)
    targets = iter_target_linears(model, cfg=cfg, model_type=apply_cfg.model_type)
    if not targets:
        raise RuntimeError(f"No target linears found for model_type={apply_cfg.model_type}.")
    out: Dict[str, Tuple[torch.Tensor, torch.Tensor, int, int]] = {}
    for _, _, full_name, linear in targets:
        fp16_ids, (n_tr, n_tc) = load_fp16_keep_ids_for_layer(keep_dir=keep_dir, layer_name=full_name,
                                                              tile_m=cfg.tile_m, tile_n=cfg.tile_n)
        expected = _tile_grid(linear.weight.shape, cfg.tile_m, cfg.tile_n)
        if (n_tr, n_tc) != expected:
            raise RuntimeError(f"FP16 keep-id shape mismatch for {full_name}: archive={(n_tr, n_tc)} "
                               f"expected={expected}")
        total = n_tr * n_tc
        ids = fp16_ids.to(torch.int64)
        if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= total):
            raise RuntimeError(f"FP16 keep-id out of range for {full_name}: total_tiles={total} "
                               f"min={int(ids.min())} max={int(ids.max())}")
        keep = torch.zeros(total, dtype=torch.bool)
        keep[ids] = True
        int8_ids = torch.nonzero(~keep, as_tuple=False).reshape(-1).to(torch.int32).contiguous()
        out[full_name] = (ids.to(torch.int32).contiguous(), int8_ids, int(n_tr), int(n_tc))
    return out


def resolve_safetensor_shards(local_model_dir) -> Iterator[Path]:
    """The checkpoint's shard files: those named by ``model.safetensors.index.json``
    (sorted, each must exist), else ``model.safetensors`` (api.py:121-145)."""
    local_model_dir = Path(local_model_dir)
    index_path = local_model_dir / "model.safetensors.index.json"
    if index_path.exists():
        with open(index_path, "r", encoding="utf-8") as f:
            weight_map = json.load(f).get("weight_map", {})
        if not isinstance(weight_map, dict) or not weight_map:
            raise RuntimeError(f"Invalid or empty weight_map in index: {index_path}")
        for rel in sorted(set(weight_map.values())):
            shard = local_model_dir / rel
            if not shard.exists():
                raise RuntimeError(f"Missing shard file listed in index: {shard}")
            yield shard
        return
    single = local_model_dir / "model.safetensors"
    if single.exists():
        yield single
        return
    raise RuntimeError(f"No safetensors checkpoint found in {local_model_dir}. "
                       "Expected model.safetensors or model.safetensors.index.json.")


@contextmanager
def parameters_on_meta():
    """Every parameter registered inside the block is moved to the meta device as it is
    registered (buffers stay where they are made), so a model skeleton holds no dense
    weights and its initialisers run on meta tensors."""
    original = nn.Module.register_parameter

    def register(module, name, param):
        original(module, name, param)
        p = module._parameters.get(name)
        if p is not None and p.device.type != "meta":
            module._parameters[name] = nn.Parameter(p.to("meta"), requires_grad=p.requires_grad)

    nn.Module.register_parameter = register
    try:
        yield
    finally:
        nn.Module.register_parameter = original


def set_module_tensor(model: nn.Module, key: str, device, value: torch.Tensor) -> None:
    """Install ``value`` on ``device`` as the parameter or buffer named ``key``
    (``a.b.weight``) of ``model``."""
    mod_name, _, attr = key.rpartition(".")
    module = model.get_submodule(mod_name) if mod_name else model
    value = value.to(device)
    if attr in module._parameters:
        old = module._parameters[attr]
        module._parameters[attr] = nn.Parameter(value, requires_grad=bool(old is not None and old.requires_grad
                                                                          and value.is_floating_point()))
    elif attr in module._buffers:
        module._buffers[attr] = value
    else:
        raise KeyError(f"checkpoint tensor {key} has no parameter or buffer in the model")


def _cast(tensor: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return tensor.to(dtype=dtype) if tensor.is_floating_point() else tensor


@traced("tq.load_mixed_precision_model_from_masks")
def load_mixed_precision_model_from_masks(local_model_dir, keep_dir, apply_cfg: ApplyConfig,
                                          torch_dtype: torch.dtype, device,
                                          attn_implementation: Optional[str] = None):
    """Build the model of ``local_model_dir`` with its target projections packed as
    ``MixedLinear`` from the tile maps of ``keep_dir`` while the shards stream in; returns
    ``(model, stats)`` with the reference's statistics keys (api.py:154-310)."""
    from safetensors import safe_open
    from transformers import AutoConfig, AutoModelForCausalLM

    started = time.perf_counter()
    local_model_dir = Path(local_model_dir)
    cfg = make_cfg(apply_cfg)
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("load-time packing runs on the GPU (there is no CPU path)")
    config_kwargs = {"attn_implementation": attn_implementation} if attn_implementation else {}
    config = AutoConfig.from_pretrained(str(local_model_dir), **config_kwargs)
    with parameters_on_meta():
        model = AutoModelForCausalLM.from_config(config, dtype=torch_dtype, **config_kwargs)

    targets = iter_target_linears(model, cfg=cfg, model_type=apply_cfg.model_type)
    if not targets:
        raise RuntimeError(f"No target linears found for model_type={apply_cfg.model_type}.")
    target_meta = {full: (parent, attr) for parent, attr, full, _ in targets}
    fp16_data = validate_fp16_ids_coverage_and_shapes(model, keep_dir, apply_cfg)
    target_names = set(fp16_data)
    quant_style = str(getattr(apply_cfg, "quant_style", "gi")).lower()
    iaa_stats = load_iaa_channel_stats(keep_dir, apply_cfg) if quant_style == "iaa" else {}

    pending_bias: Dict[str, torch.Tensor] = {}
    loaded_non_target = replaced = 0
    pack_total = non_target_total = 0.0
    for shard in resolve_safetensor_shards(local_model_dir):
        with safe_open(str(shard), framework="pt", device="cpu") as sf:
            for key in sf.keys():
                tensor = sf.get_tensor(key)
                if key.endswith(".weight") and key[:-len(".weight")] in target_names:
                    name = key[:-len(".weight")]
                    t0 = time.perf_counter()
                    parent, attr = target_meta[name]
                    fp16_ids, int8_ids, n_tr, n_tc = fp16_data[name]
                    imp = iaa_stats.get(name.replace(".", "_")) if quant_style == "iaa" else None
                    if imp is not None:
                        imp = imp.to(device=device, dtype=torch.float32)
                    w = _cast(tensor, torch_dtype).to(device)
                    pack = pack_weight_from_tile_ids(w, int8_tile_ids=int8_ids, fp16_tile_ids=fp16_ids, n_tr=n_tr,
                                                     n_tc=n_tc, iaa_col_importance=imp, cfg=cfg)
                    mod = MixedLinear(pack=pack, bias=None, cfg=cfg).to(device)
                    setattr(parent, attr, mod)
                    replaced += 1
                    if name in pending_bias:
                        bias = _cast(pending_bias.pop(name), torch_dtype).to(device)
                        mod.bias = nn.Parameter(bias, requires_grad=False)
                    pack_total += time.perf_counter() - t0
                    continue
                if key.endswith(".bias") and key[:-len(".bias")] in target_names:
                    name = key[:-len(".bias")]
                    mod = model.get_submodule(name)
                    if isinstance(mod, MixedLinear):
                        mod.bias = nn.Parameter(_cast(tensor, torch_dtype).to(device), requires_grad=False)
                    else:
                        pending_bias[name] = tensor
                    continue
                t0 = time.perf_counter()
                set_module_tensor(model, key, device, _cast(tensor, torch_dtype))
                non_target_total += time.perf_counter() - t0
                loaded_non_target += 1

    if pending_bias:
        raise RuntimeError("Found target bias tensors without corresponding target weight loads, "
                           f"e.g. {list(pending_bias)[:3]}")
    modules = dict(model.named_modules())
    for name in target_names:
        if not isinstance(modules.get(name), MixedLinear):
            raise RuntimeError(f"Target module is not MixedLinear after load-time apply: {name}")
    # buffers made on the host by the skeleton (e.g. RoPE inv_freq) go to the device, so
    # a forward issues no implicit host-to-device copy (which would also break capture)
    for module in model.modules():
        for bname, buf in list(module._buffers.items()):
            if buf is not None and buf.device != device and buf.device.type != "meta":
                module._buffers[bname] = buf.to(device)
        value = getattr(module, "original_inv_freq", None)
        if isinstance(value, torch.Tensor) and value.device != device:
            module.original_inv_freq = value.to(device)
    fused = fuse_projection_groups(model)
    if hasattr(model, "tie_weights"):
        model.tie_weights()
    still_meta = [n for n, p in model.named_parameters() if p.device.type == "meta"]
    if still_meta:
        raise RuntimeError(f"Parameters missing from the checkpoint, e.g. {still_meta[:3]}")
    model.eval()
    return model, {
        "num_targets": len(target_names),
        "num_replaced": len(target_names),
        "num_replaced_during_load": replaced,
        "num_loaded_non_target_tensors": loaded_non_target,
        "load_total": float(time.perf_counter() - started),
        "quant_pack_total": float(pack_total),
        "non_target_load_total": float(non_target_total),
        "attn_implementation": attn_implementation,
        "fused_projection_groups": int(fused),
    }
