"""Turn a decoder's projection ``nn.Linear`` modules into ``MixedLinear`` in place.

The reference applies tile maps while loading a safetensors checkpoint
(src/quantization/api.py:80-118 builds the INT8 ids as the complement of the kept BF16
ids, :154-310 loads and swaps the modules).  Here the same swap works on a model that
is already in memory -- the benchmark configurations use random-init weights -- with
the tile maps given per module name (``{name: kept 16-bit tile ids}``), read from the
reference's archives (``mask_io.load_fp16_keep_ids_for_layer``), or drawn uniformly at
random (``random_keep_ids``, the benchmark configurations' masks).  Packing runs on the
weights' device with the CUDA packer.
"""

from __future__ import annotations

import math
from types import SimpleNamespace
from typing import Any, Callable, Dict, Mapping, Optional, Union

import torch
import torch.nn as nn

from .mixed_linear import MixedLinear, fuse_projection_groups
from .pack import pack_weight_from_tile_ids
from .rules import iter_target_linears

KeepIds = Union[Mapping[str, torch.Tensor], Callable[[str, int, int], torch.Tensor]]


def default_cfg(**overrides: Any) -> SimpleNamespace:
    """The reference's default apply config for the 64x64 path (GI-style INT8 scales,
    BF16 output)."""
    cfg = dict(tile_m=64, tile_n=64, pad_to_tile=True, quant_style="gi", dtype_out="bf16")
    cfg.update(overrides)
    return SimpleNamespace(**cfg)


def tile_grid(weight: torch.Tensor, cfg: Any) -> tuple:
    m, k = weight.shape
    return math.ceil(m / cfg.tile_m), math.ceil(k / cfg.tile_n)


def random_keep_ids(n_tr: int, n_tc: int, fraction: float, generator: torch.Generator) -> torch.Tensor:
    """ceil(fraction * tiles) distinct tile ids, uniformly at random, ascending."""
    total = n_tr * n_tc
    n_keep = min(total, int(math.ceil(fraction * total)))
    return torch.randperm(total, generator=generator)[:n_keep].sort().values.to(torch.int32)


def complement_ids(keep: torch.Tensor, total: int) -> torch.Tensor:
    """INT8 tile ids: every tile not kept in 16 bits, ascending (api.py:104-112)."""
    mask = torch.ones(total, dtype=torch.bool)
    if keep.numel():
        mask[keep.to(torch.int64)] = False
    return torch.nonzero(mask, as_tuple=False).reshape(-1).to(torch.int32)


@torch.no_grad()
def apply_tile_maps(model: nn.Module, keep_ids: KeepIds, cfg: Any = None, *, model_type: str = "llama",
                    iaa_channel_stats: Optional[Mapping[str, torch.Tensor]] = None,
                    fuse_groups: bool = True) -> Dict[str, MixedLinear]:
    """Replace every target projection of ``model`` by a ``MixedLinear``.

    ``keep_ids`` maps a module's full name to its kept 16-bit tile ids, or is a callable
    ``(name, n_tr, n_tc) -> ids``.  With ``cfg.quant_style == 'iaa'``,
    ``iaa_channel_stats[name]`` (f32[K], the mean |x| per input channel) drives the
    INT8 scale search.  Q/K/V and gate/up siblings are then stacked so each group runs
    one quantization and one GEMM (``fuse_projection_groups``).  Returns the new
    modules by name.
    """
    cfg = cfg or default_cfg()
    targets = iter_target_linears(model, cfg, model_type=model_type)
    if not targets:
        raise RuntimeError(f"No target linears found for model_type={model_type}.")
    swapped: Dict[str, MixedLinear] = {}
    for parent, attr, name, linear in targets:
        w = linear.weight.detach()
        n_tr, n_tc = tile_grid(w, cfg)
        keep = keep_ids(name, n_tr, n_tc) if callable(keep_ids) else keep_ids[name]
        keep = torch.as_tensor(keep, dtype=torch.int32).reshape(-1).sort().values
        if keep.numel() and (int(keep.min()) < 0 or int(keep.max()) >= n_tr * n_tc):
            raise RuntimeError(f"16-bit tile id out of range for {name}")
        imp = None
        if str(getattr(cfg, "quant_style", "gi")).lower() == "iaa":
            if iaa_channel_stats is None or name not in iaa_channel_stats:
                raise RuntimeError(f"IAA channel stats missing for {name}")
            imp = iaa_channel_stats[name].to(device=w.device, dtype=torch.float32)
        pack = pack_weight_from_tile_ids(w, n_tr=n_tr, n_tc=n_tc, int8_tile_ids=complement_ids(keep, n_tr * n_tc),
                                         fp16_tile_ids=keep, iaa_col_importance=imp, cfg=cfg)
        bias = None if linear.bias is None else linear.bias.detach()
        mixed = MixedLinear(pack, bias, cfg).to(w.device)
        setattr(parent, attr, mixed)
        swapped[name] = mixed
    if fuse_groups:
        fuse_projection_groups(model)
    return swapped


def apply_random_tile_maps(model: nn.Module, fraction: float, seed: int, cfg: Any = None, *,
                           model_type: str = "llama") -> Dict[str, MixedLinear]:
    """``apply_tile_maps`` with ``fraction`` of every projection's tiles kept in 16 bits,
    chosen uniformly at random (seeded per module, in module order)."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(int(seed))
    return apply_tile_maps(model, lambda name, n_tr, n_tc: random_keep_ids(n_tr, n_tc, fraction, gen), cfg,
                           model_type=model_type)
