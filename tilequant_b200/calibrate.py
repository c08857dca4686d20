"""Tile-importance calibration (GI and IAA) on the GPU, and the top-k tile maps.

Drop-in for the reference's collectors (src/kernels/calibrate.py of
HanzhiZhang-Ulrica/TileQuant) with the same names, arguments, config keys, checkpoint
files and results:

* ``collect_gi_tile_scores``                      -- calibrate.py:42-184
* ``collect_iaa_tile_scores``                     -- calibrate.py:187-199
* ``collect_iaa_tile_scores_with_channel_stats``  -- calibrate.py:202-369
* ``topk_mask``                                    -- decisions.py:174-183 (``_topk_mask``)

The per-tile reductions run on this package's CUDA kernels and stay on the device for
the whole run: GI adds sum over each 64x64 tile of |W * dL/dW| into an FP32 device
accumulator after every backward (``tq_calib_gi_accumulate``; the reference moves
every batch's tile sums to the host), IAA adds sum over rows of |x| per input channel
into an FP64 device accumulator from a forward pre-hook
(``tq_calib_iaa_channel_accumulate``) and forms the tile scores sum |W| * mean|x| at the
end (``tq_calib_iaa_tile_scores``).  Scores are returned on the CPU as FP32, like the
reference's, and the resumable checkpoints use the reference's file names and fields.
Activations, weights and gradients must be BF16 or FP16 CUDA tensors.
"""

from __future__ import annotations

import math
from pathlib import Path
from typing import Any, Callable, Dict, Iterable, Tuple

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _native as N


def _cfg_get(cfg: Any, key: str, default=None):
    if isinstance(cfg, dict):
        return cfg.get(key, default)
    return getattr(cfg, key, default)


def _grid(module: nn.Linear, tile_m: int, tile_n: int) -> Tuple[int, int]:
    m, k = module.weight.shape
    return (int(m) + tile_m - 1) // tile_m, (int(k) + tile_n - 1) // tile_n


def _check_tiles(tile_m: int, tile_n: int) -> None:
    if (tile_m, tile_n) != (64, 64):
        raise ValueError(f"tilequant_b200 calibrates 64x64 tiles, got {tile_m}x{tile_n}")


# ------------------------------------------------------------------ kernel wrappers

def gi_accumulate(tile_scores: torch.Tensor, w: torch.Tensor, g: torch.Tensor) -> None:
    """tile_scores[r, c] += sum over tile (r, c) of |f32(W) * f32(G)| (in place, device)."""
    N.require_cuda(tile_scores, w, g)
    if w.shape != g.shape or w.dtype != g.dtype or w.dim() != 2:
        raise ValueError("weight and gradient must be 2-D tensors of one shape and dtype")
    m, k = w.shape
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    if tile_scores.dtype != torch.float32 or tuple(tile_scores.shape) != (n_tr, n_tc) or not tile_scores.is_contiguous():
        raise ValueError("tile_scores must be a contiguous float32 (n_tr, n_tc) tensor")
    if w.stride(1) != 1 or g.stride(1) != 1:
        raise ValueError("weight and gradient rows must be contiguous")
    rc = N.load().tq_calib_gi_accumulate(w.data_ptr(), g.data_ptr(), N.dtype_code(w.dtype), m, k, w.stride(0),
                                         g.stride(0), n_tr, n_tc, tile_scores.data_ptr(), N.stream_of(w))
    N.check(rc, "gi_accumulate")


def iaa_channel_accumulate(act_sum: torch.Tensor, x: torch.Tensor) -> int:
    """act_sum[j] += sum over rows of |f32(x[:, j])| in FP64 (device); returns the rows."""
    N.require_cuda(act_sum, x)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    rows, k = x2.shape
    if act_sum.dtype != torch.float64 or act_sum.numel() != k or not act_sum.is_contiguous():
        raise ValueError("act_sum must be a contiguous float64 tensor of the input features")
    if rows:
        rc = N.load().tq_calib_iaa_channel_accumulate(x2.data_ptr(), N.dtype_code(x2.dtype), rows, k, x2.stride(0),
                                                      act_sum.data_ptr(), N.stream_of(x2))
        N.check(rc, "iaa_channel_accumulate")
    return int(rows)


def iaa_tile_scores(w: torch.Tensor, act_sum: torch.Tensor, count: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(mean |x| per channel as f32(act_sum / count), tile scores sum |W| * mean) on the device."""
    N.require_cuda(w, act_sum)
    m, k = w.shape
    if w.stride(1) != 1:
        raise ValueError("weight rows must be contiguous")
    if count <= 0:
        raise ValueError("count must be positive")
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    mean = torch.empty((k,), device=w.device, dtype=torch.float32)
    scores = torch.empty((n_tr, n_tc), device=w.device, dtype=torch.float32)
    rc = N.load().tq_calib_iaa_tile_scores(w.data_ptr(), N.dtype_code(w.dtype), m, k, w.stride(0), act_sum.data_ptr(),
                                           int(count), mean.data_ptr(), scores.data_ptr(), N.stream_of(w))
    N.check(rc, "iaa_tile_scores")
    return mean, scores


# ------------------------------------------------------------------ collectors

def _next_token_ce_loss(model_outputs, input_ids: torch.Tensor) -> torch.Tensor:
    logits = model_outputs.logits if hasattr(model_outputs, "logits") else model_outputs
    return F.cross_entropy(logits[:, :-1, :].reshape(-1, logits.size(-1)), input_ids[:, 1:].reshape(-1),
                           reduction="mean")


def _model_input_device(model: nn.Module) -> torch.device:
    device_map = getattr(model, "hf_device_map", None)
    if isinstance(device_map, dict) and device_map:
        first = next(iter(device_map.values()))
        if isinstance(first, str) and first not in {"cpu", "disk"}:
            return torch.device(first)
    return next(model.parameters()).device


def _calib_options(cfg: Any, progress_file: str):
    tile_m, tile_n = int(_cfg_get(cfg, "tile_m", 64)), int(_cfg_get(cfg, "tile_n", 64))
    _check_tiles(tile_m, tile_n)
    calib = _cfg_get(cfg, "calib", {}) or {}
    num_samples = _cfg_get(calib, "num_samples", None)
    max_tokens = _cfg_get(calib, "max_tokens", None)
    every = int(_cfg_get(calib, "checkpoint_every_batches", 0))
    resume = bool(_cfg_get(calib, "resume_from_checkpoint", False))
    ckpt = None
    if _cfg_get(calib, "checkpoint_dir", None):
        d = Path(str(_cfg_get(calib, "checkpoint_dir"))).resolve()
        d.mkdir(parents=True, exist_ok=True)
        ckpt = d / progress_file
    return tile_m, tile_n, num_samples, max_tokens, every, resume, ckpt


def _targets(model: nn.Module, target_filter_fn: Callable[[str], bool], what: str) -> Dict[str, nn.Linear]:
    found = {n: m for n, m in model.named_modules() if isinstance(m, nn.Linear) and target_filter_fn(n)}
    if not found:
        raise RuntimeError(f"No target linear layers matched for {what} calibration")
    return found


def _atomic_torch_save(payload, path: Path) -> None:
    tmp = path.with_suffix(".tmp")
    torch.save(payload, tmp)
    tmp.replace(path)


def collect_gi_tile_scores(model: nn.Module, dataloader: Iterable, target_filter_fn: Callable[[str], bool],
                           cfg: Any) -> Dict[str, torch.Tensor]:
    """GI tile importance: sum over calibration batches of sum over each tile of
    |W * dL/dW| for the next-token cross-entropy loss (calibrate.py:42-184)."""
    tile_m, tile_n, num_samples, max_tokens, every, resume, ckpt = _calib_options(cfg, "gi_tile_scores_progress.pt")
    targets = _targets(model, target_filter_fn, "GI")
    scores = {n: torch.zeros(_grid(m, tile_m, tile_n), dtype=torch.float32, device=m.weight.device)
              for n, m in targets.items()}
    processed, tokens = 0, 0
    if ckpt is not None and resume and ckpt.exists():
        state = torch.load(ckpt, map_location="cpu", weights_only=False)
        processed, tokens = int(state.get("processed_batches", 0)), int(state.get("tokens_seen", 0))
        for n, saved in state.get("tile_scores", {}).items():
            if n in scores and np.asarray(saved).size == scores[n].numel():
                scores[n].copy_(torch.as_tensor(np.asarray(saved, dtype=np.float32)).reshape(scores[n].shape))

    def save() -> None:
        if ckpt is not None:
            _atomic_torch_save({"processed_batches": processed, "tokens_seen": tokens,
                                "tile_scores": {n: s.cpu().numpy().astype(np.float32) for n, s in scores.items()}},
                               ckpt)

    dev = _model_input_device(model)
    was_training = model.training
    model.eval()
    model.zero_grad(set_to_none=True)
    try:
        for i, batch in enumerate(dataloader):
            if i < processed:
                continue
            if not isinstance(batch, dict):
                raise TypeError("Calibration dataloader must yield dict batches with input_ids")
            model.zero_grad(set_to_none=True)
            inputs = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in batch.items()}
            ids = inputs.get("input_ids")
            if ids is None:
                raise ValueError("Calibration batch dict must include input_ids")
            _next_token_ce_loss(model(**inputs), ids).backward()
            with torch.no_grad():
                for n, mod in targets.items():
                    if mod.weight.grad is None:
                        raise RuntimeError(f"Missing gradient for target linear: {n}")
                    gi_accumulate(scores[n], mod.weight.detach(), mod.weight.grad.detach())
            processed += 1
            tokens += int(ids.numel())
            if ckpt is not None and every > 0 and processed % every == 0:
                save()
            if num_samples is not None and processed >= num_samples:
                break
            if max_tokens is not None and tokens >= max_tokens:
                break
        save()
    finally:
        model.zero_grad(set_to_none=True)
        if was_training:
            model.train()
    return {n: s.cpu().contiguous() for n, s in scores.items()}


def collect_iaa_tile_scores_with_channel_stats(model: nn.Module, dataloader: Iterable,
                                               target_filter_fn: Callable[[str], bool], cfg: Any
                                               ) -> Tuple[Dict[str, torch.Tensor], Dict[str, torch.Tensor]]:
    """IAA tile importance: mean |x| per input channel of every target's input over the
    calibration batches, then per tile sum |W| * mean|x| (calibrate.py:202-369).
    Returns (tile scores, channel means), both FP32 on the CPU."""
    tile_m, tile_n, num_samples, max_tokens, every, resume, ckpt = _calib_options(cfg,
                                                                                  "iaa_activation_progress.pt")
    targets = _targets(model, target_filter_fn, "IAA")
    act_sum = {n: torch.zeros((m.in_features,), dtype=torch.float64, device=m.weight.device)
               for n, m in targets.items()}
    act_count = {n: 0 for n in targets}
    hooks = []
    for n, mod in targets.items():
        def pre_hook(_mod, inputs, name=n):
            x = inputs[0]
            if torch.is_tensor(x) and x.numel():
                act_count[name] += iaa_channel_accumulate(act_sum[name], x)

        hooks.append(mod.register_forward_pre_hook(pre_hook))
    processed, tokens = 0, 0
    if ckpt is not None and resume and ckpt.exists():
        state = torch.load(ckpt, map_location="cpu", weights_only=False)
        for n, c in state.get("act_count", {}).items():
            if n in act_count:
                act_count[n] = int(c)
        for n, s in state.get("act_sum", {}).items():
            if n in act_sum and np.asarray(s).size == act_sum[n].numel():
                act_sum[n].copy_(torch.as_tensor(np.asarray(s, dtype=np.float64)).reshape(act_sum[n].shape))
        processed, tokens = int(state.get("processed_batches", 0)), int(state.get("tokens_seen", 0))

    def save() -> None:
        if ckpt is not None:
            _atomic_torch_save({"processed_batches": processed, "tokens_seen": tokens,
                                "act_count": dict(act_count),
                                "act_sum": {n: s.cpu().numpy().astype(np.float64) for n, s in act_sum.items()}},
                               ckpt)

    dev = _model_input_device(model)
    was_training = model.training
    model.eval()
    try:
        with torch.no_grad():
            for i, batch in enumerate(dataloader):
                if i < processed:
                    continue
                if not isinstance(batch, dict):
                    raise TypeError("Calibration dataloader must yield dict batches with input_ids")
                inputs = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in batch.items()}
                ids = inputs.get("input_ids")
                if ids is None:
                    raise ValueError("Calibration batch dict must include input_ids")
                model(**inputs)
                processed += 1
                tokens += int(ids.numel())
                if ckpt is not None and every > 0 and processed % every == 0:
                    save()
                if num_samples is not None and processed >= num_samples:
                    break
                if max_tokens is not None and tokens >= max_tokens:
                    break
            save()
    finally:
        for h in hooks:
            h.remove()
        if was_training:
            model.train()
    tile_scores: Dict[str, torch.Tensor] = {}
    channel_stats: Dict[str, torch.Tensor] = {}
    for n, mod in targets.items():
        if act_count[n] <= 0:
            raise RuntimeError(f"No activation samples captured for target linear: {n}")
        mean, sc = iaa_tile_scores(mod.weight.detach(), act_sum[n], act_count[n])
        channel_stats[n] = mean.cpu()
        tile_scores[n] = sc.cpu()
    return tile_scores, channel_stats


def collect_iaa_tile_scores(model: nn.Module, dataloader: Iterable, target_filter_fn: Callable[[str], bool],
                            cfg: Any) -> Dict[str, torch.Tensor]:
    """IAA tile scores only (calibrate.py:187-199)."""
    return collect_iaa_tile_scores_with_channel_stats(model, dataloader, target_filter_fn, cfg)[0]


# ------------------------------------------------------------------ decisions

def topk_mask(importance: np.ndarray, keep_frac: float) -> np.ndarray:
    """uint8 mask of the ceil(keep_frac * tiles) most important tiles (at least one),
    chosen with numpy's argpartition exactly as the reference (decisions.py:174-183)."""
    values = np.asarray(importance).reshape(-1)
    k = max(1, int(math.ceil(float(keep_frac) * int(values.size))))
    idx = np.arange(values.size) if k >= values.size else np.argpartition(values, -k)[-k:]
    mask = np.zeros_like(values, dtype=np.uint8)
    mask[idx] = 1
    return mask.reshape(np.asarray(importance).shape)


def keep_ids_from_scores(scores: Dict[str, torch.Tensor], keep_frac: float) -> Dict[str, torch.Tensor]:
    """Kept 16-bit tile ids (ascending int32) of every target from its tile scores."""
    return {n: torch.from_numpy(np.flatnonzero(topk_mask(s.numpy(), keep_frac)).astype(np.int32))
            for n, s in scores.items()}
