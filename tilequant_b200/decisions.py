"""Decision directories: calibration scores -> tile-map archives at several keep
fractions, in the reference's on-disk layout (src/quantization/decisions.py:23-388), so
``loader.load_mixed_precision_model_from_masks`` (and the reference's own loader) can
read them.

    <decision_dir>/
      {gi,iaa}_tile_scores_tile64x64.npz     f32 tile scores by stem
      iaa_channel_mean_abs.npz               (IAA) f32 channel mean |x| by stem
      tile_masks/keepNN/fp16_keep_ids_tile64x64.npz + meta.json   (NN = 01, 02, 05, 10, 20)
      decision_meta.json, decision_ready.flag

The reference tokenizes a summarization dataset; the calibration data here is whatever
token batches the caller passes (the benchmark configurations use seeded uniform-random
ids), and the collectors are the GPU ones of ``calibrate.py`` with their resumable
progress files in the decision directory.
"""

from __future__ import annotations

import json
from pathlib import Path
from types import SimpleNamespace
from typing import Dict, Iterable, Optional, Sequence

import numpy as np
import torch
import torch.nn as nn

from .calibrate import collect_gi_tile_scores, collect_iaa_tile_scores_with_channel_stats, topk_mask
from .mask_io import save_mask_keep_archive
from .rules import iter_target_linears

DEFAULT_KEEP_FRACS = (0.01, 0.02, 0.05, 0.10, 0.20)
SCORE_RULES = {"iaa": "iaa_like_absW_times_meanAbsX_tile_sum",
               "gi": "gi_absW_times_grad_tile_sum_accumulated_per_batch"}


def infer_model_type(local_model_dir) -> str:
    """"qwen" or "llama" from a checkpoint's config.json (decisions.py:26-33)."""
    from transformers import AutoConfig

    model_type = str(getattr(AutoConfig.from_pretrained(str(local_model_dir)), "model_type", "")).lower()
    if "qwen" in model_type:
        return "qwen"
    if "llama" in model_type:
        return "llama"
    raise RuntimeError(f"Unsupported model_type for decision build: {model_type!r}")


def score_npz_path(decision_dir, quant_style: str, tile_m: int = 64, tile_n: int = 64) -> Path:
    """decisions.py:36-37."""
    return Path(decision_dir) / f"{quant_style}_tile_scores_tile{tile_m}x{tile_n}.npz"


def keep_tag(keep_frac: float) -> str:
    """Directory name of a keep fraction: keep01 for 0.01 (decisions.py:198)."""
    return f"keep{int(float(keep_frac) * 100):02d}"


def _replace_atomically(path: Path, write) -> None:
    tmp = path.parent / f"{path.name}.tmp"
    write(tmp)
    tmp.replace(path)


def _save_npz(path: Path, arrays: Dict[str, np.ndarray]) -> None:
    def write(tmp):
        with open(tmp, "wb") as f:
            np.savez_compressed(f, **arrays)

    _replace_atomically(path, write)


def _save_json(path: Path, payload: Dict[str, object]) -> None:
    _replace_atomically(path, lambda tmp: tmp.write_text(json.dumps(payload, indent=2), encoding="utf-8"))


def load_npz_map(path) -> Dict[str, np.ndarray]:
    with np.load(path, allow_pickle=False) as data:
        return {str(k): np.asarray(data[k], dtype=np.float32) for k in data.files}


def save_masks(decision_dir, scores_by_stem: Dict[str, np.ndarray], keep_fracs: Sequence[float],
               model_name_or_path: str, dataset_id: str, dataset_split: str, quant_style: str,
               tile_m: int = 64, tile_n: int = 64) -> Dict[float, Path]:
    """One archive (top ceil(f * tiles) scores per layer kept 16-bit) and meta.json per
    keep fraction f (decisions.py:186-224); returns the keep directories."""
    root = Path(decision_dir) / "tile_masks"
    out = {}
    for frac in keep_fracs:
        d = root / keep_tag(frac)
        d.mkdir(parents=True, exist_ok=True)
        save_mask_keep_archive(d, {stem: topk_mask(s, float(frac)) for stem, s in scores_by_stem.items()},
                               tile_m=tile_m, tile_n=tile_n)
        _save_json(d / "meta.json", {
            "model_name_or_path": model_name_or_path, "dataset_id": dataset_id, "dataset_split": dataset_split,
            "quant_style": quant_style, "tile_m": tile_m, "tile_n": tile_n, "keep_frac": float(frac),
            "mask_rule": "topk_by_importance"})
        out[float(frac)] = d
    return out


def _prune_progress_files(decision_dir: Path) -> None:
    """The collectors' resumable progress files go once the scores are final
    (decisions.py:61-78)."""
    for pattern in ("*_iaa_sum.npy", "*_gi_sum.npy"):
        for p in decision_dir.glob(pattern):
            if p.is_file():
                p.unlink()
    for rel in ("iaa_activation_progress.pt", "gi_tile_scores_progress.pt", "iaa_layer_stats.json", "iaa_meta.json",
                "done_iaa.flag", "tile_masks/eval_results.json"):
        p = decision_dir / rel
        if p.exists():
            p.unlink()


def build_decisions_from_batches(model: nn.Module, batches: Iterable, decision_dir, quant_style: str = "gi",
                                 model_type: str = "llama", model_name_or_path: str = "",
                                 keep_fracs: Sequence[float] = DEFAULT_KEEP_FRACS,
                                 dataset_id: str = "synthetic:uniform-random-token-ids", dataset_split: str = "-",
                                 tile_m: int = 64, tile_n: int = 64, num_batches: int = -1,
                                 checkpoint_every_batches: int = 100, dtype: str = "bf16",
                                 batch_size: Optional[int] = None) -> Path:
    """Score every target projection of ``model`` over ``batches`` (dicts with
    ``input_ids``) on the GPU, then write the decision directory (decisions.py:227-388).
    Existing score files are reused, and an interrupted collection resumes from its
    progress file, as in the reference."""
    quant_style = str(quant_style).lower()
    if quant_style not in SCORE_RULES:
        raise ValueError(f"Unsupported quant_style={quant_style}. Expected one of: gi, iaa")
    decision_dir = Path(decision_dir)
    decision_dir.mkdir(parents=True, exist_ok=True)
    keep_fracs = [float(f) for f in keep_fracs]
    scores_path = score_npz_path(decision_dir, quant_style, tile_m, tile_n)
    stats_path = decision_dir / "iaa_channel_mean_abs.npz"
    if scores_path.exists() and (quant_style != "iaa" or stats_path.exists()):
        scores_by_stem = load_npz_map(scores_path)
    else:
        cfg = SimpleNamespace(tile_m=tile_m, tile_n=tile_n, module_filters=[], calib=SimpleNamespace(
            num_samples=None if num_batches <= 0 else int(num_batches), max_tokens=None,
            checkpoint_dir=str(decision_dir), checkpoint_every_batches=int(checkpoint_every_batches),
            resume_from_checkpoint=True))
        names = {n for _, _, n, _ in iter_target_linears(model, cfg, model_type=model_type)}
        if not names:
            raise RuntimeError(f"No target linears found for model_type={model_type}")
        if quant_style == "iaa":
            scores, stats = collect_iaa_tile_scores_with_channel_stats(model, batches, lambda n: n in names, cfg)
            _save_npz(stats_path, {n.replace(".", "_"): v.cpu().numpy().astype(np.float32) for n, v in stats.items()})
        else:
            scores = collect_gi_tile_scores(model, batches, lambda n: n in names, cfg)
        scores_by_stem = {n.replace(".", "_"): v.cpu().numpy().astype(np.float32) for n, v in scores.items()}
        _save_npz(scores_path, scores_by_stem)
    save_masks(decision_dir, scores_by_stem, keep_fracs, model_name_or_path, dataset_id, dataset_split, quant_style,
               tile_m, tile_n)
    _save_json(decision_dir / "decision_meta.json", {
        "model_name_or_path": model_name_or_path, "model_type": model_type, "dataset_id": dataset_id,
        "dataset_split": dataset_split, "quant_style": quant_style, "num_batches": int(num_batches),
        "batch_size": batch_size, "tile_m": tile_m, "tile_n": tile_n, "dtype": dtype,
        "checkpoint_every_batches": int(checkpoint_every_batches), "keep_fracs": keep_fracs,
        "num_targets": len(scores_by_stem), "score_rule": SCORE_RULES[quant_style], "score_file": scores_path.name,
        "channel_stats_file": stats_path.name if quant_style == "iaa" else None})
    _replace_atomically(decision_dir / "decision_ready.flag", lambda tmp: tmp.write_text("done\n", encoding="utf-8"))
    _prune_progress_files(decision_dir)
    return decision_dir


# ------------------------------------------------------------------ resolution

def resolve_decision_dir(local_model_dir, quant_style: str, decision_root="Decision") -> Path:
    """``<decision_root>/<model dir name>/<style>``, which must exist (resolve.py:22-26)."""
    d = Path(decision_root).resolve() / Path(local_model_dir).name / str(quant_style).lower()
    if not d.exists():
        raise RuntimeError(f"Decision directory not found: {d}")
    return d


def resolve_keep_dir(decision_dir, keep_tag: Optional[str] = None) -> Path:
    """``tile_masks/<keep_tag>``, or the newest keepNN directory when no tag is given
    (resolve.py:29-41)."""
    root = Path(decision_dir) / "tile_masks"
    if not root.exists():
        raise RuntimeError(f"Mask root not found: {root}")
    keep_dirs = [p for p in root.iterdir() if p.is_dir() and p.name.startswith("keep")]
    if not keep_dirs:
        raise RuntimeError(f"No keepXX folders found under: {root}")
    if keep_tag is not None:
        picked = root / keep_tag
        if not picked.exists():
            raise RuntimeError(f"Requested keep dir not found: {picked}")
        return picked
    return sorted(keep_dirs, key=lambda p: (p.stat().st_mtime, p.name), reverse=True)[0]


def resolve_decision_and_keep_dir(local_model_dir, quant_style: str, keep_tag: Optional[str] = None,
                                  decision_root="Decision"):
    """resolve.py:44-51."""
    d = resolve_decision_dir(local_model_dir, quant_style, decision_root)
    return d, resolve_keep_dir(d, keep_tag)


def load_model_and_tokenizer(model_dir, *, quant_style: str = "gi", keep_tag: Optional[str] = "keep01",
                             dtype: str = "bf16", device="cuda", iaa_channel_stats_path: Optional[str] = None,
                             decision_root="Decision", tile_m: int = 64, tile_n: int = 64,
                             attn_implementation: Optional[str] = "sdpa", batches: Optional[Iterable] = None):
    """The model of a local checkpoint with its tile maps applied at load, its
    tokenizer, and a description (the reference's application.load_model_and_tokenizer,
    application.py:58-139).  Missing decision artifacts are built first from the
    calibration ``batches`` (``ensure_decision_artifacts``)."""
    from transformers import AutoTokenizer

    from .loader import ApplyConfig, TileConfig, load_mixed_precision_model_from_masks

    model_dir, decision_dir, keep_dir = ensure_decision_artifacts(model_dir, quant_style, keep_tag, decision_root,
                                                                  batches=batches, device=device, dtype=dtype)
    model_type = infer_model_type(model_dir)
    quant_style = str(quant_style).lower()
    if quant_style == "iaa" and not iaa_channel_stats_path:
        auto = decision_dir / "iaa_channel_mean_abs.npz"
        if not auto.exists():
            raise FileNotFoundError(f"IAA channel stats not found: {auto}")
        iaa_channel_stats_path = str(auto)
    tokenizer = AutoTokenizer.from_pretrained(str(model_dir), use_fast=True)
    if tokenizer.pad_token is None:
        tokenizer.pad_token = tokenizer.eos_token
    device = torch.device(device)
    model, stats = load_mixed_precision_model_from_masks(
        model_dir, keep_dir,
        ApplyConfig(model_type=model_type, dtype_out=dtype, tile=TileConfig(tile_m, tile_n), module_filters=[],
                    quant_style=quant_style, iaa_channel_stats_path=iaa_channel_stats_path),
        torch.float16 if dtype == "fp16" else torch.bfloat16, device, attn_implementation=attn_implementation)
    info = {"device": device, "local_model_dir": model_dir, "decision_dir": decision_dir, "keep_dir": keep_dir,
            "model_type": model_type, "quant_style": quant_style, "tile_m": tile_m, "tile_n": tile_n,
            "iaa_channel_stats_path": iaa_channel_stats_path, "attn_implementation": attn_implementation,
            "stats": stats}
    return model, tokenizer, info


def ensure_decision_artifacts(model_dir, quant_style: str = "gi", keep_tag: Optional[str] = "keep01",
                              decision_root="Decision", batches: Optional[Iterable] = None, device="cuda",
                              dtype: str = "bf16", keep_fracs: Sequence[float] = DEFAULT_KEEP_FRACS,
                              checkpoint_every_batches: int = 100):
    """``(model_dir, decision_dir, keep_dir)``, building the decision directory first
    when it, its IAA channel statistics or the requested keep directory is missing
    (decisions.py:391-451).  Building needs calibration ``batches`` (dicts with
    ``input_ids``; the reference draws them from its dataset instead) and runs the
    dense checkpoint on ``device``."""
    model_dir = Path(model_dir)
    quant_style = str(quant_style).lower()
    build = False
    try:
        decision_dir = resolve_decision_dir(model_dir, quant_style, decision_root)
    except RuntimeError:
        build = True
        decision_dir = Path(decision_root).resolve() / model_dir.name / quant_style
    if quant_style == "iaa" and not (decision_dir / "iaa_channel_mean_abs.npz").exists():
        build = True
    if not build:
        try:
            resolve_keep_dir(decision_dir, keep_tag)
        except RuntimeError:
            build = True
    if build:
        if batches is None:
            raise RuntimeError(f"Decision artifacts missing under {decision_dir} and no calibration batches given")
        from transformers import AutoModelForCausalLM

        model = AutoModelForCausalLM.from_pretrained(str(model_dir),
                                                     dtype=torch.float16 if dtype == "fp16" else torch.bfloat16)
        model = model.to(torch.device(device)).eval()
        model.config.use_cache = False
        build_decisions_from_batches(model, batches, decision_dir, quant_style=quant_style,
                                     model_type=infer_model_type(model_dir), model_name_or_path=str(model_dir),
                                     keep_fracs=keep_fracs, checkpoint_every_batches=checkpoint_every_batches,
                                     dtype=dtype)
        del model
    return model_dir, decision_dir, resolve_keep_dir(decision_dir, keep_tag)
