"""Tile-map archives: which 64x64 tiles of each layer stay 16-bit.

Reads and writes the reference's on-disk format unchanged (src/kernels/mask_io.py of
HanzhiZhang-Ulrica/TileQuant, :36-127), so released ``Decision/`` maps load as is:
an ``np.savez_compressed`` archive ``fp16_keep_ids_tile{tm}x{tn}.npz`` holding
``stems`` (str array, sorted) and, for stem i, ``shape_i`` (int32 [n_tr, n_tc]) and
``ids_i`` (flat row-major ids of the kept tiles; uint16 when the grid has at most
65535 tiles, else uint32).  A stem is the module name with '.' replaced by '_'.
"""

from __future__ import annotations

from pathlib import Path
from typing import Dict, Tuple

import numpy as np
import torch

ARCHIVE_STEM = "fp16_keep_ids"
_CACHE: Dict[str, Dict[str, Tuple[Tuple[int, int], np.ndarray]]] = {}


def layer_name_to_stem(layer_name: str) -> str:
    return layer_name.replace(".", "_")


def archive_path(keep_dir, tile_m: int = 64, tile_n: int = 64) -> Path:
    return Path(keep_dir) / f"{ARCHIVE_STEM}_tile{tile_m}x{tile_n}.npz"


def _binary(mask_keep) -> np.ndarray:
    arr = np.asarray(mask_keep)
    if arr.ndim != 2:
        raise ValueError(f"mask_keep must be 2D, got shape={tuple(arr.shape)}")
    arr = arr.astype(np.uint8, copy=False)
    bad = set(np.unique(arr).tolist()) - {0, 1}
    if bad:
        raise ValueError(f"mask_keep must be binary {{0,1}}, got values={sorted(set(np.unique(arr).tolist()))}")
    return arr


def _keep_ids(mask: np.ndarray) -> np.ndarray:
    flat = mask.reshape(-1)
    ids = np.flatnonzero(flat)
    return ids.astype(np.uint16 if flat.size <= 0xFFFF else np.uint32, copy=False)


def save_mask_keep_archive(keep_dir, masks_by_stem: Dict[str, np.ndarray], tile_m: int = 64, tile_n: int = 64) -> Path:
    keep_dir = Path(keep_dir)
    keep_dir.mkdir(parents=True, exist_ok=True)
    if not masks_by_stem:
        raise ValueError("masks_by_stem is empty")
    stems = sorted(str(k) for k in masks_by_stem)
    payload: Dict[str, np.ndarray] = {"stems": np.asarray(stems, dtype=np.str_)}
    for i, stem in enumerate(stems):
        mask = _binary(masks_by_stem[stem])
        payload[f"shape_{i}"] = np.asarray(mask.shape, dtype=np.int32)
        payload[f"ids_{i}"] = _keep_ids(mask)
    path = archive_path(keep_dir, tile_m, tile_n)
    np.savez_compressed(path, **payload)
    _CACHE.pop(str(path.resolve()), None)
    return path


def _load(keep_dir, tile_m: int, tile_n: int) -> Dict[str, Tuple[Tuple[int, int], np.ndarray]]:
    path = archive_path(keep_dir, tile_m, tile_n)
    if not path.exists():
        raise FileNotFoundError(f"FP16 keep-id archive not found: {path}")
    key = str(path.resolve())
    if key in _CACHE:
        return _CACHE[key]
    table: Dict[str, Tuple[Tuple[int, int], np.ndarray]] = {}
    with np.load(path, allow_pickle=False) as data:
        for i, stem in enumerate(str(s) for s in np.asarray(data["stems"]).tolist()):
            shape = np.asarray(data[f"shape_{i}"], dtype=np.int64)
            if shape.shape != (2,):
                raise RuntimeError(f"Invalid shape metadata for stem={stem} in {path}")
            n_tr, n_tc = int(shape[0]), int(shape[1])
            ids = np.asarray(data[f"ids_{i}"])
            if ids.dtype not in (np.uint16, np.uint32):
                ids = ids.astype(np.uint32, copy=False)
            if ids.size and int(ids.max()) >= n_tr * n_tc:
                raise RuntimeError(f"Out-of-bound fp16 tile id for stem={stem} in {path}")
            table[stem] = ((n_tr, n_tc), ids)
    _CACHE[key] = table
    return table


def _lookup(keep_dir, layer_name: str, tile_m: int, tile_n: int):
    stem = layer_name_to_stem(layer_name)
    table = _load(keep_dir, tile_m, tile_n)
    if stem not in table:
        raise FileNotFoundError(f"Layer stem not found in archive for layer '{layer_name}': stem={stem}")
    return table[stem]


def _mask(grid: Tuple[int, int], ids: np.ndarray) -> torch.Tensor:
    arr = np.zeros((grid[0] * grid[1],), dtype=np.uint8)
    arr[ids.astype(np.int64, copy=False)] = 1
    return torch.from_numpy(arr.reshape(grid)).contiguous()


def load_mask_keep_for_layer(keep_dir, layer_name: str, tile_m: int = 64, tile_n: int = 64) -> torch.Tensor:
    grid, ids = _lookup(keep_dir, layer_name, tile_m, tile_n)
    return _mask(grid, ids)


def load_fp16_keep_ids_for_layer(keep_dir, layer_name: str, tile_m: int = 64,
                                 tile_n: int = 64) -> Tuple[torch.Tensor, Tuple[int, int]]:
    grid, ids = _lookup(keep_dir, layer_name, tile_m, tile_n)
    return torch.from_numpy(ids.astype(np.int64, copy=False)).to(torch.int32).contiguous(), grid


def load_mask_keep_stem_dict(keep_dir, tile_m: int = 64, tile_n: int = 64) -> Dict[str, torch.Tensor]:
    return {stem: _mask(grid, ids) for stem, (grid, ids) in _load(keep_dir, tile_m, tile_n).items()}


def int8_ids_from_keep(fp16_ids: torch.Tensor, n_tr: int, n_tc: int) -> torch.Tensor:
    """Ascending ids of the INT8 tiles: the complement of the kept (16-bit) ids
    (the reference derives them the same way at load, src/quantization/api.py:112-117)."""
    keep = torch.zeros((n_tr * n_tc,), dtype=torch.bool, device=fp16_ids.device)
    if fp16_ids.numel():
        keep[fp16_ids.to(torch.int64)] = True
    return torch.nonzero(~keep, as_tuple=False).reshape(-1).to(torch.int32)
