"""Load-time tile packer (host side of ``csrc/pack.cu``).

Drop-in for the reference's ``src/kernels/pack.py`` (HanzhiZhang-Ulrica/TileQuant):
the same ``Pack`` fields and tensor layouts (int8[T8][64][64] codes, f32[T8] scales,
sorted int32 tile ids, CSR row pointers, 16-bit [T16][64][64] tiles), the same
``cfg`` keys and errors.  The per-tile work (absmax scale, IAA scale search, INT8
codes, 16-bit gather) runs in CUDA kernels; the id sort and CSR row pointers are
index bookkeeping on the device.

* ``Pack``                       -- pack.py:11-29
* ``pack_weight_from_tile_ids``  -- pack.py:206-224 (body :65-203)
* ``pack_weight``                -- pack.py:227-236
* ``is_row_major_pack``          -- pack.py:239-243
* ``concat_packs_along_rows``    -- pack.py:246-321

Packing happens on a CUDA device: ``W_fp`` on the CPU is copied to ``device`` (default
the current CUDA device) and the returned Pack lives there.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, Optional, Sequence

import torch

from . import _native as N


@dataclass
class Pack:
    M_orig: int
    K_orig: int
    M: int
    K: int
    tile_m: int
    tile_n: int
    n_tr: int
    n_tc: int
    int8_tiles: torch.Tensor
    int8_scales: torch.Tensor
    int8_tile_ids: torch.Tensor
    int8_row_ptr: torch.Tensor
    int8_row_indices: torch.Tensor
    fp16_tiles: torch.Tensor
    fp16_tile_ids: torch.Tensor
    fp16_row_ptr: torch.Tensor
    fp16_row_indices: torch.Tensor


def _cfg_get(cfg: Any, key: str, default=None):
    if isinstance(cfg, dict):
        return cfg.get(key, default)
    return getattr(cfg, key, default)


def _sorted_ids(tile_ids: torch.Tensor) -> torch.Tensor:
    """Tile ids in ascending (row-major) order: the tiles of row tile r then occupy
    one contiguous run of the arena, in ascending input-column order."""
    return tile_ids.sort().values.contiguous() if tile_ids.numel() > 1 else tile_ids.contiguous()


def _csr_rows(sorted_ids: torch.Tensor, *, n_tr: int, n_tc: int):
    """CSR pointers of a sorted id list: row_ptr[r] = #ids below r * n_tc.  Also the
    reference's ``row_indices`` field, which for a sorted unique list is 0..T-1."""
    bounds = torch.arange(n_tr + 1, device=sorted_ids.device, dtype=torch.int64) * n_tc
    row_ptr = torch.searchsorted(sorted_ids, bounds).to(torch.int32)
    return row_ptr, torch.arange(sorted_ids.numel(), device=sorted_ids.device, dtype=torch.int32)


def _validate_ids(int8_ids: torch.Tensor, fp16_ids: torch.Tensor, total: int) -> None:
    """Reject a map whose ids are out of range, repeated, or shared by both lists
    before any kernel reads tiles through them (host-side check, load time only)."""
    both = torch.cat([int8_ids, fp16_ids])
    if both.numel() == 0:
        return
    lo, hi = int(both.min()), int(both.max())
    if lo < 0 or hi >= total:
        raise ValueError(f"tile id out of range [0, {total}): min={lo} max={hi}")
    if int(torch.unique(both).numel()) != int(both.numel()):
        raise ValueError("tile ids repeat within or across the INT8 and 16-bit lists")


def _pack_weight_with_tile_ids(W_fp: torch.Tensor, *, n_tr: int, n_tc: int, int8_tile_ids: torch.Tensor,
                               fp16_tile_ids: torch.Tensor, iaa_col_importance: Optional[torch.Tensor], cfg: Any,
                               device: Optional[torch.device] = None) -> Pack:
    if W_fp.dim() != 2:
        raise ValueError(f"Expected W to be 2D, got shape={tuple(W_fp.shape)}")
    tile_m = int(_cfg_get(cfg, "tile_m", 64))
    tile_n = int(_cfg_get(cfg, "tile_n", 64))
    use_pad = bool(_cfg_get(cfg, "pad_to_tile", True))
    quant_style = str(_cfg_get(cfg, "quant_style", "gi")).lower()
    if quant_style not in ("gi", "iaa"):
        raise ValueError(f"Unsupported quant_style={quant_style}. Expected one of: gi, iaa")
    if tile_m != 64 or tile_n != 64:
        raise ValueError(f"tilequant_b200 packs 64x64 tiles only, got {tile_m}x{tile_n}")

    M_orig, K_orig = (int(v) for v in W_fp.shape)
    if use_pad:
        M = ((M_orig + 63) // 64) * 64
        K = ((K_orig + 63) // 64) * 64
    else:
        if (M_orig % tile_m) != 0 or (K_orig % tile_n) != 0:
            raise ValueError("pad_to_tile=False but weight shape is not multiple of tile size")
        M, K = M_orig, K_orig
    if n_tr * tile_m != M or n_tc * tile_n != K:
        raise ValueError(
            f"PrecisionMap dimensions mismatch: map(n_tr={n_tr}, n_tc={n_tc}) "
            f"vs weight(M={M}, K={K}, tile_m={tile_m}, tile_n={tile_n})"
        )
    if device is None:
        device = W_fp.device if W_fp.is_cuda else torch.device("cuda", torch.cuda.current_device())
    dcode = N.dtype_code(W_fp.dtype)
    W = W_fp.to(device=device)
    if W.stride(1) != 1:
        W = W.contiguous()

    int8_ids = _sorted_ids(int8_tile_ids.to(device=device, dtype=torch.int64).reshape(-1))
    fp16_ids = _sorted_ids(fp16_tile_ids.to(device=device, dtype=torch.int64).reshape(-1))
    t8, t16 = int(int8_ids.numel()), int(fp16_ids.numel())
    if t8 + t16 != n_tr * n_tc:
        raise RuntimeError(f"Packed tile count mismatch: T8={t8}, T16={t16}, total={n_tr * n_tc}")
    _validate_ids(int8_ids, fp16_ids, n_tr * n_tc)
    int8_row_ptr, int8_row_indices = _csr_rows(int8_ids, n_tr=n_tr, n_tc=n_tc)
    fp16_row_ptr, fp16_row_indices = _csr_rows(fp16_ids, n_tr=n_tr, n_tc=n_tc)
    ids8_i32 = int8_ids.to(torch.int32).contiguous()
    ids16_i32 = fp16_ids.to(torch.int32).contiguous()
    lib = N.load()
    stream = torch.cuda.current_stream(device).cuda_stream

    int8_tiles = torch.empty((t8, 64, 64), device=device, dtype=torch.int8)
    int8_scales = torch.empty((t8,), device=device, dtype=torch.float32)
    if t8:
        col_imp = None
        if quant_style == "iaa" and iaa_col_importance is not None:
            src = iaa_col_importance.to(device=device, dtype=torch.float32).reshape(-1)
            col_imp = torch.zeros((K,), device=device, dtype=torch.float32)
            n = min(int(src.numel()), K)
            col_imp[:n] = src[:n]
        with torch.cuda.device(device):
            rc = lib.tq_pack_int8_tiles(W.data_ptr(), dcode, M_orig, K_orig, W.stride(0), n_tc, ids8_i32.data_ptr(),
                                        t8, N.ptr(col_imp), int8_tiles.data_ptr(), int8_scales.data_ptr(), stream)
        N.check(rc, "pack_weight_from_tile_ids")
    fp16_tiles = torch.empty((t16, 64, 64), device=device, dtype=W_fp.dtype)
    if t16:
        with torch.cuda.device(device):
            rc = lib.tq_gather_fp_tiles(W.data_ptr(), dcode, M_orig, K_orig, W.stride(0), n_tc, ids16_i32.data_ptr(),
                                        t16, fp16_tiles.data_ptr(), stream)
        N.check(rc, "pack_weight_from_tile_ids")

    return Pack(
        M_orig=M_orig, K_orig=K_orig, M=M, K=K, tile_m=tile_m, tile_n=tile_n, n_tr=n_tr, n_tc=n_tc,
        int8_tiles=int8_tiles, int8_scales=int8_scales, int8_tile_ids=ids8_i32,
        int8_row_ptr=int8_row_ptr.contiguous(), int8_row_indices=int8_row_indices.contiguous(),
        fp16_tiles=fp16_tiles, fp16_tile_ids=ids16_i32,
        fp16_row_ptr=fp16_row_ptr.contiguous(), fp16_row_indices=fp16_row_indices.contiguous(),
    )


def pack_weight_from_tile_ids(W_fp: torch.Tensor, *, n_tr: int, n_tc: int, int8_tile_ids: torch.Tensor,
                              fp16_tile_ids: torch.Tensor, iaa_col_importance: Optional[torch.Tensor] = None,
                              cfg: Any, device: Optional[torch.device] = None) -> Pack:
    return _pack_weight_with_tile_ids(W_fp=W_fp, n_tr=int(n_tr), n_tc=int(n_tc), int8_tile_ids=int8_tile_ids,
                                      fp16_tile_ids=fp16_tile_ids, iaa_col_importance=iaa_col_importance, cfg=cfg,
                                      device=device)


def pack_weight(W_fp: torch.Tensor, pmap: Dict[str, Any], cfg: Any, device: Optional[torch.device] = None) -> Pack:
    return _pack_weight_with_tile_ids(W_fp=W_fp, n_tr=int(pmap["n_tr"]), n_tc=int(pmap["n_tc"]),
                                      int8_tile_ids=pmap["int8_tile_ids"], fp16_tile_ids=pmap["fp16_tile_ids"],
                                      iaa_col_importance=None, cfg=cfg, device=device)


def is_row_major_pack(pack: Pack) -> bool:
    for ids in (pack.int8_tile_ids, pack.fp16_tile_ids):
        if ids.numel() > 1 and not bool((ids[1:] > ids[:-1]).all()):
            return False
    return True


def concat_packs_along_rows(packs: Sequence[Pack]) -> Pack:
    """Stack packs of projections that share one input along the output rows.

    Members need the same input geometry and tile-aligned output widths, so member
    row tiles map one-to-one onto consecutive stacked row tiles and every member's
    output is an exact column slice; payloads and scales are copied unchanged
    (same contract as the reference's pack.py:246-321)."""
    if not packs:
        raise ValueError("Expected at least one pack")
    first = packs[0]
    geometry = (first.K_orig, first.K, first.tile_m, first.tile_n, first.n_tc)
    for pack in packs:
        if (pack.K_orig, pack.K, pack.tile_m, pack.tile_n, pack.n_tc) != geometry:
            raise ValueError("Packs must share input geometry to be stacked")
        if pack.M_orig != pack.M or pack.M_orig % pack.tile_m != 0:
            raise ValueError("Stacked packs require tile-aligned output widths")
        if not is_row_major_pack(pack):
            raise ValueError("Stacked packs require row-major tile order")
    n_tc = first.n_tc
    dev = first.int8_tiles.device
    # member i starts at stacked row tile row0[i]; its tiles shift by the tiles before it
    row0 = [0]
    for pack in packs[:-1]:
        row0.append(row0[-1] + pack.n_tr)

    def stacked(kind: str):
        counts = [int(getattr(p, f"{kind}_tile_ids").numel()) for p in packs]
        before = [sum(counts[:i]) for i in range(len(packs))]
        ids = torch.cat([getattr(p, f"{kind}_tile_ids").to(torch.int64) + row0[i] * n_tc
                         for i, p in enumerate(packs)]).to(torch.int32)
        ptr = torch.cat([torch.zeros((1,), dtype=torch.int32, device=dev)] +
                        [getattr(p, f"{kind}_row_ptr")[1:].to(torch.int32) + before[i] for i, p in enumerate(packs)])
        idx = torch.cat([getattr(p, f"{kind}_row_indices").to(torch.int32) + before[i] for i, p in enumerate(packs)])
        tiles = torch.cat([getattr(p, f"{kind}_tiles") for p in packs], dim=0)
        return tiles.contiguous(), ids.contiguous(), ptr.contiguous(), idx.contiguous()

    int8_tiles, int8_ids, int8_row_ptr, int8_row_indices = stacked("int8")
    fp16_tiles, fp16_ids, fp16_row_ptr, fp16_row_indices = stacked("fp16")
    int8_scales = torch.cat([p.int8_scales for p in packs]).contiguous()
    M = sum(pack.M for pack in packs)
    return Pack(M_orig=M, K_orig=first.K_orig, M=M, K=first.K, tile_m=first.tile_m, tile_n=first.tile_n,
                n_tr=sum(pack.n_tr for pack in packs), n_tc=n_tc, int8_tiles=int8_tiles, int8_scales=int8_scales,
                int8_tile_ids=int8_ids, int8_row_ptr=int8_row_ptr, int8_row_indices=int8_row_indices,
                fp16_tiles=fp16_tiles, fp16_tile_ids=fp16_ids, fp16_row_ptr=fp16_row_ptr,
                fp16_row_indices=fp16_row_indices)
