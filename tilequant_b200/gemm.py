"""Mixed INT8/BF16 64x64 tile GEMM (host side of ``csrc/gemm*.cu``).

``gemm_mixed_rows_splitk`` is a drop-in for the reference function of the same name
(src/kernels/triton/gemm_rows_splitk_64x64.py:225-323): same keyword arguments,
result and errors.  The numerics are the reference kernel's (:78-190): per output
row tile and split, exact INT32 tile products scaled by ``sx[c] * sw`` and added in
ascending column order, then the 16-bit tiles, split partials added in split order,
rounded to ``out_dtype``, then ``bias`` added the way the reference adds it.

There is no per-(device, stream) workspace: split-K partials meet in distributed
shared memory inside one launch (see ``csrc/gemm_rows.cu``), so nothing has to stay
allocated across calls or CUDA-graph captures.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _native as N

SPLITK_MAX = 16


def select_split_k(*, n_tr: int, n_blocks: int = 1, n_tc: int, device: torch.device, n_rows: Optional[int] = None,
                   dtype: torch.dtype = torch.bfloat16, fused: bool = False) -> int:
    """Split count the row kernel uses when ``split_k`` is None.

    The reference picks it by a fixed rule (gemm_rows_splitk_64x64.py:52-67, about 4
    CTAs per SM); here the grid is sized to one wave of resident CTAs of this device
    (see ``tq_gemm_rows_plan``).  The split fixes the FP32 summation order; passing the
    returned value as ``split_k`` gives the same result."""
    import ctypes

    rows = int(n_rows) if n_rows is not None else 16 * int(n_blocks)
    sp, rpc = ctypes.c_int(0), ctypes.c_int(0)
    index = device.index if device.index is not None else torch.cuda.current_device()
    with torch.cuda.device(index):
        rc = N.load().tq_gemm_rows_plan(rows, int(n_tr), int(n_tc), N.dtype_code(dtype), int(fused),
                                        ctypes.byref(sp), ctypes.byref(rpc))
    N.check(rc, "select_split_k")
    return int(sp.value)


def _check_common(int8_tiles, int8_scales, int8_tile_ids, int8_row_ptr, fp16_tiles, fp16_tile_ids, fp16_row_ptr,
                  M, K, n_tr, n_tc):
    if int8_tiles.dtype != torch.int8 or (int8_tiles.numel() and tuple(int8_tiles.shape[1:]) != (64, 64)):
        raise ValueError("int8_tiles must be int8 [T8, 64, 64]")
    if int8_scales.dtype != torch.float32 or int8_scales.numel() != int8_tiles.shape[0]:
        raise ValueError("int8_scales must be float32 [T8]")
    for name, t in (("int8_tile_ids", int8_tile_ids), ("int8_row_ptr", int8_row_ptr),
                    ("fp16_tile_ids", fp16_tile_ids), ("fp16_row_ptr", fp16_row_ptr)):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous int32 tensor")
    if int8_row_ptr.numel() != int(n_tr) + 1 or (fp16_tiles.numel() and fp16_row_ptr.numel() != int(n_tr) + 1):
        raise ValueError("row_ptr must have n_tr + 1 entries")
    if int(n_tr) != (int(M) + 63) // 64 or int(n_tc) != (int(K) + 63) // 64:
        raise ValueError(f"tile grid ({n_tr}, {n_tc}) does not match (M={M}, K={K})")
    if int8_tiles.shape[0] + fp16_tiles.shape[0] != int(n_tr) * int(n_tc):
        raise ValueError("INT8 + 16-bit tiles must cover the n_tr x n_tc grid")
    for t in (int8_tiles, int8_scales, fp16_tiles):
        if not t.is_contiguous():
            raise ValueError("tile arenas and scales must be contiguous")


def gemm_mixed_rows_splitk(
    *,
    x_fp: torch.Tensor,
    x_int8: torch.Tensor,
    sx: torch.Tensor,
    int8_tiles: torch.Tensor,
    int8_scales: torch.Tensor,
    int8_tile_ids: torch.Tensor,
    int8_row_ptr: torch.Tensor,
    fp16_tiles: torch.Tensor,
    fp16_tile_ids: torch.Tensor,
    fp16_row_ptr: torch.Tensor,
    M: int,
    K: int,
    n_tr: int,
    n_tc: int,
    out_dtype: torch.dtype,
    bias: Optional[torch.Tensor] = None,
    split_k: Optional[int] = None,
    out: Optional[torch.Tensor] = None,
    algo: int = N.TQ_ALGO_AUTO,
) -> torch.Tensor:
    """Return ``x @ W^T (+ bias)`` for a row-major packed mixed INT8/16-bit weight.

    ``bias`` must already have dtype ``out_dtype`` and be contiguous.  ``out``
    (optional) is an (N, M) tensor with unit column stride to write into.
    """
    device = N.require_cuda(x_fp, x_int8, sx, int8_tiles, fp16_tiles, out, bias)
    n = int(x_fp.shape[0])
    _check_common(int8_tiles, int8_scales, int8_tile_ids, int8_row_ptr, fp16_tiles, fp16_tile_ids, fp16_row_ptr,
                  M, K, n_tr, n_tc)
    if x_fp.dim() != 2 or x_fp.shape[1] != int(K) or x_fp.stride(1) != 1:
        raise ValueError("x_fp must be (N, K) with unit column stride")
    if x_int8.dtype != torch.int8 or tuple(x_int8.shape) != (n, int(K)) or x_int8.stride(1) != 1:
        raise ValueError("x_int8 must be int8 (N, K) with unit column stride")
    if sx.dtype != torch.float32 or sx.numel() != int(n_tc) or not sx.is_contiguous():
        raise ValueError("sx must be contiguous float32 [n_tc]")
    if fp16_tiles.numel() and fp16_tiles.dtype != x_fp.dtype:
        raise ValueError("fp16_tiles and x_fp must share one 16-bit dtype")
    if out is None:
        out = torch.empty((n, int(M)), device=device, dtype=out_dtype)
    elif tuple(out.shape) != (n, int(M)) or out.dtype != out_dtype or out.stride(1) != 1:
        raise ValueError("out must be an (N, M) tensor of out_dtype with unit column stride")
    if bias is not None and (bias.dtype != out_dtype or not bias.is_contiguous() or bias.numel() != int(M)):
        raise ValueError("bias must be a contiguous [M] tensor of out_dtype")
    if split_k is not None and not 1 <= int(split_k) <= SPLITK_MAX:
        raise ValueError(f"split_k must be in 1..{SPLITK_MAX}")
    if n == 0:
        return out
    t8, t16 = int(int8_tiles.shape[0]), int(fp16_tiles.shape[0])
    rc = N.load().tq_gemm_mixed(
        x_int8.data_ptr(), x_int8.stride(0), sx.data_ptr(), int8_tiles.data_ptr(), int8_scales.data_ptr(),
        int8_tile_ids.data_ptr(), int8_row_ptr.data_ptr(), t8, x_fp.data_ptr(), x_fp.stride(0),
        fp16_tiles.data_ptr() if t16 else None, fp16_tile_ids.data_ptr() if t16 else None,
        fp16_row_ptr.data_ptr() if t16 else None, t16, N.dtype_code(x_fp.dtype), out.data_ptr(), out.stride(0),
        N.dtype_code(out_dtype), N.ptr(bias), n, int(M), int(K), int(n_tr), int(n_tc),
        0 if split_k is None else int(split_k), int(algo), None, torch.cuda.current_stream(device).cuda_stream)
    N.check(rc, "gemm_mixed_rows_splitk")
    return out


def gemm_mixed_fused_quant(
    *,
    x_fp: torch.Tensor,
    int8_tiles: torch.Tensor,
    int8_scales: torch.Tensor,
    int8_tile_ids: torch.Tensor,
    int8_row_ptr: torch.Tensor,
    fp16_tiles: torch.Tensor,
    fp16_tile_ids: torch.Tensor,
    fp16_row_ptr: torch.Tensor,
    M: int,
    K: int,
    n_tr: int,
    n_tc: int,
    out_dtype: torch.dtype,
    bias: Optional[torch.Tensor] = None,
    split_k: Optional[int] = None,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Decode form (N <= 64): the activation quantizer runs inside the GEMM launch.

    Same result as ``quantize_activation_tile_absmax`` followed by
    ``gemm_mixed_rows_splitk``, in one kernel launch."""
    device = N.require_cuda(x_fp, int8_tiles, fp16_tiles, out, bias)
    n = int(x_fp.shape[0])
    if n > 64:
        raise ValueError("gemm_mixed_fused_quant handles at most 64 activation rows")
    _check_common(int8_tiles, int8_scales, int8_tile_ids, int8_row_ptr, fp16_tiles, fp16_tile_ids, fp16_row_ptr,
                  M, K, n_tr, n_tc)
    if x_fp.dim() != 2 or x_fp.shape[1] != int(K) or x_fp.stride(1) != 1:
        raise ValueError("x_fp must be (N, K) with unit column stride")
    if fp16_tiles.numel() and fp16_tiles.dtype != x_fp.dtype:
        raise ValueError("fp16_tiles and x_fp must share one 16-bit dtype")
    if out is None:
        out = torch.empty((n, int(M)), device=device, dtype=out_dtype)
    elif tuple(out.shape) != (n, int(M)) or out.dtype != out_dtype or out.stride(1) != 1:
        raise ValueError("out must be an (N, M) tensor of out_dtype with unit column stride")
    if bias is not None and (bias.dtype != out_dtype or not bias.is_contiguous() or bias.numel() != int(M)):
        raise ValueError("bias must be a contiguous [M] tensor of out_dtype")
    if split_k is not None and not 1 <= int(split_k) <= SPLITK_MAX:
        raise ValueError(f"split_k must be in 1..{SPLITK_MAX}")
    if n == 0:
        return out
    t8, t16 = int(int8_tiles.shape[0]), int(fp16_tiles.shape[0])
    rc = N.load().tq_gemm_mixed_fused_quant(
        x_fp.data_ptr(), x_fp.stride(0), N.dtype_code(x_fp.dtype), int8_tiles.data_ptr(), int8_scales.data_ptr(),
        int8_tile_ids.data_ptr(), int8_row_ptr.data_ptr(), t8, fp16_tiles.data_ptr() if t16 else None,
        fp16_tile_ids.data_ptr() if t16 else None, fp16_row_ptr.data_ptr() if t16 else None, t16, out.data_ptr(),
        out.stride(0), N.dtype_code(out_dtype), N.ptr(bias), n, int(M), int(K), int(n_tr), int(n_tc),
        0 if split_k is None else int(split_k), None, torch.cuda.current_stream(device).cuda_stream)
    N.check(rc, "gemm_mixed_fused_quant")
    return out


def gemm_int8_partials(*, x_int8: torch.Tensor, int8_tiles: torch.Tensor, int8_tile_ids: torch.Tensor,
                       int8_row_ptr: torch.Tensor, K: int, n_tr: int, n_tc: int,
                       algo: int = N.TQ_ALGO_ROWS) -> torch.Tensor:
    """Debug view of the exact INT32 tile products the GEMM kernel forms:
    int32[T8, N, 64], ``[t, n, j] = sum_k x_int8[n, 64c + k] * int8_tiles[t, j, k]``."""
    device = N.require_cuda(x_int8, int8_tiles)
    n = int(x_int8.shape[0])
    t8 = int(int8_tiles.shape[0])
    parts = torch.zeros((t8, n, 64), device=device, dtype=torch.int32)
    if n == 0 or t8 == 0:
        return parts
    rc = N.load().tq_gemm_int8_partials(
        x_int8.data_ptr(), x_int8.stride(0), int8_tiles.data_ptr(), int8_tile_ids.data_ptr(),
        int8_row_ptr.data_ptr(), t8, n, int(K), int(n_tr), int(n_tc), parts.data_ptr(), int(algo),
        torch.cuda.current_stream(device).cuda_stream)
    N.check(rc, "gemm_int8_partials")
    return parts
