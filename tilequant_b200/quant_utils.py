"""Per-64-column activation INT8 quantizer (host side of the CUDA kernels).

Drop-in for the reference's ``src/kernels/quant_utils.py`` (HanzhiZhang-Ulrica/
TileQuant): same function names, arguments, results and exceptions for the
activation quantizer, with every call on the CUDA kernels of ``csrc/quantize.cu``:

* ``activation_tile_absmax_scales``        -- quant_utils.py:41-74
* ``quantize_activation_tile_with_scales`` -- quant_utils.py:78-115
* ``quantize_activation_tile_absmax``      -- quant_utils.py:119-134
* ``pad_to_multiple``                      -- quant_utils.py:152-164

sx[c] = f32(dtype(f32(absmax over all rows of x[:, 64c:64c+64]) / 127)) (1.0 for an
all-zero column tile); q = clamp(rint(f32(x) / sx[c]), -127, 127).  Inputs must be
2-D CUDA tensors of bfloat16 or float16 with ``tile_n == 64`` (the reference's CUDA
path has the same domain); anything else raises instead of falling back.
"""

from __future__ import annotations

from typing import Tuple

import torch

from . import _native as N

INT8_MAX = 127.0
TILE = 64


def _check_2d(x_fp: torch.Tensor, tile_n: int) -> None:
    if x_fp.dim() != 2:
        raise ValueError(f"Expected 2D activation tensor, got shape={tuple(x_fp.shape)}")
    if tile_n <= 0:
        raise ValueError(f"tile_n must be > 0, got {tile_n}")
    if tile_n != TILE:
        raise ValueError(f"tilequant_b200 quantizes 64-column tiles only, got tile_n={tile_n}")
    N.require_cuda(x_fp)
    N.dtype_code(x_fp.dtype)


def activation_tile_absmax_scales(x_fp: torch.Tensor, tile_n: int = 64) -> torch.Tensor:
    """f32[n_tc] scales of the 64-column tiles of ``x_fp`` (quant_utils.py:41-74).  Zero
    rows with columns raise IndexError, as the reference's amax over the empty row
    dimension does (quant_utils.py:68-69); ``quantize_activation_tile_absmax`` instead
    gives scale 1.0 per tile there, like the reference's fused kernel."""
    _check_2d(x_fp, tile_n)
    n, k = x_fp.shape
    n_tc = (int(k) + TILE - 1) // TILE
    sx = torch.empty((n_tc,), device=x_fp.device, dtype=torch.float32)
    if k == 0:
        return sx
    if n == 0:
        raise IndexError("activation_tile_absmax_scales: x has no rows (a maximum over an empty dimension)")
    rc = N.load().tq_act_scales(x_fp.data_ptr(), N.dtype_code(x_fp.dtype), int(n), int(k), x_fp.stride(0),
                                x_fp.stride(1), sx.data_ptr(), N.stream_of(x_fp))
    N.check(rc, "activation_tile_absmax_scales")
    return sx


def quantize_activation_tile_with_scales(x_fp: torch.Tensor, sx: torch.Tensor, tile_n: int = 64) -> torch.Tensor:
    """INT8 codes of ``x_fp`` given the tile scales (quant_utils.py:78-115)."""
    _check_2d(x_fp, tile_n)
    n, k = x_fp.shape
    if k == 0:
        return torch.zeros_like(x_fp, dtype=torch.int8)
    n_tc = (int(k) + TILE - 1) // TILE
    if sx.numel() != n_tc:
        raise ValueError(f"Scale length mismatch: got {sx.numel()}, expected {n_tc}")
    sx_work = sx.to(device=x_fp.device, dtype=torch.float32).contiguous()
    q = torch.empty((n, k), device=x_fp.device, dtype=torch.int8)
    rc = N.load().tq_quantize_with_scales(x_fp.data_ptr(), N.dtype_code(x_fp.dtype), int(n), int(k), x_fp.stride(0),
                                          x_fp.stride(1), sx_work.data_ptr(), q.data_ptr(), int(k), N.stream_of(x_fp))
    N.check(rc, "quantize_activation_tile_with_scales")
    return q


def quantize_activation_tile_absmax(x_fp: torch.Tensor, tile_n: int = 64) -> Tuple[torch.Tensor, torch.Tensor]:
    """(INT8 codes, f32 tile scales) in one call (quant_utils.py:119-134)."""
    _check_2d(x_fp, tile_n)
    n, k = x_fp.shape
    n_tc = (int(k) + TILE - 1) // TILE
    q = torch.empty((n, k), device=x_fp.device, dtype=torch.int8)
    sx = torch.empty((n_tc,), device=x_fp.device, dtype=torch.float32)
    if k == 0:
        return q, sx
    rc = N.load().tq_quantize_act(x_fp.data_ptr(), N.dtype_code(x_fp.dtype), int(n), int(k), x_fp.stride(0),
                                  x_fp.stride(1), q.data_ptr(), int(k), sx.data_ptr(), N.stream_of(x_fp))
    N.check(rc, "quantize_activation_tile_absmax")
    return q, sx


def pad_to_multiple(W: torch.Tensor, multiple: int = 64) -> Tuple[torch.Tensor, int, int]:
    """Zero-pad a 2-D weight to multiples of ``multiple`` (quant_utils.py:152-164)."""
    if W.dim() != 2:
        raise ValueError(f"Expected 2D weight tensor, got shape={tuple(W.shape)}")
    M, K = W.shape
    M_pad = ((M + multiple - 1) // multiple) * multiple
    K_pad = ((K + multiple - 1) // multiple) * multiple
    if M_pad == M and K_pad == K:
        return W, M, K
    W_pad = W.new_zeros((M_pad, K_pad))
    W_pad[:M, :K] = W
    return W_pad, M_pad, K_pad
