"""TEST INFRASTRUCTURE ONLY: the CPU oracle for the TileQuant mixed tile GEMM path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline``
leg and its ``--impl reference`` arm) may import this module, and only as the
checker or as the timed CPU baseline.  The product package ``tilequant_b200``
never imports it and has no CPU fallback.

It wraps ``tq_oracle.c`` (a plain C restatement of the reference's arithmetic,
file:line citations in that file) through ctypes, plus numpy restatements of the
reference's host-side index work:

* tile-id sorting and CSR row pointers   -- src/kernels/pack.py:38-62
* BF16 tile gather                        -- src/kernels/pack.py:172-177
* int8 ids as the complement of keep ids  -- src/quantization/api.py:112-117
* top-k keep mask                         -- src/quantization/decisions.py:174-183

Parity of the restatement is pinned by ``tests/test_oracle_golden.py`` against
fixtures written by ``tests/golden/make_golden.py``, which runs the reference
implementation itself (its CPU quantizer and packer, and its Triton GEMM kernel
under the Triton interpreter).
"""

from __future__ import annotations

import ctypes
import math
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
SRC_PATH = HERE / "tq_oracle.c"

BF16, F16 = 0, 1

_lib = None


def build(force: bool = False) -> Path:
    """Compile tq_oracle.c with gcc (no fast-math, no FP contraction)."""
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < SRC_PATH.stat().st_mtime:
        tmp = LIB_PATH.with_suffix(".so.tmp")
        subprocess.check_call(
            ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC", "-shared",
             "-o", str(tmp), str(SRC_PATH), "-lm"]
        )
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.tqo_act_scales.argtypes = [P, I, I64, I64, I64, I64, P]
        L.tqo_quantize_with_scales.argtypes = [P, I, I64, I64, I64, I64, P, P]
        L.tqo_pack_int8.argtypes = [P, I, I64, I64, I64, I, P, I64, P, P, P]
        L.tqo_gemm_mixed.argtypes = [P, I64, P, P, P, P, P, P, I64, I, P, P, P, P, I64, I, P,
                                     I64, I64, I64, I, I, I, I, P, P]
        L.tqo_calib_gi_accumulate.argtypes = [P, P, I, I64, I64, I, I, P]
        L.tqo_iaa_channel_accumulate.argtypes = [P, I, I64, I64, P]
        L.tqo_iaa_tile_scores.argtypes = [P, I, I64, I64, I, I, P, I64, P, P]
        L.tqo_set_threads.argtypes = [I]
        L.tqo_set_threads.restype = I
        for fn in ("tqo_act_scales", "tqo_quantize_with_scales", "tqo_pack_int8", "tqo_gemm_mixed",
                   "tqo_calib_gi_accumulate", "tqo_iaa_channel_accumulate", "tqo_iaa_tile_scores"):
            getattr(L, fn).restype = None
        _lib = L
    return _lib


def set_threads(n: int) -> int:
    """Threads of the restatement's OpenMP loops on the calling thread (whatever
    OMP_NUM_THREADS the process inherited, e.g. 1 under torchrun); returns the count
    its next loop will use."""
    return int(lib().tqo_set_threads(int(n)))


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _h16(a: np.ndarray) -> np.ndarray:
    if a.dtype != np.uint16:
        raise TypeError("16-bit float arrays are passed as uint16 bit patterns")
    return a


# ------------------------------------------------------------ bf16 helpers (numpy)

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def h_to_f32(bits: np.ndarray, dtype: int) -> np.ndarray:
    return bf16_bits_to_f32(bits) if dtype == BF16 else bits.view(np.float16).astype(np.float32)


# ------------------------------------------------------------ activation quantizer

def act_scales(x_bits: np.ndarray, dtype: int = BF16) -> np.ndarray:
    x_bits = _h16(x_bits)
    n, k = x_bits.shape
    sx = np.empty(((k + 63) // 64,), np.float32)
    lib().tqo_act_scales(_ptr(x_bits), dtype, n, k, x_bits.strides[0] // 2, x_bits.strides[1] // 2, _ptr(sx))
    return sx


def quantize_with_scales(x_bits: np.ndarray, sx: np.ndarray, dtype: int = BF16) -> np.ndarray:
    x_bits = _h16(x_bits)
    n, k = x_bits.shape
    sx = np.ascontiguousarray(sx, np.float32)
    q = np.empty((n, k), np.int8)
    lib().tqo_quantize_with_scales(_ptr(x_bits), dtype, n, k, x_bits.strides[0] // 2,
                                   x_bits.strides[1] // 2, _ptr(sx), _ptr(q))
    return q


def quantize_act(x_bits: np.ndarray, dtype: int = BF16):
    sx = act_scales(x_bits, dtype)
    return quantize_with_scales(x_bits, sx, dtype), sx


# ------------------------------------------------------------------------ packer

def row_schedule(tile_ids: np.ndarray, n_tr: int, n_tc: int):
    """Sorted int32 ids and CSR row_ptr (pack.py:38-62)."""
    ids = np.sort(np.asarray(tile_ids, np.int64))
    rows = ids // n_tc if ids.size else np.zeros((0,), np.int64)
    counts = np.bincount(rows, minlength=n_tr).astype(np.int64)
    row_ptr = np.zeros((n_tr + 1,), np.int32)
    row_ptr[1:] = np.cumsum(counts)
    return ids.astype(np.int32), row_ptr


def int8_ids_from_keep(fp16_ids: np.ndarray, n_tr: int, n_tc: int) -> np.ndarray:
    """Complement of the BF16 keep ids, ascending (api.py:112-117)."""
    mask = np.zeros((n_tr * n_tc,), bool)
    mask[np.asarray(fp16_ids, np.int64)] = True
    return np.flatnonzero(~mask).astype(np.int32)


def pack(w_bits: np.ndarray, n_tr: int, n_tc: int, int8_ids, fp16_ids, dtype: int = BF16,
         col_importance: np.ndarray | None = None) -> dict:
    """Restatement of _pack_weight_with_tile_ids (pack.py:65-203), pad_to_tile=True."""
    w_bits = np.ascontiguousarray(_h16(w_bits))
    m, k = w_bits.shape
    if n_tr * 64 != ((m + 63) // 64) * 64 or n_tc * 64 != ((k + 63) // 64) * 64:
        raise ValueError("map dimensions mismatch")
    ids8, rp8 = row_schedule(int8_ids, n_tr, n_tc)
    ids16, rp16 = row_schedule(fp16_ids, n_tr, n_tc)
    if ids8.size + ids16.size != n_tr * n_tc:
        raise RuntimeError("Packed tile count mismatch")
    t8 = ids8.size
    tiles = np.empty((t8, 64, 64), np.int8)
    scales = np.empty((t8,), np.float32)
    ci = None
    if col_importance is not None:
        ci = np.zeros((n_tc * 64,), np.float32)
        src = np.asarray(col_importance, np.float32).reshape(-1)[: n_tc * 64]
        ci[: src.size] = src
    lib().tqo_pack_int8(_ptr(w_bits), dtype, m, k, k, n_tc, _ptr(ids8), t8, _ptr(ci), _ptr(tiles), _ptr(scales))
    wp = np.zeros((n_tr * 64, n_tc * 64), np.uint16)
    wp[:m, :k] = w_bits
    tv = wp.reshape(n_tr, 64, n_tc, 64).transpose(0, 2, 1, 3)
    fp_tiles = np.ascontiguousarray(tv[ids16 // n_tc, ids16 % n_tc]) if ids16.size else np.zeros((0, 64, 64), np.uint16)
    return dict(M_orig=m, K_orig=k, M=n_tr * 64, K=n_tc * 64, n_tr=n_tr, n_tc=n_tc,
                int8_tiles=tiles, int8_scales=scales, int8_tile_ids=ids8, int8_row_ptr=rp8,
                fp16_tiles=fp_tiles, fp16_tile_ids=ids16, fp16_row_ptr=rp16)


# -------------------------------------------------------------------------- GEMM

def select_split_k_reference(n_tr: int, n_blocks: int, n_tc: int, sm_count: int) -> int:
    """The reference's split heuristic (gemm_rows_splitk_64x64.py:52-67)."""
    target = 4 * sm_count
    ctas = max(1, n_tr * n_blocks)
    if ctas >= target:
        return 1
    split = 1 << max(0, (target + ctas - 1) // ctas - 1).bit_length()
    split = min(split, 16)
    while split > 1 and n_tc // split < 4:
        split //= 2
    return max(1, split)


def gemm(x_i8, sx, pk: dict, x_bits, M: int, K: int, *, split_k: int = 1, bias_bits=None,
         xdtype: int = BF16, odtype: int = BF16, use_fma: bool = True, want_partials: bool = False,
         want_f32: bool = False):
    """Restatement of the mixed GEMM (gemm_rows_splitk_64x64.py:108-190).

    Returns the output as uint16 bits of ``odtype``, then (when asked) the INT32 tile
    partials [t8, n_rows, 64] and the FP32 sums before the output rounding [n_rows, M]."""
    x_i8 = np.ascontiguousarray(x_i8, np.int8)
    x_bits = np.ascontiguousarray(_h16(x_bits))
    n = x_i8.shape[0]
    out = np.zeros((n, M), np.uint16)
    t8 = pk["int8_tiles"].shape[0]
    parts = np.zeros((t8, n, 64), np.int32) if want_partials else None
    acc = np.zeros((n, M), np.float32) if want_f32 else None
    w16 = np.ascontiguousarray(pk["fp16_tiles"], np.uint16)
    bias = None if bias_bits is None else np.ascontiguousarray(bias_bits, np.uint16)
    lib().tqo_gemm_mixed(
        _ptr(x_i8), x_i8.strides[0], _ptr(np.ascontiguousarray(sx, np.float32)),
        _ptr(np.ascontiguousarray(pk["int8_tiles"], np.int8)),
        _ptr(np.ascontiguousarray(pk["int8_scales"], np.float32)),
        _ptr(np.ascontiguousarray(pk["int8_tile_ids"], np.int32)),
        _ptr(np.ascontiguousarray(pk["int8_row_ptr"], np.int32)),
        _ptr(x_bits), x_bits.strides[0] // 2, xdtype, _ptr(w16),
        _ptr(np.ascontiguousarray(pk["fp16_tile_ids"], np.int32)),
        _ptr(np.ascontiguousarray(pk["fp16_row_ptr"], np.int32)),
        _ptr(out), M, odtype, _ptr(bias), n, M, K, pk["n_tr"], pk["n_tc"], int(split_k),
        1 if use_fma else 0, _ptr(parts), _ptr(acc))
    extra = ([parts] if want_partials else []) + ([acc] if want_f32 else [])
    return tuple([out] + extra) if extra else out


def peer_sum(partials_f32, odtype: int = BF16, bias_bits=None) -> np.ndarray:
    """Row-parallel sum of the ranks' FP32 partial outputs, as the decode kernel's peer
    sum forms it: added in rank order 0..world-1 in FP32, rounded to ``odtype``, then
    the bias added the way the GEMM adds it.  (No counterpart in the reference, which
    runs on one GPU.)"""
    total = np.array(partials_f32[0], dtype=np.float32, copy=True)
    for p in partials_f32[1:]:
        total = (total + np.asarray(p, np.float32)).astype(np.float32)
    out = _round16(total, odtype)
    if bias_bits is not None:
        b = h_to_f32(np.asarray(bias_bits, np.uint16), odtype)[None, :]
        out = _round16((h_to_f32(out, odtype) + b).astype(np.float32), odtype)
    return out


def _round16(x: np.ndarray, dtype: int) -> np.ndarray:
    """f32 -> 16-bit bits, round to nearest even."""
    if dtype == BF16:
        return f32_to_bf16_bits(x)
    return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint16)


# ------------------------------------------------------------------- calibration

def gi_accumulate(tile_scores: np.ndarray, w_bits: np.ndarray, g_bits: np.ndarray, dtype: int = BF16):
    w_bits = np.ascontiguousarray(_h16(w_bits))
    g_bits = np.ascontiguousarray(_h16(g_bits))
    m, k = w_bits.shape
    n_tr, n_tc = tile_scores.shape
    lib().tqo_calib_gi_accumulate(_ptr(w_bits), _ptr(g_bits), dtype, m, k, n_tr, n_tc, _ptr(tile_scores))
    return tile_scores


def iaa_channel_accumulate(act_sum: np.ndarray, x_bits: np.ndarray, dtype: int = BF16):
    x_bits = np.ascontiguousarray(_h16(x_bits)).reshape(-1, x_bits.shape[-1])
    lib().tqo_iaa_channel_accumulate(_ptr(x_bits), dtype, x_bits.shape[0], x_bits.shape[1], _ptr(act_sum))
    return act_sum


def iaa_tile_scores(w_bits: np.ndarray, act_sum: np.ndarray, count: int, dtype: int = BF16):
    w_bits = np.ascontiguousarray(_h16(w_bits))
    m, k = w_bits.shape
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    mean = np.empty((k,), np.float32)
    scores = np.empty((n_tr, n_tc), np.float32)
    lib().tqo_iaa_tile_scores(_ptr(w_bits), dtype, m, k, n_tr, n_tc,
                              _ptr(np.ascontiguousarray(act_sum, np.float64)), int(count), _ptr(mean), _ptr(scores))
    return mean, scores


def topk_mask(importance: np.ndarray, keep_frac: float) -> np.ndarray:
    """Keep mask of the ceil(keep_frac * T) largest scores (decisions.py:174-183).

    Ties at the k-th value are broken towards the larger flat index (the set is
    otherwise the reference's argpartition selection)."""
    values = np.asarray(importance).reshape(-1)
    k = max(1, int(math.ceil(float(keep_frac) * int(values.size))))
    mask = np.zeros_like(values, dtype=np.uint8)
    if k >= values.size:
        mask[:] = 1
    else:
        mask[np.argsort(values, kind="stable")[-k:]] = 1
    return mask.reshape(np.asarray(importance).shape)
