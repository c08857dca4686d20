"""ctypes binding of the C ABI in ``include/tilequant_b200.h``.

The library is ``libtilequant_b200.so`` next to this file (built by
``python -m tilequant_b200.build``).  There is no fallback: if the library is
missing, or the tensors are not on a CUDA device, the calls raise.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libtilequant_b200.so"

TQ_OK, TQ_ERR_INVALID, TQ_ERR_UNSUPPORTED, TQ_ERR_CUDA, TQ_ERR_TIMEOUT = range(5)
TQ_DTYPE_BF16, TQ_DTYPE_F16 = 0, 1
TQ_ALGO_AUTO, TQ_ALGO_ROWS, TQ_ALGO_UMMA, TQ_ALGO_GEMV, TQ_ALGO_STREAM = 0, 1, 2, 3, 4
ABI_VERSION = 1

_P, _I64, _I, _F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float


class AttnArgs(ctypes.Structure):
    """``tq_attn_args`` of the header, field for field."""

    _fields_ = [(name, _P) for name in ("q", "k", "v", "cos", "sin", "k_cache", "v_cache", "pos", "ws_m", "ws_l",
                                        "ws_o", "err")] + \
               [(name, _I64) for name in ("ld_q", "ld_k", "ld_v")] + \
               [(name, _I) for name in ("B", "Hq", "Hkv", "D", "L", "S")] + \
               [("scale_log2", ctypes.c_float), ("reserved", _I)]

# name -> argument types, in header order
SIGNATURES = {
    "tq_abi_version": [],
    "tq_last_error": [],
    "tq_status_string": [_I],
    "tq_kernel_launches": [],
    "tq_act_scales": [_P, _I, _I64, _I64, _I64, _I64, _P, _P],
    "tq_quantize_with_scales": [_P, _I, _I64, _I64, _I64, _I64, _P, _P, _I64, _P],
    "tq_quantize_act": [_P, _I, _I64, _I64, _I64, _I64, _P, _I64, _P, _P],
    "tq_gemm_mixed": [_P, _I64, _P, _P, _P, _P, _P, _I64, _P, _I64, _P, _P, _P, _I64, _I, _P, _I64, _I, _P,
                      _I64, _I64, _I64, _I, _I, _I, _I, _P, _P],
    "tq_gemm_mixed_fused_quant": [_P, _I64, _I, _P, _P, _P, _P, _I64, _P, _P, _P, _I64, _P, _I64, _I, _P, _I64,
                                  _I64, _I64, _I, _I, _I, _P, _P],
    "tq_gemm_rows_plan": [_I64, _I, _I, _I, _I, _P, _P],
    "tq_gemm_int8_partials": [_P, _I64, _P, _P, _P, _I64, _I64, _I64, _I, _I, _P, _I, _P],
    "tq_pack_int8_tiles": [_P, _I, _I64, _I64, _I64, _I, _P, _I64, _P, _P, _P, _P],
    "tq_gather_fp_tiles": [_P, _I, _I64, _I64, _I64, _I, _P, _I64, _P, _P],
    "tq_add_rmsnorm": [_P, _I64, _P, _I64, _P, _P, _I64, _P, _I64, _I64, _I64, _F, _I, _P],
    "tq_silu_mul_quant": [_P, _P, _I64, _I64, _I64, _P, _I64, _P, _I64, _P, _I, _P],
    "tq_attn_decode_splits": [_I, _I, _I],
    "tq_attn_decode": [ctypes.POINTER(AttnArgs), _P, _I64, _P, _I64, _P, _I, _P],
    "tq_greedy_pick": [_P, _I64, _I64, _I64, _I, _P, _P, _P, _P, _I64, _I64, _P, _I64, _P],
    "tq_calib_gi_accumulate": [_P, _P, _I, _I64, _I64, _I64, _I64, _I, _I, _P, _P],
    "tq_calib_iaa_channel_accumulate": [_P, _I, _I64, _I64, _I64, _P, _P],
    "tq_calib_iaa_tile_scores": [_P, _I, _I64, _I64, _I64, _P, _I64, _P, _P, _P],
    "tq_peer_buffer_bytes": [_I, _I],
    "tq_peer_alloc": [_I, _I, _P],
    "tq_peer_free": [_P],
    "tq_peer_ipc_handle": [_P, _P],
    "tq_peer_ipc_open": [_P, _P],
    "tq_peer_ipc_close": [_P],
    "tq_peer_reset": [_P, _I, _I, _P, _P],
    "tq_gemm_mixed_peer_sum": [_P, _I64, _P, _P, _P, _P, _P, _I64, _P, _I64, _P, _P, _P, _I64, _I, _P, _I64, _I, _P,
                               _I64, _I64, _I64, _I, _I, _I, _P, _P, _I, _I, _I, _I64, _P, _P],
    "tq_gemm_mixed_peer_sum_noalloc": [_P, _I64, _P, _P, _P, _P, _P, _I64, _P, _I64, _P, _P, _P, _I64, _I, _P, _I64,
                                       _I, _P, _I64, _I64, _I64, _I, _I, _I, _I64, _I, _P, _P],
}

TQ_PEER_MAX_WORLD, TQ_PEER_MAX_SLOTS, TQ_IPC_HANDLE_BYTES = 8, 65536, 64

_lib = None
_lock = threading.Lock()


class TileQuantError(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load the native library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise TileQuantError(
                    f"native library {LIB_PATH} is missing: build it with `python -m tilequant_b200.build`"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, argtypes in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = _I
            lib.tq_last_error.restype = ctypes.c_char_p
            lib.tq_status_string.restype = ctypes.c_char_p
            lib.tq_kernel_launches.restype = ctypes.c_int64
            lib.tq_peer_buffer_bytes.restype = ctypes.c_int64
            if lib.tq_abi_version() != ABI_VERSION:
                raise TileQuantError("libtilequant_b200.so ABI version mismatch; rebuild it")
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    """Map a C status to the exception the reference raises for the same problem."""
    if rc == TQ_OK:
        return
    msg = load().tq_last_error().decode(errors="replace")
    if rc == TQ_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    raise TileQuantError(f"{what}: {load().tq_status_string(rc).decode()}: {msg}")


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return TQ_DTYPE_BF16
    if dtype == torch.float16:
        return TQ_DTYPE_F16
    raise ValueError(f"unsupported 16-bit float dtype {dtype}; expected bfloat16 or float16")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("tilequant_b200 kernels need CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def kernel_launches() -> int:
    """Kernels this library has launched in the process so far."""
    return int(load().tq_kernel_launches())
