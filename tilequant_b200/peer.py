"""Row-parallel peer sum: the decode GEMM of a K-split projection adds the ranks'
partial outputs itself, over NVLink, in place of a separate all-reduce.

No counterpart in the reference, which runs on one GPU.  A tensor-parallel O or down
projection (``parallel.py``) gives each rank a slice of the input columns, so each
rank's GEMM yields a partial output that has to be summed over the ranks.  With a
``PeerExchange`` the decode kernel (1..64 activation rows) writes its FP32 partial
tiles straight into every rank's exchange buffer, waits for the other ranks' tiles of
the same output block (bounded by ``timeout_s``; a timeout sets an error word, it
never hangs), and sums them in rank order before rounding: every rank ends up with
the same output, summed in FP32 from unrounded partials (a BF16 all-reduce sums
partials already rounded to BF16).

One process per GPU: each rank allocates its buffer on its own GPU, the 64-byte CUDA
IPC handles are exchanged through ``torch.distributed`` (``connect``), and each rank
maps every peer's buffer.  ``connect_local`` wires buffers of one process instead
(world 1, and the timeout test, where the "peer" is a buffer that nobody writes).
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import torch

from . import _native as N
from .gemm import _check_common

DEFAULT_SLOTS = 1024  # decode CTAs of one call: 4 per 64-row output tile (M <= 16384)


class PeerExchange:
    """Exchange buffer of one rank plus the mappings of its peers' buffers."""

    def __init__(self, device, world: int, rank: int, slots: int = DEFAULT_SLOTS, timeout_s: float = 2.0):
        if not 1 <= int(world) <= N.TQ_PEER_MAX_WORLD or not 0 <= int(rank) < int(world):
            raise ValueError(f"need 1 <= world <= {N.TQ_PEER_MAX_WORLD} and 0 <= rank < world")
        if not 1 <= int(slots) <= N.TQ_PEER_MAX_SLOTS:
            raise ValueError(f"slots must be in 1..{N.TQ_PEER_MAX_SLOTS}")
        if not timeout_s > 0:
            raise ValueError("timeout_s must be positive")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("the peer sum needs a CUDA device (there is no CPU path)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.world, self.rank, self.slots = int(world), int(rank), int(slots)
        self.timeout_ns = int(timeout_s * 1e9)
        lib = N.load()
        buf = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            N.check(lib.tq_peer_alloc(self.world, self.slots, ctypes.byref(buf)), "PeerExchange")
        self._own: Optional[int] = buf.value
        self._opened: List[int] = []
        self._connected = False  # mapped across processes by connect()
        self._group = None
        self.epochs = torch.zeros(self.slots, dtype=torch.int32, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.bufs: Optional[torch.Tensor] = None  # int64 [world] device pointers, own at index rank

    @property
    def buffer_ptr(self) -> int:
        return int(self._own)

    def ipc_handle(self) -> bytes:
        h = ctypes.create_string_buffer(N.TQ_IPC_HANDLE_BYTES)
        with torch.cuda.device(self.device):
            N.check(N.load().tq_peer_ipc_handle(ctypes.c_void_p(self._own), h), "PeerExchange.ipc_handle")
        return h.raw

    def _set_bufs(self, ptrs: Sequence[int]) -> None:
        self.bufs = torch.tensor([int(p) for p in ptrs], dtype=torch.int64, device=self.device)

    def connect(self, group=None) -> "PeerExchange":
        """Exchange IPC handles with the other ranks of ``group`` (collective; with the
        NCCL backend, call it with this rank's device current) and map their buffers."""
        import torch.distributed as dist

        if dist.get_world_size(group) != self.world or dist.get_rank(group) != self.rank:
            raise ValueError("process group does not match the exchange's world / rank")
        handles: List[Optional[bytes]] = [None] * self.world
        dist.all_gather_object(handles, self.ipc_handle(), group=group)
        ptrs = []
        lib = N.load()
        with torch.cuda.device(self.device):
            for p, h in enumerate(handles):
                if p == self.rank:
                    ptrs.append(self._own)
                    continue
                out = ctypes.c_void_p()
                N.check(lib.tq_peer_ipc_open(ctypes.create_string_buffer(h, N.TQ_IPC_HANDLE_BYTES),
                                             ctypes.byref(out)), "PeerExchange.connect")
                self._opened.append(out.value)
                ptrs.append(out.value)
        self._set_bufs(ptrs)
        self._group = group
        self._connected = True
        dist.barrier(group=group)
        return self

    def connect_local(self, peers: Sequence["PeerExchange"] = ()) -> "PeerExchange":
        """Use buffers of this process as the peers' (``peers`` in rank order without
        this one).  For world 1, and for tests on one GPU."""
        if len(peers) != self.world - 1:
            raise ValueError("connect_local needs world - 1 peer exchanges")
        others = iter(peers)
        self._set_bufs([self._own if p == self.rank else next(others).buffer_ptr for p in range(self.world)])
        return self

    def status(self) -> int:
        """TQ_OK, or TQ_ERR_TIMEOUT once a wait for a peer ran out (synchronizes)."""
        return int(self.err.item())

    def reset(self) -> None:
        """Zero this rank's buffer, counters and error word (stream-ordered).  Every rank
        resets, then synchronizes with the others, before the next peer-sum call."""
        N.check(N.load().tq_peer_reset(ctypes.c_void_p(self._own), self.world, self.slots, self.epochs.data_ptr(),
                                       N.stream_of(self.epochs)), "PeerExchange.reset")
        self.err.zero_()

    def close(self) -> None:
        """Unmap the peers' buffers and free this one.  Call on every rank, once no rank
        has peer-sum work in flight; after ``connect`` it is collective: every rank
        unmaps, then all wait for each other before any buffer is freed."""
        lib = N.load()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for p in self._opened:
                lib.tq_peer_ipc_close(ctypes.c_void_p(p))
            self._opened = []
            if self._connected:
                import torch.distributed as dist

                dist.barrier(group=self._group)  # no rank still maps this buffer
                self._connected = False
            if self._own is not None:
                lib.tq_peer_free(ctypes.c_void_p(self._own))
                self._own = None
        self.bufs = None


def gemm_mixed_peer_sum(
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
    exchange: PeerExchange,
    bias: Optional[torch.Tensor] = None,
    split_k: Optional[int] = None,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """``gemm_mixed_rows_splitk`` on this rank's K slice, summed over the exchange's
    ranks inside the kernel (rank order, FP32), then rounded and ``bias`` added: the
    same (N, M) result on every rank.  1..64 rows; every rank makes the same calls."""
    device = N.require_cuda(x_fp, x_int8, sx, int8_tiles, fp16_tiles, out, bias)
    if exchange.bufs is None:
        raise ValueError("the exchange is not connected")
    if exchange.device != device:
        raise ValueError(f"exchange on {exchange.device}, operands on {device}")
    n = int(x_fp.shape[0])
    _check_common(int8_tiles, int8_scales, int8_tile_ids, int8_row_ptr, fp16_tiles, fp16_tile_ids, fp16_row_ptr,
                  M, K, n_tr, n_tc)
    if x_fp.dim() != 2 or x_fp.shape[1] != int(K) or x_fp.stride(1) != 1:
        raise ValueError("x_fp must be (N, K) with unit column stride")
    if x_int8.dtype != torch.int8 or tuple(x_int8.shape) != (n, int(K)) or x_int8.stride(1) != 1:
        raise ValueError("x_int8 must be int8 (N, K) with unit column stride")
    if sx.dtype != torch.float32 or sx.numel() != int(n_tc) or not sx.is_contiguous():
        raise ValueError("sx must be contiguous float32 [n_tc]")
    if out is None:
        out = torch.empty((n, int(M)), device=device, dtype=out_dtype)
    elif tuple(out.shape) != (n, int(M)) or out.dtype != out_dtype or out.stride(1) != 1:
        raise ValueError("out must be an (N, M) tensor of out_dtype with unit column stride")
    if bias is not None and (bias.dtype != out_dtype or not bias.is_contiguous() or bias.numel() != int(M)):
        raise ValueError("bias must be a contiguous [M] tensor of out_dtype")
    t8, t16 = int(int8_tiles.shape[0]), int(fp16_tiles.shape[0])
    rc = N.load().tq_gemm_mixed_peer_sum(
        x_int8.data_ptr(), x_int8.stride(0), sx.data_ptr(), int8_tiles.data_ptr(), int8_scales.data_ptr(),
        int8_tile_ids.data_ptr(), int8_row_ptr.data_ptr(), t8, x_fp.data_ptr(), x_fp.stride(0),
        fp16_tiles.data_ptr() if t16 else None, fp16_tile_ids.data_ptr() if t16 else None,
        fp16_row_ptr.data_ptr() if t16 else None, t16, N.dtype_code(x_fp.dtype), out.data_ptr(), out.stride(0),
        N.dtype_code(out_dtype), N.ptr(bias), n, int(M), int(K), int(n_tr), int(n_tc),
        0 if split_k is None else int(split_k), exchange.bufs.data_ptr(), exchange.epochs.data_ptr(),
        exchange.world, exchange.rank, exchange.slots, exchange.timeout_ns, exchange.err.data_ptr(),
        torch.cuda.current_stream(device).cuda_stream)
    N.check(rc, "gemm_mixed_peer_sum")
    return out
