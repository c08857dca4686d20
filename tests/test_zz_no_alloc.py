"""The peer-sum decode GEMM entry point that allocates nothing.

Some callers cannot call cudaMalloc: serving runtimes that hand all free device
memory to their own pools at start-up, and real-time host loops that cannot take the
device synchronization an allocation may cause.  ``tq_gemm_mixed_peer_sum_noalloc``
keeps its scratch (exchange words, call counters, address table) in a static device
array instead of a cudaMalloc'd exchange buffer, for a world of one GPU.  These tests
call it through the C ABI and compare it with the allocating entry points on two calls
in a row (the array keeps its state between calls, so the second call runs on the other
call-parity half of it), then after a reset, and check the size limit.

This file is collected last on purpose: the array is shared by every call in the
process, and nothing else here uses it.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

import tilequant_b200 as tq
from tilequant_b200 import _native as N
from tilequant_b200.peer import PeerExchange, gemm_mixed_peer_sum
from tests.golden import inputs as I

pytestmark = pytest.mark.gpu
TIMEOUT_NS = 2_000_000_000


def _pack(w, keep):
    m, k = w.shape
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    cfg = SimpleNamespace(tile_m=64, tile_n=64, pad_to_tile=True, quant_style="gi")
    return tq.pack_weight_from_tile_ids(w, n_tr=n_tr, n_tc=n_tc, int8_tile_ids=I.complement_ids(keep, n_tr * n_tc),
                                        fp16_tile_ids=keep, cfg=cfg)


def _weights(p):
    return dict(int8_tiles=p.int8_tiles, int8_scales=p.int8_scales, int8_tile_ids=p.int8_tile_ids,
                int8_row_ptr=p.int8_row_ptr, fp16_tiles=p.fp16_tiles, fp16_tile_ids=p.fp16_tile_ids,
                fp16_row_ptr=p.fp16_row_ptr, M=p.M_orig, K=p.K_orig, n_tr=p.n_tr, n_tc=p.n_tc)


def _noalloc(p, x, q, sx, out, bias, err, reset_only=0):
    """One call of the no-alloc entry point through the C ABI (current device)."""
    t8, t16 = int(p.int8_tiles.shape[0]), int(p.fp16_tiles.shape[0])
    return N.load().tq_gemm_mixed_peer_sum_noalloc(
        q.data_ptr(), q.stride(0), sx.data_ptr(), p.int8_tiles.data_ptr(), p.int8_scales.data_ptr(),
        p.int8_tile_ids.data_ptr(), p.int8_row_ptr.data_ptr(), t8, x.data_ptr(), x.stride(0),
        p.fp16_tiles.data_ptr() if t16 else None, p.fp16_tile_ids.data_ptr() if t16 else None,
        p.fp16_row_ptr.data_ptr() if t16 else None, t16, N.TQ_DTYPE_BF16, out.data_ptr(), out.stride(0),
        N.TQ_DTYPE_BF16, N.ptr(bias), x.shape[0], p.M_orig, p.K_orig, p.n_tr, p.n_tc, 0, TIMEOUT_NS, reset_only,
        err.data_ptr(), torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_allocating_entry_points_two_calls(cuda_device):
    dev = cuda_device
    torch.cuda.set_device(dev)
    m, k = 3072, 3072
    w = I.weight(m, k, 60).to(dev)
    p = _pack(w, I.keep_ids(m // 64, k // 64, 0.01, 61))
    bias = (torch.randn(m, generator=I.gen(62)) * 0.5).to(dev, torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ex = PeerExchange(dev, world=1, rank=0).connect_local()
    try:
        for call, rows in enumerate((16, 3, 9)):  # two calls in a row on the same scratch, then a reset
            x = I.activations(rows, k, 63 + call).to(dev)
            q, sx = tq.quantize_activation_tile_absmax(x)
            out = torch.full((rows, m), float("nan"), device=dev, dtype=torch.bfloat16)
            if call == 2:
                assert _noalloc(p, x, q, sx, out, None, err, reset_only=1) == N.TQ_OK
                assert bool(torch.isnan(out.float()).all())  # a reset launches nothing
            rc = _noalloc(p, x, q, sx, out, bias, err)
            assert rc == N.TQ_OK, N.load().tq_last_error()
            want_peer = gemm_mixed_peer_sum(x_fp=x, x_int8=q, sx=sx, out_dtype=torch.bfloat16, bias=bias,
                                            exchange=ex, **_weights(p))
            want = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, out_dtype=torch.bfloat16, bias=bias,
                                             algo=N.TQ_ALGO_GEMV, **_weights(p))
            torch.cuda.synchronize()
            assert int(err.item()) == N.TQ_OK
            # the same decode kernel and rank order: the same bits
            assert torch.equal(out.view(torch.int16), want_peer.view(torch.int16)), call
            assert torch.equal(out.view(torch.int16), want.view(torch.int16)), call
    finally:
        ex.close()


def test_noalloc_rejects_sizes_beyond_its_array(cuda_device):
    dev = cuda_device
    torch.cuda.set_device(dev)
    m, k = 16448, 64  # 257 row tiles: 1028 CTAs > the array's 1024 slots
    p = _pack(I.weight(m, k, 70).to(dev), torch.zeros(0, dtype=torch.int32))
    x = I.activations(4, k, 71).to(dev)
    q, sx = tq.quantize_activation_tile_absmax(x)
    out = torch.full((4, m), float("nan"), device=dev, dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    assert _noalloc(p, x, q, sx, out, None, err) == N.TQ_ERR_INVALID
    assert b"1024" in N.load().tq_last_error()
    # more than 16 rows is not a decode call
    x = I.activations(17, k, 72).to(dev)
    q, sx = tq.quantize_activation_tile_absmax(x)
    out = torch.empty(17, 1024, device=dev, dtype=torch.bfloat16)
    p = _pack(I.weight(1024, k, 73).to(dev), torch.zeros(0, dtype=torch.int32))
    assert _noalloc(p, x, q, sx, out, None, err) == N.TQ_ERR_UNSUPPORTED
    torch.cuda.synchronize()
    assert int(err.item()) == N.TQ_OK
