"""Row-parallel peer sum on one GPU.

* world 1: the peer-sum form of the decode kernel (partial written to the exchange
  with its call number, waited for, summed) gives the same bits as the decode kernel, over
  consecutive calls (both call-parity buffers) and CUDA-graph replays;
* a wait that nothing will satisfy -- world 2 where the second "rank" is a buffer no
  kernel ever writes -- ends at the timeout with TQ_ERR_TIMEOUT in the error word and
  a usable context; reset clears it;
* grids that cannot be resident at once and too few slots are rejected on the host.

The two-rank exchange over NVLink is covered by test_gpu_tensor_parallel.py (2 GPUs).
"""

from __future__ import annotations

import time
from types import SimpleNamespace

import pytest
import torch

import tilequant_b200 as tq
from tilequant_b200 import _native as N
from tilequant_b200.peer import PeerExchange, gemm_mixed_peer_sum
from tests.golden import inputs as I

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _pack(m, k, keep, seed):
    w = I.weight(m, k, seed).to(DEV)
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    fp16 = I.keep_ids(n_tr, n_tc, keep, seed + 1)
    cfg = SimpleNamespace(tile_m=64, tile_n=64, pad_to_tile=True, quant_style="gi")
    return tq.pack_weight_from_tile_ids(w, n_tr=n_tr, n_tc=n_tc, int8_tile_ids=I.complement_ids(fp16, n_tr * n_tc),
                                        fp16_tile_ids=fp16, cfg=cfg)


def _weights(p):
    return dict(int8_tiles=p.int8_tiles, int8_scales=p.int8_scales, int8_tile_ids=p.int8_tile_ids,
                int8_row_ptr=p.int8_row_ptr, fp16_tiles=p.fp16_tiles, fp16_tile_ids=p.fp16_tile_ids,
                fp16_row_ptr=p.fp16_row_ptr, M=p.M_orig, K=p.K_orig, n_tr=p.n_tr, n_tc=p.n_tc)


@pytest.mark.parametrize("rows,m,k,keep,use_bias", [(1, 512, 1024, 0.05, False), (5, 1000, 4160, 0.2, True),
                                                   (16, 3072, 3072, 0.01, True)])
def test_world1_peer_sum_matches_decode_kernel(cuda_device, rows, m, k, keep, use_bias):
    p = _pack(m, k, keep, 11)
    ex = PeerExchange(DEV, world=1, rank=0).connect_local()
    bias = (torch.randn(m, generator=I.gen(3)) * 0.5).to(DEV, torch.bfloat16) if use_bias else None
    try:
        for call in range(3):  # both parities of the exchange, then the first again
            x = I.activations(rows, k, 20 + call).to(DEV)
            q, sx = tq.quantize_activation_tile_absmax(x)
            want = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, out_dtype=torch.bfloat16, bias=bias,
                                             algo=N.TQ_ALGO_GEMV, **_weights(p))
            got = gemm_mixed_peer_sum(x_fp=x, x_int8=q, sx=sx, out_dtype=torch.bfloat16, bias=bias, exchange=ex,
                                      **_weights(p))
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int16), want.view(torch.int16)), call
        assert ex.status() == N.TQ_OK
        assert int(ex.epochs[0].item()) == 3
    finally:
        ex.close()


def test_world1_peer_sum_in_cuda_graph(cuda_device):
    rows, m, k = 8, 1536, 2048
    p = _pack(m, k, 0.05, 12)
    ex = PeerExchange(DEV, world=1, rank=0).connect_local()
    x = I.activations(rows, k, 30).to(DEV)
    q, sx = tq.quantize_activation_tile_absmax(x)
    out = torch.empty(rows, m, device=DEV, dtype=torch.bfloat16)
    want = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, out_dtype=torch.bfloat16, algo=N.TQ_ALGO_GEMV,
                                     **_weights(p))
    try:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):  # warm-up outside the capture
            gemm_mixed_peer_sum(x_fp=x, x_int8=q, sx=sx, out_dtype=torch.bfloat16, exchange=ex, out=out,
                                **_weights(p))
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            gemm_mixed_peer_sum(x_fp=x, x_int8=q, sx=sx, out_dtype=torch.bfloat16, exchange=ex, out=out,
                                **_weights(p))
        for _ in range(3):
            out.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out.view(torch.int16), want.view(torch.int16))
        assert ex.status() == N.TQ_OK
        del g
    finally:
        ex.close()


def test_missing_peer_times_out_with_status(cuda_device):
    rows, m, k = 4, 256, 512
    p = _pack(m, k, 0.0, 13)
    x = I.activations(rows, k, 31).to(DEV)
    q, sx = tq.quantize_activation_tile_absmax(x)
    me = PeerExchange(DEV, world=2, rank=0, timeout_s=0.2)
    silent = PeerExchange(DEV, world=2, rank=1)  # stands for a rank that never calls
    me.connect_local([silent])
    try:
        t0 = time.time()
        gemm_mixed_peer_sum(x_fp=x, x_int8=q, sx=sx, out_dtype=torch.bfloat16, exchange=me, **_weights(p))
        torch.cuda.synchronize()
        elapsed = time.time() - t0
        assert me.status() == N.TQ_ERR_TIMEOUT
        assert 0.15 < elapsed < 30.0
        me.reset()
        assert me.status() == N.TQ_OK and int(me.epochs.abs().sum().item()) == 0
        # the context is still usable
        y = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, out_dtype=torch.bfloat16, **_weights(p))
        torch.cuda.synchronize()
        assert torch.isfinite(y.float()).all()
    finally:
        me.close()
        silent.close()


@pytest.mark.parametrize("rows", [17, 40, 64])
def test_world1_peer_sum_row_blocks_match_row_kernel(cuda_device, rows):
    """17..64 rows run as 16-row blocks; at the same split the sums are the split-K row
    kernel's, bit for bit."""
    m, k = 1536, 2048
    p = _pack(m, k, 0.05, 15)
    ex = PeerExchange(DEV, world=1, rank=0).connect_local()
    bias = (torch.randn(m, generator=I.gen(4)) * 0.5).to(DEV, torch.bfloat16)
    try:
        for call in range(2):
            x = I.activations(rows, k, 40 + call).to(DEV)
            q, sx = tq.quantize_activation_tile_absmax(x)
            want = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, out_dtype=torch.bfloat16, bias=bias,
                                             split_k=4, algo=N.TQ_ALGO_ROWS, **_weights(p))
            got = gemm_mixed_peer_sum(x_fp=x, x_int8=q, sx=sx, out_dtype=torch.bfloat16, bias=bias, split_k=4,
                                      exchange=ex, **_weights(p))
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int16), want.view(torch.int16)), call
        assert ex.status() == N.TQ_OK
    finally:
        ex.close()


def test_peer_sum_host_side_rejections(cuda_device):
    x = I.activations(65, 512, 32).to(DEV)
    q, sx = tq.quantize_activation_tile_absmax(x)
    p = _pack(256, 512, 0.0, 14)
    ex = PeerExchange(DEV, world=1, rank=0).connect_local()
    try:
        with pytest.raises(N.TileQuantError):  # more than 64 rows: not a decode call
            gemm_mixed_peer_sum(x_fp=x, x_int8=q, sx=sx, out_dtype=torch.bfloat16, exchange=ex, **_weights(p))
    finally:
        ex.close()
    small = PeerExchange(DEV, world=1, rank=0, slots=8).connect_local()
    try:
        with pytest.raises(ValueError):  # 4 * n_tr = 16 CTAs > 8 slots
            gemm_mixed_peer_sum(x_fp=x[:4], x_int8=q[:4], sx=sx, out_dtype=torch.bfloat16, exchange=small,
                                **_weights(p))
    finally:
        small.close()
    with pytest.raises(ValueError):
        PeerExchange(DEV, world=9, rank=0)
    with pytest.raises(ValueError):
        PeerExchange(DEV, world=2, rank=2)

