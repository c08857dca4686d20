"""GPU parity of the stream decode kernel (TQ_ALGO_STREAM, csrc/gemm_stream.cu): up to
16 activation rows, one CTA per (split, row tile), splits reduced in a cluster.

Without 16-bit tiles it reproduces the reference arithmetic exactly (the oracle run at
the same split with a separate multiply and add per INT8 tile); with 16-bit tiles and
bias it is bit-identical to the split-K row kernel at the same split (same partition,
same order); the automatic choice for <= 16 rows is this kernel at select_split_k's
split, and where it cannot take a call the row kernel at that split gives the same bits.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import tilequant_b200 as tq
from tilequant_b200 import _native as N
from oracle import oracle as O
from tests.golden import inputs as I
from tests.helpers import from_torch16

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _cfg():
    return SimpleNamespace(tile_m=64, tile_n=64, pad_to_tile=True, quant_style="gi")


def _pack(w, n_tr, n_tc, keep, seed):
    fp16 = I.keep_ids(n_tr, n_tc, keep, seed) if keep else torch.zeros(0, dtype=torch.int32)
    return tq.pack_weight_from_tile_ids(w.to(DEV), n_tr=n_tr, n_tc=n_tc,
                                        int8_tile_ids=I.complement_ids(fp16, n_tr * n_tc), fp16_tile_ids=fp16,
                                        cfg=_cfg()), fp16


def _kw(p, m, k, split, bias=None, dtype=torch.bfloat16):
    return dict(int8_tiles=p.int8_tiles, int8_scales=p.int8_scales, int8_tile_ids=p.int8_tile_ids,
                int8_row_ptr=p.int8_row_ptr, fp16_tiles=p.fp16_tiles, fp16_tile_ids=p.fp16_tile_ids,
                fp16_row_ptr=p.fp16_row_ptr, M=m, K=k, n_tr=p.n_tr, n_tc=p.n_tc, out_dtype=dtype, bias=bias,
                split_k=split)


@pytest.mark.parametrize("rows,m,k,split", [(1, 64, 64, 1), (7, 200, 320, 3), (16, 3072, 3072, 3),
                                            (9, 1000, 4160, 8), (4, 16384, 3072, 1), (16, 192, 8192, 2),
                                            (3, 128, 128, 8)])
def test_stream_int8_only_bit_exact_vs_oracle(cuda_device, rows, m, k, split):
    x = I.activations(rows, k, 700 + rows, outliers=2)
    w = I.weight(m, k, 701 + m)
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    p, _ = _pack(w, n_tr, n_tc, 0.0, 0)
    xd = x.to(DEV)
    q, sx = tq.quantize_activation_tile_absmax(xd)
    y = tq.gemm_mixed_rows_splitk(x_fp=xd, x_int8=q, sx=sx, algo=N.TQ_ALGO_STREAM, **_kw(p, m, k, split))
    qo, sxo = O.quantize_act(I.bits(x))
    pk = O.pack(I.bits(w), n_tr, n_tc, np.arange(n_tr * n_tc), np.arange(0))
    ref = O.gemm(qo, sxo, pk, I.bits(x), m, k, split_k=split, use_fma=False)
    np.testing.assert_array_equal(from_torch16(y), ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,m,k,keep,split", [(16, 3072, 3072, 0.01, None), (5, 320, 384, 0.1, 4),
                                                 (16, 448, 8256, 0.3, 8), (1, 64, 192, 1.0, 2),
                                                 (4, 5120, 3072, 0.05, None), (12, 640, 1024, 0.1, 1)])
def test_stream_identical_to_row_kernel(cuda_device, dtype, rows, m, k, keep, split):
    """Same partition, same order: bit-identical to the row kernel with 16-bit tiles and
    bias, in both 16-bit types."""
    x = I.activations(rows, k, 710 + rows, outliers=2).to(DEV).to(dtype)
    w = I.weight(m, k, 711).to(dtype)
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    p, _ = _pack(w, n_tr, n_tc, keep, 712)
    b = I.weight(1, m, 713, std=0.3).reshape(-1).to(DEV).to(dtype)
    if split is None:
        split = tq.select_split_k(n_tr=n_tr, n_tc=n_tc, n_rows=rows, device=torch.device(DEV), dtype=dtype)
    q, sx = tq.quantize_activation_tile_absmax(x)
    kw = _kw(p, m, k, split, b, dtype)
    want = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, algo=N.TQ_ALGO_ROWS, **kw)
    got = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, algo=N.TQ_ALGO_STREAM, **kw)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("rows,m,k", [(4, 3072, 3072), (8, 16384, 3072), (1, 3072, 8192)])
def test_auto_is_stream_at_the_planned_split(cuda_device, rows, m, k):
    """Up to 8 rows the automatic choice is this kernel at select_split_k's split."""
    x = I.activations(rows, k, 720 + rows, outliers=2).to(DEV)
    w = I.weight(m, k, 721)
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    p, _ = _pack(w, n_tr, n_tc, 0.01, 722)
    split = tq.select_split_k(n_tr=n_tr, n_tc=n_tc, n_rows=rows, device=torch.device(DEV))
    q, sx = tq.quantize_activation_tile_absmax(x)
    auto = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, **_kw(p, m, k, None))
    stream = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, algo=N.TQ_ALGO_STREAM, **_kw(p, m, k, split))
    assert torch.equal(auto.view(torch.int16), stream.view(torch.int16))


def test_auto_falls_back_to_row_kernel_at_the_same_split(cuda_device):
    """A K that is not a multiple of 16 (activation rows the bulk copy cannot take): the
    automatic choice runs the row kernel at the stream kernel's split."""
    rows, m, k = 5, 640, 1000
    x = I.activations(rows, k, 730, outliers=2).to(DEV)
    w = I.weight(m, k, 731)
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    p, _ = _pack(w, n_tr, n_tc, 0.1, 732)
    split = tq.select_split_k(n_tr=n_tr, n_tc=n_tc, n_rows=rows, device=torch.device(DEV))
    q, sx = tq.quantize_activation_tile_absmax(x)
    with pytest.raises(N.TileQuantError):
        tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, algo=N.TQ_ALGO_STREAM, **_kw(p, m, k, split))
    auto = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, **_kw(p, m, k, None))
    rows_y = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, algo=N.TQ_ALGO_ROWS, **_kw(p, m, k, split))
    assert torch.equal(auto.view(torch.int16), rows_y.view(torch.int16))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,m,k,keep", [(4, 3072, 3072, 0.01), (16, 640, 1024, 0.1), (1, 5120, 3072, 0.0),
                                           (9, 3072, 8192, 0.05), (16, 192, 4160, 0.3)])
def test_fused_quant_stream_identical_to_two_steps(cuda_device, dtype, rows, m, k, keep):
    """The quantizer inside the GEMM launch (the stream kernel up to 8 rows, the row kernel
    beyond): the same bits as quantize + GEMM at the same split."""
    x = (I.activations(rows, k, 740 + rows, outliers=3).to(DEV) * 3).to(dtype)
    w = I.weight(m, k, 741).to(dtype)
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    p, _ = _pack(w, n_tr, n_tc, keep, 742)
    b = I.weight(1, m, 743, std=0.3).reshape(-1).to(DEV).to(dtype)
    split = tq.select_split_k(n_tr=n_tr, n_tc=n_tc, n_rows=rows, device=torch.device(DEV), dtype=dtype, fused=True)
    kw = _kw(p, m, k, split, b, dtype)
    q, sx = tq.quantize_activation_tile_absmax(x)
    two = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, **kw)
    one = tq.gemm_mixed_fused_quant(x_fp=x, **kw)
    assert torch.equal(one.view(torch.int16), two.view(torch.int16))
