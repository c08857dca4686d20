"""GPU parity of the persistent TMA + tcgen05 prefill GEMM (TQ_ALGO_UMMA).

Its INT8 arithmetic is acc = fma(f32(i32 tile dot), sx*sw, acc) in ascending column
order (the FP32 multiply-add Triton's default contraction gives the reference), so
without 16-bit tiles it is bit-exact against the oracle run with use_fma=True; the
INT32 tile products are exact; with 16-bit tiles the output is within 1 BF16 ulp.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import tilequant_b200 as tq
from oracle import oracle as O
from tests.golden import inputs as I
from tests.helpers import assert_close_gemm, assert_close_with_bias, from_torch16, ulp_dist16

pytestmark = pytest.mark.gpu
DEV = "cuda"
UMMA, ROWS = 2, 1


def cfg():
    return SimpleNamespace(tile_m=64, tile_n=64, pad_to_tile=True, quant_style="gi")


def _case(rows, m, k, keep, seed):
    x = I.activations(rows, k, seed, outliers=3)
    w = I.weight(m, k, seed + 1)
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    fp16 = I.keep_ids(n_tr, n_tc, keep, seed + 2)
    int8 = I.complement_ids(fp16, n_tr * n_tc)
    p = tq.pack_weight_from_tile_ids(w.to(DEV), n_tr=n_tr, n_tc=n_tc, int8_tile_ids=int8, fp16_tile_ids=fp16, cfg=cfg())
    pk = O.pack(I.bits(w), n_tr, n_tc, int8.numpy(), fp16.numpy())
    return x, p, pk


def _run(x, p, m, k, bias=None, algo=UMMA):
    xg = x.to(DEV)
    q, sx = tq.quantize_activation_tile_absmax(xg)
    y = tq.gemm_mixed_rows_splitk(x_fp=xg, x_int8=q, sx=sx, int8_tiles=p.int8_tiles, int8_scales=p.int8_scales,
                                  int8_tile_ids=p.int8_tile_ids, int8_row_ptr=p.int8_row_ptr, fp16_tiles=p.fp16_tiles,
                                  fp16_tile_ids=p.fp16_tile_ids, fp16_row_ptr=p.fp16_row_ptr, M=m, K=k, n_tr=p.n_tr,
                                  n_tc=p.n_tc, out_dtype=torch.bfloat16, bias=bias, split_k=1, algo=algo)
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("rows,m,k", [(128, 64, 64), (128, 128, 256), (200, 192, 320), (1024, 512, 1024),
                                      (300, 136, 192)])
def test_umma_int8_only_bit_exact(cuda_device, rows, m, k):
    x, p, pk = _case(rows, m, k, 0.0, 500 + rows)
    y = from_torch16(_run(x, p, m, k))
    q, sx = O.quantize_act(I.bits(x))
    ref = O.gemm(q, sx, pk, I.bits(x), m, k, split_k=1, use_fma=True)
    np.testing.assert_array_equal(y, ref)


@pytest.mark.parametrize("rows,m,k,keep", [(128, 128, 128, 0.25), (333, 320, 384, 0.1), (2048, 1024, 3072, 0.05),
                                           (130, 64, 4096, 0.2)])
def test_umma_mixed_within_one_ulp(cuda_device, rows, m, k, keep):
    x, p, pk = _case(rows, m, k, keep, 600 + rows)
    y = from_torch16(_run(x, p, m, k))
    q, sx = O.quantize_act(I.bits(x))
    ref = O.gemm(q, sx, pk, I.bits(x), m, k, split_k=1, use_fma=True)
    assert_close_gemm(y, ref, f"rows={rows}")
    assert (ulp_dist16(y, ref) == 0).mean() > 0.98


def test_umma_partials_bit_exact(cuda_device):
    x, p, pk = _case(256, 192, 320, 0.1, 700)
    q, sx = tq.quantize_activation_tile_absmax(x.to(DEV))
    parts = tq.gemm_int8_partials(x_int8=q, int8_tiles=p.int8_tiles, int8_tile_ids=p.int8_tile_ids,
                                  int8_row_ptr=p.int8_row_ptr, K=320, n_tr=3, n_tc=5, algo=UMMA)
    _, ref = O.gemm(q.cpu().numpy(), sx.cpu().numpy(), pk, I.bits(x), 192, 320, want_partials=True)
    np.testing.assert_array_equal(parts.cpu().numpy(), ref)


def test_umma_bias_and_ragged_rows(cuda_device):
    """Bias, a partial last row tile (M = 200) and a partial last token block."""
    x, p, pk = _case(333, 200, 256, 0.05, 800)
    bias = I.weight(1, 200, 801, std=0.5).reshape(-1).to(torch.bfloat16)
    y = from_torch16(_run(x, p, 200, 256, bias=bias.to(DEV)))
    q, sx = O.quantize_act(I.bits(x))
    ref = O.gemm(q, sx, pk, I.bits(x), 200, 256, split_k=1, bias_bits=I.bits(bias), use_fma=True)
    assert_close_with_bias(y, ref, I.bits(bias), "umma bias")


def test_auto_picks_tcgen05_for_prefill(cuda_device):
    x, p, pk = _case(512, 256, 512, 0.05, 900)
    assert torch.equal(_run(x, p, 256, 512, algo=0), _run(x, p, 256, 512, algo=UMMA))


# ------------------------------------------------------------------ multi-wave cases
# The kernel is persistent (one CTA per SM, 148 on a B200) and walks output tiles of
# 128 activation rows x 128 output columns; the cases below hold two to seven times as
# many tiles as CTAs, so every CTA reuses its column-table ring slots, its TMEM groups
# and its barrier phases across tiles.

def _tiles(rows, m):
    return ((rows + 127) // 128) * ((m + 127) // 128)


@pytest.mark.parametrize("rows,m,k", [(2048, 2560, 512), (4096, 4096, 256)])
def test_umma_multiwave_int8_only_bit_exact(cuda_device, rows, m, k):
    assert _tiles(rows, m) > 2 * 148
    x, p, pk = _case(rows, m, k, 0.0, 1100 + rows)
    y = from_torch16(_run(x, p, m, k))
    q, sx = O.quantize_act(I.bits(x))
    ref = O.gemm(q, sx, pk, I.bits(x), m, k, split_k=1, use_fma=True)
    np.testing.assert_array_equal(y, ref)


def test_umma_multiwave_ragged_mixed_within_one_ulp(cuda_device):
    """1500 rows (a partial last token block), 2240 = 35 row tiles (an odd count: the
    last output tile has one row tile), 576 = 9 column tiles, 10 % 16-bit tiles."""
    rows, m, k = 1500, 2240, 576
    assert _tiles(rows, m) > 148
    x, p, pk = _case(rows, m, k, 0.1, 1200)
    y = from_torch16(_run(x, p, m, k))
    q, sx = O.quantize_act(I.bits(x))
    ref = O.gemm(q, sx, pk, I.bits(x), m, k, split_k=1, use_fma=True)
    assert_close_gemm(y, ref, "ragged multi-wave")
    assert (ulp_dist16(y, ref) == 0).mean() > 0.98


def test_umma_multiwave_partials_bit_exact(cuda_device):
    rows, m, k = 2048, 2560, 512
    x, p, pk = _case(rows, m, k, 0.1, 1300)
    q, sx = tq.quantize_activation_tile_absmax(x.to(DEV))
    parts = tq.gemm_int8_partials(x_int8=q, int8_tiles=p.int8_tiles, int8_tile_ids=p.int8_tile_ids,
                                  int8_row_ptr=p.int8_row_ptr, K=k, n_tr=p.n_tr, n_tc=p.n_tc, algo=UMMA)
    _, ref = O.gemm(q.cpu().numpy(), sx.cpu().numpy(), pk, I.bits(x), m, k, want_partials=True)
    np.testing.assert_array_equal(parts.cpu().numpy(), ref)


# ------------------------------------------------- the shapes bench.py times (config 2)
# One Llama-3.2-3B block at prefill: 8192 activation rows, 5 % 16-bit tiles.  Output
# rows are independent once the activation scales are fixed, so the oracle checks a
# sample of rows (one in every 128-row token block, at a different lane each time) of
# the full-size launch, with the scales of the whole batch.

CONFIG2 = {"qkv": (5120, 3072), "o": (3072, 3072), "gate_up": (16384, 3072), "down": (3072, 8192)}


def sample_rows(rows: int, seed: int = 0) -> np.ndarray:
    blocks = (rows + 127) // 128
    rng = np.random.default_rng(seed)
    return np.array([min(rows - 1, b * 128 + int(rng.integers(0, 128))) for b in range(blocks)], np.int64)


@pytest.mark.parametrize("name", sorted(CONFIG2))
def test_umma_config2_shapes_sampled_rows(cuda_device, name):
    m, k = CONFIG2[name]
    rows = 8192
    x, p, pk = _case(rows, m, k, 0.05, 1400 + m + k)
    y = _run(x, p, m, k)
    sel = sample_rows(rows, seed=m + k)
    y_s = from_torch16(y[torch.from_numpy(sel).to(DEV)])
    xb = I.bits(x)
    sx = O.act_scales(xb)  # scales of the whole batch
    xs = np.ascontiguousarray(xb[sel])
    q = O.quantize_with_scales(xs, sx)
    ref = O.gemm(q, sx, pk, xs, m, k, split_k=1, use_fma=True)
    assert_close_gemm(y_s, ref, f"{name} {rows}x{m}x{k}")
    assert (ulp_dist16(y_s, ref) == 0).mean() > 0.98
