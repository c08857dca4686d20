"""GPU parity of the sm_100a kernels against the CPU oracle and the reference fixtures.

Bit-exact: activation codes and scales, packed INT8 tiles and scales, INT32 tile
partials, and GEMM outputs whenever the reference arithmetic has no 16-bit tile dot
in it.  GEMM outputs with 16-bit tiles: within 1 BF16 ulp of the oracle (tolerance
of the north star: 1 ulp / rel <= 1e-2), and almost all bit-identical.
"""

from __future__ import annotations

from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import tilequant_b200 as tq
from tilequant_b200 import _native as N
from oracle import oracle as O
from tests.golden import inputs as I
from tests.helpers import assert_close_with_bias, assert_within_ulp, from_torch16, to_torch16

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / "golden"
QUANT = np.load(G / "quant.npz")
PACK = np.load(G / "pack.npz")
GEMM = np.load(G / "gemm.npz")
DEV = "cuda"


def _cases(npz, suffix):
    return sorted({k.split("__")[0] for k in npz.files if k.endswith(suffix)})


def cfg(style="gi", **kw):
    return SimpleNamespace(tile_m=64, tile_n=64, pad_to_tile=True, quant_style=style, **kw)


# ------------------------------------------------------------------- quantizer

@pytest.mark.parametrize("name", _cases(QUANT, "__q"))
def test_quantizer_bit_exact(cuda_device, name):
    dt = torch.bfloat16 if QUANT[f"{name}__dtype"][0] == 0 else torch.float16
    x = to_torch16(QUANT[f"{name}__x"], dt, DEV)
    if QUANT[f"{name}__strided"][0]:
        x = x.t().contiguous().t()
    q, sx = tq.quantize_activation_tile_absmax(x)
    np.testing.assert_array_equal(sx.cpu().numpy().view(np.uint32), QUANT[f"{name}__sx"].view(np.uint32))
    np.testing.assert_array_equal(q.cpu().numpy(), QUANT[f"{name}__q"])
    # the two-pass API agrees
    sx2 = tq.activation_tile_absmax_scales(x)
    q2 = tq.quantize_activation_tile_with_scales(x, sx2)
    assert torch.equal(sx2, sx) and torch.equal(q2, q)


@pytest.mark.parametrize("rows,k", [(1, 64), (129, 3072), (1000, 200), (8192, 3072), (40000, 512)])
def test_quantizer_large_rows_match_oracle(cuda_device, rows, k):
    x = I.activations(rows, k, 100 + rows, outliers=4)
    xg = x.to(DEV)
    q, sx = tq.quantize_activation_tile_absmax(xg)
    q_ref, sx_ref = O.quantize_act(I.bits(x))
    np.testing.assert_array_equal(sx.cpu().numpy(), sx_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)


def test_quantizer_rejects_bad_input(cuda_device):
    with pytest.raises(ValueError):
        tq.quantize_activation_tile_absmax(torch.zeros(4, 64, device=DEV, dtype=torch.float32))
    with pytest.raises(ValueError):
        tq.quantize_activation_tile_with_scales(torch.zeros(4, 128, device=DEV, dtype=torch.bfloat16),
                                                torch.ones(3, device=DEV))
    with pytest.raises(ValueError):
        tq.quantize_activation_tile_absmax(torch.zeros(4, 64, dtype=torch.bfloat16))  # CPU tensor


def test_empty_batch_follows_the_reference(cuda_device):
    """Zero rows: the unfused scales raise as the reference's amax over an empty dimension
    does (quant_utils.py:68-69); the fused quantizer gives no codes and scale 1.0 per tile,
    as the reference's fused kernel reducing over no rows does (quantize_activation.py:
    100-106); codes with given scales, the GEMM and MixedLinear return empty outputs."""
    x = torch.empty((0, 200), device=DEV, dtype=torch.bfloat16)
    with pytest.raises(IndexError):
        tq.activation_tile_absmax_scales(x)
    q, sx = tq.quantize_activation_tile_absmax(x)
    torch.cuda.synchronize()
    assert q.shape == (0, 200) and q.dtype == torch.int8
    assert torch.equal(sx.cpu(), torch.ones(4))
    assert tq.quantize_activation_tile_with_scales(x, sx).shape == (0, 200)
    lin, *_ = _linear(128, 200, 0.1, 5)
    with torch.inference_mode():
        y = lin(x)
        y3 = lin(torch.empty((2, 0, 200), device=DEV, dtype=torch.bfloat16))
    assert y.shape == (0, 128) and y3.shape == (2, 0, 128)


# ---------------------------------------------------------------------- packer

@pytest.mark.parametrize("name", _cases(PACK, "__in_int8_ids"))
def test_packer_bit_exact(cuda_device, name):
    dt = torch.bfloat16 if PACK[f"{name}__wdtype"][0] == 0 else torch.float16
    w = to_torch16(PACK[f"{name}__w"], dt, DEV)
    n_tr, n_tc = (int(v) for v in PACK[f"{name}__grid"])
    style = str(PACK[f"{name}__style"])
    imp = torch.from_numpy(PACK[f"{name}__imp"]).to(DEV) if f"{name}__imp" in PACK.files else None
    p = tq.pack_weight_from_tile_ids(w, n_tr=n_tr, n_tc=n_tc,
                                     int8_tile_ids=torch.from_numpy(PACK[f"{name}__in_int8_ids"]),
                                     fp16_tile_ids=torch.from_numpy(PACK[f"{name}__in_fp16_ids"]),
                                     iaa_col_importance=imp, cfg=cfg(style))
    for key in ("int8_tiles", "int8_tile_ids", "int8_row_ptr", "int8_row_indices", "fp16_tile_ids", "fp16_row_ptr",
                "fp16_row_indices"):
        np.testing.assert_array_equal(getattr(p, key).cpu().numpy(), PACK[f"{name}__{key}"], err_msg=key)
    np.testing.assert_array_equal(p.int8_scales.cpu().numpy().view(np.uint32),
                                  PACK[f"{name}__int8_scales"].view(np.uint32))
    np.testing.assert_array_equal(from_torch16(p.fp16_tiles), PACK[f"{name}__fp16_tiles"])


def test_packer_config1_bit_exact(cuda_device):
    x, w, fp16, int8, n_tr, n_tc = I.config1(0)
    p = tq.pack_weight_from_tile_ids(w.to(DEV), n_tr=n_tr, n_tc=n_tc, int8_tile_ids=int8, fp16_tile_ids=fp16,
                                     cfg=cfg())
    assert I.sha256(p.int8_tiles.cpu().numpy()) == str(PACK["cfg1__int8_tiles_sha"])
    assert I.sha256(from_torch16(p.fp16_tiles)) == str(PACK["cfg1__fp16_tiles_sha"])
    np.testing.assert_array_equal(p.int8_scales.cpu().numpy(), PACK["cfg1__int8_scales"])


def test_packer_iaa_large_matches_oracle(cuda_device):
    w = I.weight(1024, 960, 7, std=0.03)
    imp = torch.rand((960,), generator=I.gen(8)) * 2
    fp16 = I.keep_ids(16, 15, 0.2, 9)
    int8 = I.complement_ids(fp16, 240)
    p = tq.pack_weight_from_tile_ids(w.to(DEV), n_tr=16, n_tc=15, int8_tile_ids=int8, fp16_tile_ids=fp16,
                                     iaa_col_importance=imp.to(DEV), cfg=cfg("iaa"))
    ref = O.pack(I.bits(w), 16, 15, int8.numpy(), fp16.numpy(), O.BF16, imp.numpy())
    np.testing.assert_array_equal(p.int8_scales.cpu().numpy(), ref["int8_scales"])
    np.testing.assert_array_equal(p.int8_tiles.cpu().numpy(), ref["int8_tiles"])


def test_concat_packs_matches_reference(cuda_device):
    parts = []
    for i, m in enumerate((128, 64, 64)):
        w = to_torch16(PACK[f"stack{i}__w"], torch.bfloat16, DEV)
        ids16 = torch.from_numpy(PACK[f"stack{i}__in_fp16_ids"])
        parts.append(tq.pack_weight_from_tile_ids(w, n_tr=m // 64, n_tc=3, int8_tile_ids=I.complement_ids(ids16, m // 64 * 3),
                                                  fp16_tile_ids=ids16, cfg=cfg()))
    st = tq.concat_packs_along_rows(parts)
    for key in ("int8_tiles", "int8_scales", "int8_tile_ids", "int8_row_ptr", "int8_row_indices", "fp16_tile_ids",
                "fp16_row_ptr", "fp16_row_indices"):
        np.testing.assert_array_equal(getattr(st, key).cpu().numpy(), PACK[f"stacked__{key}"], err_msg=key)
    np.testing.assert_array_equal(from_torch16(st.fp16_tiles), PACK["stacked__fp16_tiles"])


def test_packer_rejects_bad_maps(cuda_device):
    w = torch.zeros((128, 128), device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        tq.pack_weight_from_tile_ids(w, n_tr=2, n_tc=3, int8_tile_ids=torch.arange(6), fp16_tile_ids=torch.arange(0),
                                     cfg=cfg())
    with pytest.raises(RuntimeError):
        tq.pack_weight_from_tile_ids(w, n_tr=2, n_tc=2, int8_tile_ids=torch.arange(3), fp16_tile_ids=torch.arange(0),
                                     cfg=cfg())
    with pytest.raises(ValueError):  # repeated id
        tq.pack_weight_from_tile_ids(w, n_tr=2, n_tc=2, int8_tile_ids=torch.tensor([0, 1, 1, 3]),
                                     fp16_tile_ids=torch.arange(0), cfg=cfg())
    with pytest.raises(ValueError):  # out of range
        tq.pack_weight_from_tile_ids(w, n_tr=2, n_tc=2, int8_tile_ids=torch.tensor([0, 1, 2, 9]),
                                     fp16_tile_ids=torch.arange(0), cfg=cfg())


# ------------------------------------------------------------------------ GEMM

def _gemm_case(name):
    x = GEMM[f"{name}__x"]
    M, K = (int(v) for v in GEMM[f"{name}__MK"])
    if name.startswith("cfg1"):
        _, w, fp16, int8, n_tr, n_tc = I.config1(0)
        w_bits, i16, imp, style = I.bits(w), fp16.numpy(), None, "gi"
    else:
        n_tr, n_tc = (int(v) for v in GEMM[f"{name}__grid"])
        w_bits, i16 = GEMM[f"{name}__w"], GEMM[f"{name}__fp16_ids"]
        imp = GEMM[f"{name}__imp"] if f"{name}__imp" in GEMM.files else None
        style = str(GEMM[f"{name}__style"])
    i8 = O.int8_ids_from_keep(i16, n_tr, n_tc)
    p = tq.pack_weight_from_tile_ids(to_torch16(w_bits, torch.bfloat16, DEV), n_tr=n_tr, n_tc=n_tc,
                                     int8_tile_ids=torch.from_numpy(i8), fp16_tile_ids=torch.from_numpy(i16),
                                     iaa_col_importance=None if imp is None else torch.from_numpy(imp).to(DEV),
                                     cfg=cfg(style))
    bias = GEMM[f"{name}__bias"] if f"{name}__bias" in GEMM.files else None
    return x, p, M, K, int(GEMM[f"{name}__split"][0]), bias


def _run_gemm(x_bits, p, M, K, split, bias_bits, fused=False, algo=0):
    x = to_torch16(x_bits, torch.bfloat16, DEV)
    bias = None if bias_bits is None else to_torch16(bias_bits, torch.bfloat16, DEV)
    kw = dict(int8_tiles=p.int8_tiles, int8_scales=p.int8_scales, int8_tile_ids=p.int8_tile_ids,
              int8_row_ptr=p.int8_row_ptr, fp16_tiles=p.fp16_tiles, fp16_tile_ids=p.fp16_tile_ids,
              fp16_row_ptr=p.fp16_row_ptr, M=M, K=K, n_tr=p.n_tr, n_tc=p.n_tc, out_dtype=torch.bfloat16, bias=bias,
              split_k=split)
    if fused:
        return tq.gemm_mixed_fused_quant(x_fp=x, **kw)
    q, sx = tq.quantize_activation_tile_absmax(x)
    return tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, algo=algo, **kw)


@pytest.mark.parametrize("name", _cases(GEMM, "__y"))
def test_gemm_matches_reference(cuda_device, name):
    x, p, M, K, split, bias = _gemm_case(name)
    y = from_torch16(_run_gemm(x, p, M, K, split, bias))
    d = assert_within_ulp(y, GEMM[f"{name}__y"], 1, name)
    assert (d == 0).mean() > 0.99, f"{name}: {(d == 0).mean():.4f} bit-identical"
    torch.cuda.synchronize()


@pytest.mark.parametrize("name", _cases(GEMM, "__y"))
def test_fused_decode_identical_to_two_step(cuda_device, name):
    x, p, M, K, split, bias = _gemm_case(name)
    if x.shape[0] > 64:
        pytest.skip("fused form is for <= 64 rows")
    a = _run_gemm(x, p, M, K, split, bias)
    b = _run_gemm(x, p, M, K, split, bias, fused=True)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def _int8_only_pack(w, n_tr, n_tc):
    return tq.pack_weight_from_tile_ids(w.to(DEV), n_tr=n_tr, n_tc=n_tc, int8_tile_ids=torch.arange(n_tr * n_tc),
                                        fp16_tile_ids=torch.arange(0), cfg=cfg())


@pytest.mark.parametrize("rows,m,k,split", [(1, 64, 64, 1), (16, 3072, 3072, 8), (7, 200, 136, 3), (33, 512, 1024, 16),
                                            (64, 1024, 3072, 4), (130, 256, 512, 2), (300, 192, 320, 1)])
def test_gemm_int8_only_bit_exact_vs_oracle(cuda_device, rows, m, k, split):
    """Without 16-bit tiles the reference arithmetic is fully specified: the split-K
    row kernel (mul then add, as the reference source reads) is bit-exact."""
    x = I.activations(rows, k, 200 + rows, outliers=2)
    w = I.weight(m, k, 201 + m)
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    p = _int8_only_pack(w, n_tr, n_tc)
    y = from_torch16(_run_gemm(I.bits(x), p, m, k, split, None, algo=1))
    q, sx = O.quantize_act(I.bits(x))
    pk = O.pack(I.bits(w), n_tr, n_tc, np.arange(n_tr * n_tc), np.arange(0))
    ref = O.gemm(q, sx, pk, I.bits(x), m, k, split_k=split, use_fma=False)
    np.testing.assert_array_equal(y, ref)


@pytest.mark.parametrize("rows,m,k,split", [(1, 64, 64, 1), (16, 3072, 3072, 8), (7, 200, 136, 3), (16, 512, 1024, 5),
                                            (3, 1000, 4160, 8), (16, 192, 9000, 2)])
def test_decode_kernel_int8_only_bit_exact_vs_oracle(cuda_device, rows, m, k, split):
    """The decode kernel (algo 3) reproduces the reference arithmetic exactly, like the
    split-K row kernel, for ragged and unaligned shapes and for more INT8 tiles per warp
    than it keeps in flight at once."""
    x = I.activations(rows, k, 500 + rows, outliers=2)
    w = I.weight(m, k, 501 + m)
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    p = _int8_only_pack(w, n_tr, n_tc)
    y = from_torch16(_run_gemm(I.bits(x), p, m, k, split, None, algo=N.TQ_ALGO_GEMV))
    q, sx = O.quantize_act(I.bits(x))
    pk = O.pack(I.bits(w), n_tr, n_tc, np.arange(n_tr * n_tc), np.arange(0))
    ref = O.gemm(q, sx, pk, I.bits(x), m, k, split_k=split, use_fma=False)
    np.testing.assert_array_equal(y, ref)


@pytest.mark.parametrize("rows,m,k,keep,split", [(16, 3072, 3072, 0.01, None), (5, 320, 384, 0.1, 4),
                                                 (16, 448, 8250, 0.3, 8), (1, 64, 200, 1.0, 2)])
@pytest.mark.parametrize("fused", [False, True])
def test_decode_kernel_identical_to_row_kernel(cuda_device, rows, m, k, keep, split, fused):
    if fused and split is not None and split > 8:
        pytest.skip("the decode kernel takes up to 8 splits")
    """Decode kernel and split-K row kernel at the same split: the same arithmetic in the
    same order, so bit-identical outputs (with 16-bit tiles, bias, fused quantization)."""
    x = I.activations(rows, k, 510 + rows, outliers=2).to(DEV)
    w = I.weight(m, k, 511)
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    fp16 = I.keep_ids(n_tr, n_tc, keep, 512)
    p = tq.pack_weight_from_tile_ids(w.to(DEV), n_tr=n_tr, n_tc=n_tc, int8_tile_ids=I.complement_ids(fp16, n_tr * n_tc),
                                     fp16_tile_ids=fp16, cfg=cfg())
    b = I.weight(1, m, 513, std=0.3).reshape(-1).to(DEV)
    if split is None:
        split = tq.select_split_k(n_tr=n_tr, n_tc=n_tc, n_rows=rows, device=torch.device(DEV), fused=fused)
    kw = dict(int8_tiles=p.int8_tiles, int8_scales=p.int8_scales, int8_tile_ids=p.int8_tile_ids,
              int8_row_ptr=p.int8_row_ptr, fp16_tiles=p.fp16_tiles, fp16_tile_ids=p.fp16_tile_ids,
              fp16_row_ptr=p.fp16_row_ptr, M=m, K=k, n_tr=n_tr, n_tc=n_tc, out_dtype=torch.bfloat16, bias=b,
              split_k=split)
    q, sx = tq.quantize_activation_tile_absmax(x)
    rows_y = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, algo=N.TQ_ALGO_ROWS, **kw)
    if fused:
        y = tq.gemm_mixed_fused_quant(x_fp=x, **kw)
    else:
        y = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, algo=N.TQ_ALGO_GEMV, **kw)
    assert torch.equal(y.view(torch.int16), rows_y.view(torch.int16))


@pytest.mark.parametrize("rows", [1, 16, 40, 200])
def test_int32_partials_bit_exact(cuda_device, rows):
    k, m = 448, 320
    x = I.activations(rows, k, 300 + rows, outliers=3)
    w = I.weight(m, k, 301)
    fp16 = I.keep_ids(5, 7, 0.1, 302)
    p = tq.pack_weight_from_tile_ids(w.to(DEV), n_tr=5, n_tc=7, int8_tile_ids=I.complement_ids(fp16, 35),
                                     fp16_tile_ids=fp16, cfg=cfg())
    q, sx = tq.quantize_activation_tile_absmax(x.to(DEV))
    parts = tq.gemm_int8_partials(x_int8=q, int8_tiles=p.int8_tiles, int8_tile_ids=p.int8_tile_ids,
                                  int8_row_ptr=p.int8_row_ptr, K=k, n_tr=5, n_tc=7)
    pk = O.pack(I.bits(w), 5, 7, I.complement_ids(fp16, 35).numpy(), fp16.numpy())
    _, ref = O.gemm(q.cpu().numpy(), sx.cpu().numpy(), pk, I.bits(x), m, k, want_partials=True)
    np.testing.assert_array_equal(parts.cpu().numpy(), ref)


def test_gemm_split_deterministic_and_bias_fp16_out(cuda_device):
    x, p, M, K, split, bias = _gemm_case("ragged_bias_s2")
    outs = [_run_gemm(x, p, M, K, 2, bias) for _ in range(3)]
    assert all(torch.equal(outs[0].view(torch.int16), o.view(torch.int16)) for o in outs[1:])
    # float16 output + float16 bias (MixedLinear's default dtype_out)
    xg = to_torch16(x, torch.bfloat16, DEV)
    q, sx = tq.quantize_activation_tile_absmax(xg)
    b16 = to_torch16(bias, torch.bfloat16, DEV).to(torch.float16)
    y = tq.gemm_mixed_rows_splitk(x_fp=xg, x_int8=q, sx=sx, int8_tiles=p.int8_tiles, int8_scales=p.int8_scales,
                                  int8_tile_ids=p.int8_tile_ids, int8_row_ptr=p.int8_row_ptr, fp16_tiles=p.fp16_tiles,
                                  fp16_tile_ids=p.fp16_tile_ids, fp16_row_ptr=p.fp16_row_ptr, M=M, K=K, n_tr=p.n_tr,
                                  n_tc=p.n_tc, out_dtype=torch.float16, bias=b16, split_k=2)
    pk = O.pack(to_np := I.bits(to_torch16(GEMM["ragged_bias_s2__w"], torch.bfloat16)), p.n_tr, p.n_tc,
                p.int8_tile_ids.cpu().numpy(), p.fp16_tile_ids.cpu().numpy())
    qn, sxn = O.quantize_act(x)
    ref = O.gemm(qn, sxn, pk, x, M, K, split_k=2, bias_bits=from_torch16(b16), odtype=O.F16)
    assert_close_with_bias(from_torch16(y), ref, from_torch16(b16), "fp16 out", dtype_code=1)


def test_gemm_out_view_and_errors(cuda_device):
    x, p, M, K, split, bias = _gemm_case("rows40_iaa_s1")
    xg = to_torch16(x, torch.bfloat16, DEV)
    q, sx = tq.quantize_activation_tile_absmax(xg)
    kw = dict(int8_tiles=p.int8_tiles, int8_scales=p.int8_scales, int8_tile_ids=p.int8_tile_ids,
              int8_row_ptr=p.int8_row_ptr, fp16_tiles=p.fp16_tiles, fp16_tile_ids=p.fp16_tile_ids,
              fp16_row_ptr=p.fp16_row_ptr, M=M, K=K, n_tr=p.n_tr, n_tc=p.n_tc, out_dtype=torch.bfloat16)
    full = tq.gemm_mixed_rows_splitk(x_fp=xg, x_int8=q, sx=sx, **kw)
    big = torch.zeros((50, M + 8), device=DEV, dtype=torch.bfloat16)
    view = big[5:45, 3:3 + M]
    tq.gemm_mixed_rows_splitk(x_fp=xg, x_int8=q, sx=sx, out=view, **kw)
    assert torch.equal(view, full)
    assert int(big[:5].abs().sum()) == 0 and int(big[45:].abs().sum()) == 0
    with pytest.raises(ValueError):
        tq.gemm_mixed_rows_splitk(x_fp=xg, x_int8=q, sx=sx, out=big, **kw)
    with pytest.raises(ValueError):
        tq.gemm_mixed_rows_splitk(x_fp=xg, x_int8=q, sx=sx, split_k=17, **kw)


# ----------------------------------------------------------------- MixedLinear

def _linear(m, k, keep, seed, bias=False, dtype_out="bf16", **kw):
    w = I.weight(m, k, seed)
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    fp16 = I.keep_ids(n_tr, n_tc, keep, seed + 1)
    p = tq.pack_weight_from_tile_ids(w.to(DEV), n_tr=n_tr, n_tc=n_tc, int8_tile_ids=I.complement_ids(fp16, n_tr * n_tc),
                                     fp16_tile_ids=fp16, cfg=cfg())
    b = I.weight(1, m, seed + 2, std=0.3).reshape(-1).to(DEV) if bias else None
    return tq.MixedLinear(p, b, cfg(dtype_out=dtype_out, **kw)), w, fp16, b


@pytest.mark.parametrize("rows", [1, 4, 16, 64, 65, 700])
def test_mixed_linear_forward_matches_oracle(cuda_device, rows):
    """MixedLinear vs the oracle run with the split the kernel picked.  Rows > 64 go
    to the prefill kernel when it is available, whose order is checked to 1 ulp."""
    lin, w, fp16, b = _linear(320, 384, 0.1, 400, bias=True)
    x = I.activations(rows, 384, 401, outliers=2)
    with torch.inference_mode():
        y = lin(x.to(DEV).reshape(1, rows, 384))
    assert y.shape == (1, rows, 320) and y.dtype == torch.bfloat16
    q, sx = O.quantize_act(I.bits(x))
    pk = O.pack(I.bits(w), 5, 6, I.complement_ids(fp16, 30).numpy(), fp16.numpy())
    split = 1 if rows > 64 else tq.select_split_k(n_tr=5, n_tc=6, n_rows=rows, device=torch.device(DEV))
    ref = O.gemm(q, sx, pk, I.bits(x), 320, 384, split_k=split, bias_bits=from_torch16(b))
    assert_close_with_bias(from_torch16(y.reshape(rows, 320)), ref, from_torch16(b), f"rows={rows}")


def test_mixed_linear_chunked_equals_unchunked(cuda_device):
    lin, *_ = _linear(256, 512, 0.05, 410, activation_row_chunk_size=100)
    lin_big, *_ = _linear(256, 512, 0.05, 410)
    x = I.activations(333, 512, 411).to(DEV)
    with torch.inference_mode():
        assert torch.equal(lin(x), lin_big(x))


def test_projection_groups_match_members(cuda_device):
    parent = torch.nn.Module()
    members = {}
    for i, name in enumerate(("q_proj", "k_proj", "v_proj")):
        members[name], *_ = _linear(128 if name == "q_proj" else 64, 192, 0.1, 420 + 3 * i, bias=True)
        setattr(parent, name, members[name])
    x = I.activations(40, 192, 430).to(DEV)
    with torch.inference_mode():
        ref = {n: m(x) for n, m in members.items()}
        assert tq.fuse_projection_groups(parent) == 1
        outs = {n: getattr(parent, n)(x) for n in ("q_proj", "k_proj", "v_proj")}
    for n in outs:
        assert torch.equal(outs[n], ref[n]), n


def test_mixed_linear_cuda_graph_capture(cuda_device):
    lin, *_ = _linear(512, 512, 0.02, 440)
    x = I.activations(4, 512, 441).to(DEV)
    with torch.inference_mode():
        eager = lin(x)
        static_x = x.clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            lin(static_x)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = lin(static_x)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
        x2 = I.activations(4, 512, 442).to(DEV)
        static_x.copy_(x2)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, lin(x2))
