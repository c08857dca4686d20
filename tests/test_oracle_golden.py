"""Pin the CPU oracle against fixtures produced by the reference implementation.

The fixtures (tests/golden/*.npz) were written by tests/golden/make_golden.py, which
runs the reference's own quantizer, packer, Triton GEMM kernel (interpreter),
calibration collectors and tile-map writer.  Integer and byte results must match
bit for bit; GEMM outputs within 1 BF16 ulp; calibration sums within f32 rounding.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests.golden import inputs as I
from tests.helpers import assert_within_ulp

G = Path(__file__).resolve().parent / "golden"


def _cases(npz, suffix):
    return sorted({k.split("__")[0] for k in npz.files if k.endswith(suffix)})


QUANT = np.load(G / "quant.npz")
PACK = np.load(G / "pack.npz")
GEMM = np.load(G / "gemm.npz")
CALIB = np.load(G / "calib.npz")


@pytest.mark.parametrize("name", _cases(QUANT, "__q"))
def test_quantizer_matches_reference(name):
    x = QUANT[f"{name}__x"]
    dtype = int(QUANT[f"{name}__dtype"][0])
    if QUANT[f"{name}__strided"][0]:
        # exercise the strided addressing: a transposed view of the transposed copy
        x = np.ascontiguousarray(x.T).T
    q, sx = O.quantize_act(x, dtype)
    np.testing.assert_array_equal(sx.view(np.uint32), QUANT[f"{name}__sx"].view(np.uint32))
    np.testing.assert_array_equal(q, QUANT[f"{name}__q"])


def test_quantizer_edge_semantics():
    sx = QUANT["zero_tile__sx"]
    assert sx[1] == 1.0  # all-zero column tile -> scale 1.0
    q = QUANT["ties__q"]
    assert q[0, :9].tolist() == [127, 0, 2, 2, 0, -2, -2, 126, -126]  # half to even


def _pack_inputs(name):
    w = PACK[f"{name}__w"]
    n_tr, n_tc = (int(v) for v in PACK[f"{name}__grid"])
    imp = PACK[f"{name}__imp"] if f"{name}__imp" in PACK.files else None
    if str(PACK[f"{name}__style"]) != "iaa":
        imp = None
    return w, n_tr, n_tc, PACK[f"{name}__in_int8_ids"], PACK[f"{name}__in_fp16_ids"], int(PACK[f"{name}__wdtype"][0]), imp


@pytest.mark.parametrize("name", _cases(PACK, "__in_int8_ids"))
def test_packer_matches_reference(name):
    w, n_tr, n_tc, i8, i16, dtype, imp = _pack_inputs(name)
    pk = O.pack(w, n_tr, n_tc, i8, i16, dtype, imp)
    for key in ("int8_tiles", "int8_tile_ids", "int8_row_ptr", "fp16_tile_ids", "fp16_row_ptr"):
        np.testing.assert_array_equal(pk[key], PACK[f"{name}__{key}"], err_msg=key)
    np.testing.assert_array_equal(pk["int8_scales"].view(np.uint32), PACK[f"{name}__int8_scales"].view(np.uint32))
    np.testing.assert_array_equal(pk["fp16_tiles"], PACK[f"{name}__fp16_tiles"])
    assert list(PACK[f"{name}__dims"]) == [pk["M_orig"], pk["K_orig"], pk["M"], pk["K"], n_tr, n_tc]


def test_packer_config1_matches_reference():
    x, w, fp16, int8, n_tr, n_tc = I.config1(0)
    assert I.sha256(w) == str(PACK["cfg1__w_sha"]), "seeded input generation changed"
    pk = O.pack(I.bits(w), n_tr, n_tc, int8.numpy(), fp16.numpy())
    assert I.sha256(pk["int8_tiles"]) == str(PACK["cfg1__int8_tiles_sha"])
    assert I.sha256(pk["fp16_tiles"]) == str(PACK["cfg1__fp16_tiles_sha"])
    np.testing.assert_array_equal(pk["int8_scales"], PACK["cfg1__int8_scales"])
    np.testing.assert_array_equal(pk["int8_row_ptr"], PACK["cfg1__int8_row_ptr"])
    np.testing.assert_array_equal(pk["int8_tiles"][0], PACK["cfg1__tile0"])


def test_iaa_zero_tile_takes_first_candidate():
    # an all-zero tile ties on all three candidates: the strict '<' keeps 0.75
    sc = PACK["iaa_ragged_zero__int8_scales"]
    ids = PACK["iaa_ragged_zero__int8_tile_ids"]
    assert sc[list(ids).index(2)] == np.float32(0.75)


def _gemm_inputs(name):
    x = GEMM[f"{name}__x"]
    M, K = (int(v) for v in GEMM[f"{name}__MK"])
    if name.startswith("cfg1"):
        _, w, fp16, int8, n_tr, n_tc = I.config1(0)
        pk = O.pack(I.bits(w), n_tr, n_tc, int8.numpy(), fp16.numpy())
    else:
        n_tr, n_tc = (int(v) for v in GEMM[f"{name}__grid"])
        i16 = GEMM[f"{name}__fp16_ids"]
        imp = GEMM[f"{name}__imp"] if f"{name}__imp" in GEMM.files else None
        pk = O.pack(GEMM[f"{name}__w"], n_tr, n_tc, O.int8_ids_from_keep(i16, n_tr, n_tc), i16, O.BF16, imp)
    bias = GEMM[f"{name}__bias"] if f"{name}__bias" in GEMM.files else None
    return x, pk, M, K, int(GEMM[f"{name}__split"][0]), bias


@pytest.mark.parametrize("name", _cases(GEMM, "__y"))
def test_gemm_matches_reference(name):
    x, pk, M, K, split, bias = _gemm_inputs(name)
    q, sx = O.quantize_act(x)
    y = O.gemm(q, sx, pk, x, M, K, split_k=split, bias_bits=bias, use_fma=False)
    d = assert_within_ulp(y, GEMM[f"{name}__y"], 1, name)
    assert (d == 0).mean() > 0.95, f"{name}: only {(d == 0).mean():.3f} bit-identical"


def test_gemm_int32_partials_exact():
    x, pk, M, K, split, _ = _gemm_inputs("ragged_bias_s2")
    q, sx = O.quantize_act(x)
    _, parts = O.gemm(q, sx, pk, x, M, K, want_partials=True)
    n_tc = pk["n_tc"]
    for pos, tid in enumerate(pk["int8_tile_ids"]):
        c = tid % n_tc
        xq = np.zeros((q.shape[0], 64), np.int64)
        width = min(64, K - 64 * c)
        xq[:, :width] = q[:, 64 * c: 64 * c + width]
        ref = xq @ pk["int8_tiles"][pos].astype(np.int64).T
        np.testing.assert_array_equal(parts[pos], ref)


TARGETS = ("layers.0.q_proj", "layers.0.gate_proj", "layers.0.down_proj")


@pytest.mark.parametrize("name", TARGETS)
def test_gi_scores_match_reference(name):
    w = CALIB[f"gi__{name}__w"]
    m, k = w.shape
    scores = np.zeros(((m + 63) // 64, (k + 63) // 64), np.float32)
    for b in range(3):
        O.gi_accumulate(scores, w, CALIB[f"gi__{name}__grad{b}"])
    np.testing.assert_allclose(scores, CALIB[f"gi__{name}__scores"], rtol=2e-5, atol=1e-30)


@pytest.mark.parametrize("name", TARGETS)
def test_iaa_scores_match_reference(name):
    x = CALIB[f"iaa__{name}__x"]
    acc = np.zeros((x.shape[1],), np.float64)
    O.iaa_channel_accumulate(acc, x)
    w = CALIB[f"gi__{name}__w"]
    mean, scores = O.iaa_tile_scores(w, acc, x.shape[0])
    np.testing.assert_array_equal(mean, CALIB[f"iaa__{name}__mean"])
    np.testing.assert_allclose(scores, CALIB[f"iaa__{name}__scores"], rtol=2e-5)


@pytest.mark.parametrize("i", range(4))
def test_topk_matches_reference(i):
    m = O.topk_mask(CALIB[f"topk{i}__imp"], float(CALIB[f"topk{i}__frac"][0]))
    np.testing.assert_array_equal(m, CALIB[f"topk{i}__mask"])


def test_peer_sum_restatement_matches_the_gemm_on_one_rank_and_splits_exactly():
    """The FP32 sums the oracle exposes round to its own output; a K split across two
    'ranks' summed in rank order stays within the unsplit result's rounding."""
    from tests.golden import inputs as I
    from tests.helpers import assert_close_gemm

    m, k, rows = 256, 512, 7
    n_tr, n_tc = m // 64, k // 64
    w = I.bits(I.weight(m, k, 21))
    fp16 = I.keep_ids(n_tr, n_tc, 0.2, 22).numpy()
    x = I.bits(I.activations(rows, k, 23))
    q, sx = O.quantize_act(x)
    full = O.pack(w, n_tr, n_tc, O.int8_ids_from_keep(fp16, n_tr, n_tc), fp16)
    bias = I.bits(I.weight(1, m, 24, std=0.3)).reshape(-1)
    want, acc = O.gemm(q, sx, full, x, m, k, bias_bits=bias, want_f32=True)
    np.testing.assert_array_equal(O.peer_sum([acc], bias_bits=bias), want)
    parts = []
    for c0, c1 in ((0, 4), (4, 8)):
        keep = np.asarray([t for t in fp16 if c0 <= t % n_tc < c1], np.int64)
        keep = (keep // n_tc) * (c1 - c0) + keep % n_tc - c0
        ws = np.ascontiguousarray(w[:, c0 * 64:c1 * 64])
        pk = O.pack(ws, n_tr, c1 - c0, O.int8_ids_from_keep(keep, n_tr, c1 - c0), keep)
        xs = np.ascontiguousarray(x[:, c0 * 64:c1 * 64])
        qs, ss = O.quantize_act(xs)
        np.testing.assert_array_equal(ss, sx[c0:c1])  # a column tile's scale is its own
        parts.append(O.gemm(qs, ss, pk, xs, m, (c1 - c0) * 64, want_f32=True)[1])
    got = O.peer_sum(parts)
    assert_close_gemm(got, O.peer_sum([acc]), "K split over two ranks")
