"""Write the golden fixtures of the mixed tile GEMM path by running the reference.

Run (where the reference checkout is available; it is not needed afterwards):

    TILEQUANT_REFERENCE=/path/to/TileQuant python tests/golden/make_golden.py

What runs, all on the CPU:

* the reference activation quantizer's torch path (src/kernels/quant_utils.py:41-134;
  it is taken whenever the input is not a CUDA tensor);
* the reference packer ``pack_weight_from_tile_ids`` (src/kernels/pack.py:206-224);
* the reference Triton GEMM kernel ``_gemm_mixed_rows_splitk_kernel``
  (src/kernels/triton/gemm_rows_splitk_64x64.py:78-190) under ``TRITON_INTERPRET=1``.
  Two interpreter limits are worked around here, without touching the kernel:
  ``tl.range`` yields Python ints in the interpreter, so it is replaced by a
  generator of 0-d int32 tensors; and BF16 buffers are passed as exact FP32 copies
  with an FP32 output that is rounded to BF16 afterwards (the kernel's
  ``acc.to(bf16)``).  Bias is added afterwards the way the kernel does it for a BF16
  output: ``bf16(f32(bf16(acc)) + f32(bias))``;
* the reference calibration collectors (src/kernels/calibrate.py:42-369) on a tiny
  model, and the reference tile-map writer (src/kernels/mask_io.py:45-68);
* ``_topk_mask`` (src/quantization/decisions.py:174-183), executed from its source
  text because that module does not import in this environment.

Inputs come from ``tests/golden/inputs.py`` (seeded CPU generators); each fixture
stores the inputs it needs or their SHA-256, and the reference outputs.
"""

from __future__ import annotations

import ast
import math
import os
import sys
import time
from pathlib import Path
from types import SimpleNamespace

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch
import torch.nn as nn

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
from tests.golden import inputs as I  # noqa: E402

if not os.environ.get("TILEQUANT_REFERENCE"):
    raise SystemExit("set TILEQUANT_REFERENCE to the reference checkout (see the module docstring)")
REF = Path(os.environ["TILEQUANT_REFERENCE"])
sys.path.insert(0, str(REF))

import triton.language as tl  # noqa: E402
import triton.runtime.interpreter as interp  # noqa: E402

_orig_patch_lang = interp._patch_lang


def _patched_patch_lang(fn):
    ret = _orig_patch_lang(fn)
    langs = [v for v in fn.__globals__.values() if v is tl or getattr(v, "__name__", "") == "triton.language"]

    def _range(a1, a2=None, step=None, **_):
        step = 1 if step is None else step
        start, end = (0, a1) if a2 is None else (a1, a2)
        start = int(start.handle.data) if hasattr(start, "handle") else int(start)
        end = int(end.handle.data) if hasattr(end, "handle") else int(end)
        for i in range(start, end, step):
            yield tl.core.tensor(interp.TensorHandle(np.array(i, dtype=np.int32), tl.int32), tl.int32)

    for lang in langs:
        setattr(lang, "range", _range)
    return ret


interp._patch_lang = _patched_patch_lang

from src.kernels import mask_io as ref_mask_io  # noqa: E402
from src.kernels import quant_utils as ref_qu  # noqa: E402
from src.kernels.calibrate import (  # noqa: E402
    collect_gi_tile_scores,
    collect_iaa_tile_scores_with_channel_stats,
)
from src.kernels.pack import concat_packs_along_rows, pack_weight_from_tile_ids  # noqa: E402
from src.kernels.triton import gemm_rows_splitk_64x64 as ref_gemm  # noqa: E402


def _ref_topk_mask():
    src = (REF / "src/quantization/decisions.py").read_text()
    tree = ast.parse(src)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "_topk_mask")
    ns = {"np": np, "math": math}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), "decisions.py", "exec"), ns)
    return ns["_topk_mask"]


def cfg(style="gi"):
    return SimpleNamespace(tile_m=64, tile_n=64, pad_to_tile=True, quant_style=style)


def pack_np(p, prefix=""):
    d = {}
    for name in ("int8_tiles", "int8_scales", "int8_tile_ids", "int8_row_ptr", "int8_row_indices",
                 "fp16_tile_ids", "fp16_row_ptr", "fp16_row_indices"):
        d[prefix + name] = getattr(p, name).numpy()
    d[prefix + "fp16_tiles"] = I.bits(p.fp16_tiles)
    d[prefix + "dims"] = np.array([p.M_orig, p.K_orig, p.M, p.K, p.n_tr, p.n_tc], np.int64)
    return d


# ------------------------------------------------------------------ quantizer

def make_quant():
    cases = {}
    cases["cfg1"] = I.activations(16, 3072, 0, outliers=8)
    cases["ragged_k"] = I.activations(3, 100, 11)
    cases["rows130"] = I.activations(130, 256, 12)
    z = I.activations(4, 192, 13)
    z[:, 64:128] = 0
    cases["zero_tile"] = z
    # exact ties: absmax 127 gives scale bf16(1.0); +-0.5, 1.5, 2.5 ... round half to even
    t = torch.zeros((2, 64), dtype=torch.float32)
    t[0, 0] = 127.0
    t[0, 1:9] = torch.tensor([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5, -126.5])
    t[1, :8] = torch.tensor([3.5, 4.5, -3.5, -4.5, 100.5, 101.5, 0.25, -0.75])
    cases["ties"] = t.to(torch.bfloat16)
    cases["wide_range"] = (I.activations(8, 512, 14).float() * torch.logspace(-3, 3, 512)).to(torch.bfloat16)
    cases["fp16"] = I.activations(16, 320, 15, outliers=2, dtype=torch.float16)
    cases["strided"] = I.activations(128, 8, 16).t()  # (8, 128) view with strides (1, 8)
    out = {}
    for name, x in cases.items():
        q, sx = ref_qu.quantize_activation_tile_absmax(x, tile_n=64)
        out[f"{name}__x"] = I.bits(x.contiguous())
        out[f"{name}__strided"] = np.array([1 if not x.is_contiguous() else 0])
        out[f"{name}__dtype"] = np.array([0 if x.dtype == torch.bfloat16 else 1])
        out[f"{name}__q"] = q.numpy()
        out[f"{name}__sx"] = sx.numpy()
        # the two-pass API must agree with the one-pass API
        sx2 = ref_qu.activation_tile_absmax_scales(x, tile_n=64)
        q2 = ref_qu.quantize_activation_tile_with_scales(x, sx2, tile_n=64)
        assert torch.equal(sx2, sx) and torch.equal(q2, q), name
    np.savez_compressed(HERE / "quant.npz", **out)
    print("quant.npz", len(cases), "cases")


# --------------------------------------------------------------------- packer

def make_pack():
    out = {}
    # config 1, GI: too large to store whole; hashes + scales + ids + two tiles
    x, w, fp16, int8, n_tr, n_tc = I.config1(0)
    t0 = time.time()
    p = pack_weight_from_tile_ids(w, n_tr=n_tr, n_tc=n_tc, int8_tile_ids=int8, fp16_tile_ids=fp16, cfg=cfg())
    print("config1 pack", time.time() - t0, "s")
    out["cfg1__w_sha"] = np.array(I.sha256(w))
    out["cfg1__int8_tiles_sha"] = np.array(I.sha256(p.int8_tiles.numpy()))
    out["cfg1__fp16_tiles_sha"] = np.array(I.sha256(I.bits(p.fp16_tiles)))
    out["cfg1__int8_scales"] = p.int8_scales.numpy()
    out["cfg1__int8_tile_ids"] = p.int8_tile_ids.numpy()
    out["cfg1__int8_row_ptr"] = p.int8_row_ptr.numpy()
    out["cfg1__fp16_tile_ids"] = p.fp16_tile_ids.numpy()
    out["cfg1__fp16_row_ptr"] = p.fp16_row_ptr.numpy()
    out["cfg1__tile0"] = p.int8_tiles[0].numpy()
    out["cfg1__tile_last"] = p.int8_tiles[-1].numpy()

    small = {}
    # ragged shape (padding on both axes), GI
    w = I.weight(200, 150, 21)
    ids16 = torch.tensor([1, 7], dtype=torch.int32)
    small["ragged_gi"] = (w, 4, 3, I.complement_ids(ids16, 12), ids16, "gi", None)
    # IAA with channel importance: some channels tiny / zero
    w = I.weight(256, 320, 22, std=0.05)
    imp = torch.rand((320,), generator=I.gen(23)) * 3.0
    imp[::17] = 0.0
    imp[5] = 1e-12
    ids16 = I.keep_ids(4, 5, 0.1, 24)
    small["iaa"] = (w, 4, 5, I.complement_ids(ids16, 20), ids16, "iaa", imp)
    # IAA with ragged K (importance shorter than the padded width) and a zero tile
    w = I.weight(130, 100, 25, std=0.05)
    w[64:128, 0:64] = 0
    imp = torch.rand((100,), generator=I.gen(26))
    small["iaa_ragged_zero"] = (w, 3, 2, torch.arange(6, dtype=torch.int32), torch.zeros((0,), dtype=torch.int32), "iaa", imp)
    # GI zero tile, no BF16 tiles at all
    w = I.weight(128, 128, 27)
    w[:64, 64:] = 0
    small["gi_zero_all_int8"] = (w, 2, 2, torch.arange(4, dtype=torch.int32), torch.zeros((0,), dtype=torch.int32), "gi", None)
    # all tiles BF16
    w = I.weight(64, 192, 28)
    small["all_bf16"] = (w, 1, 3, torch.zeros((0,), dtype=torch.int32), torch.arange(3, dtype=torch.int32), "gi", None)
    # FP16 weight, unsorted ids
    w = I.weight(192, 128, 29, dtype=torch.float16)
    small["fp16_unsorted"] = (w, 3, 2, torch.tensor([5, 0, 3, 1], dtype=torch.int32), torch.tensor([4, 2], dtype=torch.int32), "gi", None)
    for name, (w, n_tr, n_tc, i8, i16, style, imp) in small.items():
        p = pack_weight_from_tile_ids(w, n_tr=n_tr, n_tc=n_tc, int8_tile_ids=i8, fp16_tile_ids=i16,
                                      iaa_col_importance=imp, cfg=cfg(style))
        out[f"{name}__w"] = I.bits(w)
        out[f"{name}__wdtype"] = np.array([0 if w.dtype == torch.bfloat16 else 1])
        out[f"{name}__grid"] = np.array([n_tr, n_tc])
        out[f"{name}__in_int8_ids"] = i8.numpy()
        out[f"{name}__in_fp16_ids"] = i16.numpy()
        out[f"{name}__style"] = np.array(style)
        if imp is not None:
            out[f"{name}__imp"] = imp.numpy()
        out.update(pack_np(p, f"{name}__"))
    # concat_packs_along_rows (QKV stacking)
    parts = []
    for i, m in enumerate((128, 64, 64)):
        w = I.weight(m, 192, 30 + i)
        ids16 = I.keep_ids(m // 64, 3, 0.2, 40 + i)
        parts.append(pack_weight_from_tile_ids(w, n_tr=m // 64, n_tc=3, int8_tile_ids=I.complement_ids(ids16, m // 64 * 3),
                                               fp16_tile_ids=ids16, cfg=cfg()))
        out[f"stack{i}__w"] = I.bits(w)
        out[f"stack{i}__in_fp16_ids"] = ids16.numpy()
    out.update(pack_np(concat_packs_along_rows(parts), "stacked__"))
    np.savez_compressed(HERE / "pack.npz", **out)
    print("pack.npz written")


# ----------------------------------------------------------------------- GEMM

def ref_gemm_run(x, xq, sx, p, M, K, split_k, block_n, bias=None):
    """Reference Triton kernel under the interpreter; returns BF16 output bits."""
    n = x.shape[0]
    n_blocks = (n + block_n - 1) // block_n
    out = torch.zeros((n, M), dtype=torch.float32)
    ws = torch.zeros((max(split_k * n * M, 1),), dtype=torch.float32)
    counters = torch.zeros((max(p.n_tr * n_blocks, 4096),), dtype=torch.int32)
    xf = x.float().contiguous()
    tf = p.fp16_tiles.float().contiguous()
    has_fp16 = p.fp16_tiles.numel() != 0
    ref_gemm._gemm_mixed_rows_splitk_kernel[(p.n_tr, n_blocks, split_k)](
        xq, xq.stride(0), sx, p.int8_tiles, p.int8_scales, p.int8_tile_ids, p.int8_row_ptr,
        xf, xf.stride(0), tf if has_fp16 else xf, p.fp16_tile_ids, p.fp16_row_ptr,
        out, out.stride(0), out, ws, n * M, counters, n, M, K,
        n_tc=p.n_tc, BLOCK_N=block_n, SPLIT_K=split_k, HAS_FP16=has_fp16, HAS_BIAS=False,
        NUM_STAGES=3, num_warps=4,
    )
    assert int(counters.abs().sum()) == 0, "split-K counters must return to zero"
    y = out.to(torch.bfloat16)
    if bias is not None:
        y = (y.float() + bias.float()[None, :]).to(torch.bfloat16)
    return y


def make_gemm():
    out = {}
    cases = []
    x, w, fp16, int8, n_tr, n_tc = I.config1(0)
    p1 = pack_weight_from_tile_ids(w, n_tr=n_tr, n_tc=n_tc, int8_tile_ids=int8, fp16_tile_ids=fp16, cfg=cfg())
    cases.append(("cfg1_s1", x, None, p1, 3072, 3072, 1, 16, None))
    cases.append(("cfg1_s8", x, None, p1, 3072, 3072, 8, 16, None))
    # ragged: 5 rows, M=200, K=150, bias, split 2
    w = I.weight(200, 150, 51)
    ids16 = torch.tensor([2, 5, 9], dtype=torch.int32)
    p = pack_weight_from_tile_ids(w, n_tr=4, n_tc=3, int8_tile_ids=I.complement_ids(ids16, 12), fp16_tile_ids=ids16, cfg=cfg())
    bias = I.weight(1, 200, 52, std=0.5).reshape(-1)
    cases.append(("ragged_bias_s2", I.activations(5, 150, 53, outliers=1), w, p, 200, 150, 2, 16, bias))
    # 40 rows (BLOCK_N 64), 10 % BF16, IAA pack
    w = I.weight(256, 320, 54)
    ids16 = I.keep_ids(4, 5, 0.1, 55)
    imp = torch.rand((320,), generator=I.gen(56))
    p = pack_weight_from_tile_ids(w, n_tr=4, n_tc=5, int8_tile_ids=I.complement_ids(ids16, 20), fp16_tile_ids=ids16,
                                  iaa_col_importance=imp, cfg=cfg("iaa"))
    cases.append(("rows40_iaa_s1", I.activations(40, 320, 57, outliers=3), w, p, 256, 320, 1, 64, None))
    # all-INT8 row tiles with split 4 and a row with no INT8 tile at all
    w = I.weight(192, 512, 58)
    ids16 = torch.arange(8, 16, dtype=torch.int32)  # row tile 1 entirely BF16
    p = pack_weight_from_tile_ids(w, n_tr=3, n_tc=8, int8_tile_ids=I.complement_ids(ids16, 24), fp16_tile_ids=ids16, cfg=cfg())
    cases.append(("bf16_row_s4", I.activations(16, 512, 59), w, p, 192, 512, 4, 16, None))
    for name, x, w, p, M, K, split, block_n, bias in cases:
        t0 = time.time()
        xq, sx = ref_qu.quantize_activation_tile_absmax(x, tile_n=64)
        y = ref_gemm_run(x, xq, sx, p, M, K, split, block_n, bias)
        print(f"gemm {name}: {time.time() - t0:.1f}s")
        out[f"{name}__x"] = I.bits(x)
        out[f"{name}__y"] = I.bits(y)
        out[f"{name}__split"] = np.array([split])
        out[f"{name}__MK"] = np.array([M, K])
        if bias is not None:
            out[f"{name}__bias"] = I.bits(bias)
        if w is not None:
            out[f"{name}__w"] = I.bits(w)
            out[f"{name}__style"] = np.array("iaa" if name.endswith("iaa_s1") else "gi")
            out[f"{name}__fp16_ids"] = p.fp16_tile_ids.numpy()
            out[f"{name}__grid"] = np.array([p.n_tr, p.n_tc])
            if name.startswith("rows40_iaa"):
                out[f"{name}__imp"] = imp.numpy()
    np.savez_compressed(HERE / "gemm.npz", **out)
    print("gemm.npz written")


# ---------------------------------------------------------------- calibration

class _TinyLM(nn.Module):
    """Embedding -> q_proj / gate_proj / down_proj -> lm_head, BF16, CPU."""

    def __init__(self, vocab=64, d=96, inter=160):
        super().__init__()
        g = I.gen(70)
        self.emb = nn.Embedding(vocab, d)
        self.layers = nn.ModuleList([nn.Module()])
        blk = self.layers[0]
        blk.q_proj = nn.Linear(d, 130, bias=False)
        blk.gate_proj = nn.Linear(d, inter, bias=False)
        blk.down_proj = nn.Linear(inter, d, bias=False)
        blk.back = nn.Linear(130, d, bias=False)
        self.lm_head = nn.Linear(d, vocab, bias=False)
        with torch.no_grad():
            for prm in self.parameters():
                prm.copy_(torch.randn(prm.shape, generator=g) * 0.2)
        self.to(torch.bfloat16)

    def forward(self, input_ids, attention_mask=None):
        h = self.emb(input_ids)
        blk = self.layers[0]
        h = h + blk.back(torch.tanh(blk.q_proj(h)))
        h = h + blk.down_proj(torch.nn.functional.silu(blk.gate_proj(h)))
        return SimpleNamespace(logits=self.lm_head(h).float())


def make_calib():
    out = {}
    model = _TinyLM()
    ids = torch.randint(0, 64, (3, 2, 12), generator=I.gen(71))
    batches = [{"input_ids": ids[i]} for i in range(3)]
    targets = ("layers.0.q_proj", "layers.0.gate_proj", "layers.0.down_proj")
    flt = lambda name: name in targets  # noqa: E731
    c = SimpleNamespace(tile_m=64, tile_n=64, calib={})
    gi = collect_gi_tile_scores(model, batches, flt, c)
    # per-batch gradients, recomputed the same way the collector computes them
    for b, batch in enumerate(batches):
        model.zero_grad(set_to_none=True)
        outputs = model(**batch)
        logits = outputs.logits
        loss = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]),
                                                 batch["input_ids"][:, 1:].reshape(-1))
        loss.backward()
        for name in targets:
            mod = model.get_submodule(name)
            out[f"gi__{name}__grad{b}"] = I.bits(mod.weight.grad)
    model.zero_grad(set_to_none=True)
    for name in targets:
        mod = model.get_submodule(name)
        out[f"gi__{name}__w"] = I.bits(mod.weight.detach())
        out[f"gi__{name}__scores"] = gi[name].numpy()
    # IAA: record each target's inputs with a hook of our own, next to the collector's
    seen = {name: [] for name in targets}
    hooks = [model.get_submodule(n).register_forward_pre_hook(lambda m, a, n=n: seen[n].append(a[0].detach().clone()))
             for n in targets]
    scores, means = collect_iaa_tile_scores_with_channel_stats(model, batches, flt, c)
    for h in hooks:
        h.remove()
    for name in targets:
        out[f"iaa__{name}__x"] = I.bits(torch.cat([t.reshape(-1, t.shape[-1]) for t in seen[name]]))
        out[f"iaa__{name}__scores"] = scores[name].numpy()
        out[f"iaa__{name}__mean"] = means[name].numpy()
    # top-k keep masks
    topk = _ref_topk_mask()
    for i, frac in enumerate((0.01, 0.05, 0.2, 1.0)):
        imp = np.random.default_rng(80 + i).random((48, 48)).astype(np.float32)
        out[f"topk{i}__imp"] = imp
        out[f"topk{i}__frac"] = np.array([frac])
        out[f"topk{i}__mask"] = topk(imp, frac)
    np.savez_compressed(HERE / "calib.npz", **out)
    print("calib.npz written")


def make_masks():
    """A tile-map archive written by the reference writer (Llama-3.2-3B stems/grids)."""
    grids = {"q_proj": (48, 48), "k_proj": (16, 48), "v_proj": (16, 48), "o_proj": (48, 48),
             "gate_proj": (128, 48), "up_proj": (128, 48), "down_proj": (48, 128)}
    masks = {}
    rng = np.random.default_rng(90)
    for layer in range(2):
        for proj, (n_tr, n_tc) in grids.items():
            blk = "self_attn" if proj in ("q_proj", "k_proj", "v_proj", "o_proj") else "mlp"
            stem = f"model_layers_{layer}_{blk}_{proj}"
            m = np.zeros((n_tr * n_tc,), np.uint8)
            m[rng.choice(n_tr * n_tc, size=math.ceil(0.01 * n_tr * n_tc), replace=False)] = 1
            masks[stem] = m.reshape(n_tr, n_tc)
    big = np.zeros((300, 300), np.uint8)  # > 65535 tiles: ids stored as uint32
    big.reshape(-1)[[0, 70000, 89999]] = 1
    masks["model_layers_0_mlp_big_proj"] = big
    path = ref_mask_io.save_mask_keep_archive(HERE / "keep01", masks)
    print("tile map", path)


if __name__ == "__main__":
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    which = sys.argv[1:] or ["quant", "pack", "gemm", "calib", "masks"]
    for w in which:
        globals()[f"make_{w}"]()
