"""Write the greedy-token fixtures by running the reference's own model path on the CPU.

Run (where the reference checkout is available; it is not needed afterwards):

    TILEQUANT_REFERENCE=/path/to/TileQuant python tests/golden/make_tokens.py

For each tiny decoder (a Llama and a Qwen2 with Q/K/V bias, random-init from a fixed
seed, FP16: the reference MixedLinear's default output type), every target projection is replaced by the reference's ``MixedLinear``
(src/models/mixed_linear.py:114-254) over the reference packer's pack
(src/kernels/pack.py:206-224), 10 % of each projection's 64x64 tiles kept 16-bit
(seeded, uniform).  The reference's mixed GEMM is its Triton kernel
``_gemm_mixed_rows_splitk_kernel`` (src/kernels/triton/gemm_rows_splitk_64x64.py:78-190)
run under ``TRITON_INTERPRET=1`` (with ``make_golden``'s two interpreter work-arounds:
its ``tl.range`` patch, and FP32 copies of the 16-bit operands with the FP32 output
rounded to the 16-bit type afterwards; split 1); the reference's launcher, which needs a CUDA
stream, is the one thing replaced.  The activation quantizer is the reference's torch
path.  Attention runs on FP32 copies with its output rounded once to FP16 (the numerics of the
flash attention the reference decodes with; a CPU attention in FP16 is far less
precise).  Greedy decoding runs the Hugging Face model with a dynamic cache: the prompt
(batch 8 x 16 seeded ids), then 31 one-token steps, 32 tokens in all -- the tokens the
reference's CUDA-graph decoder produces for the same model (src/runtime/graph_decode.py
:428-452 is greedy argmax over the same logits).

Stored per model: the prompt, the 32 tokens, the FP16 logits of every step, the top-1
minus top-2 logit margin of every
step in FP16 ulps of the top logit (the slack a rounding difference elsewhere in the model
would have to overcome), the rows whose margin is at least MIN_MARGIN_ULPS at every step,
the kept tile ids of every projection, and a SHA-256 of the initial weights so the GPU
test can check it rebuilt the same model.
"""

from __future__ import annotations

import os
import sys
import time
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from tests.golden import make_golden as G  # noqa: E402  (sets up the interpreter and the reference path)
from src.kernels.pack import pack_weight_from_tile_ids  # noqa: E402
from src.models import mixed_linear as ref_ml  # noqa: E402
from src.models.rules import iter_target_linears  # noqa: E402

from tests.golden.tiny_models import (  # noqa: E402
    BATCH, DTYPE, MIN_MARGIN_ULPS, MODELS, NEW_TOKENS, PROMPT_LEN, build, keep_ids_for, margin_ulps, state_sha)


def interp_gemm(*, x_fp, x_int8, sx, int8_tiles, int8_scales, int8_tile_ids, int8_row_ptr, fp16_tiles, fp16_tile_ids,
                fp16_row_ptr, M, K, n_tr, n_tc, out_dtype, bias=None, split_k=None, out=None):
    """The reference launcher's contract, run by its kernel under the interpreter (split
    1): FP32 copies of the 16-bit operands in, an FP32 output rounded to ``out_dtype``
    afterwards, then the bias added the way the kernel adds it for a 16-bit output."""
    n = x_fp.shape[0]
    block_n = 16 if n <= 16 else 32
    n_blocks = (n + block_n - 1) // block_n
    acc = torch.zeros((n, M), dtype=torch.float32)
    ws = torch.zeros((max(n * M, 1),), dtype=torch.float32)
    counters = torch.zeros((max(n_tr * n_blocks, 4096),), dtype=torch.int32)
    xf = x_fp.float().contiguous()
    tf = fp16_tiles.float().contiguous()
    has_fp16 = fp16_tiles.numel() != 0
    G.ref_gemm._gemm_mixed_rows_splitk_kernel[(n_tr, n_blocks, 1)](
        x_int8, x_int8.stride(0), sx, int8_tiles, int8_scales, int8_tile_ids, int8_row_ptr,
        xf, xf.stride(0), tf if has_fp16 else xf, fp16_tile_ids, fp16_row_ptr,
        acc, acc.stride(0), acc, ws, n * M, counters, n, M, K,
        n_tc=n_tc, BLOCK_N=block_n, SPLIT_K=1, HAS_FP16=has_fp16, HAS_BIAS=False, NUM_STAGES=3, num_warps=4,
    )
    y = acc.to(out_dtype)
    if bias is not None:
        y = (y.float() + bias.float()[None, :]).to(out_dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def _fp32_attention(module, query, key, value, attention_mask, **kwargs):
    """Hugging Face's SDPA attention on FP32 copies, rounded once to the model's 16-bit
    type: the numerics of the attention the reference decodes with on the GPU (flash
    attention accumulates in FP32 and rounds its output once), which a CPU attention
    computed in FP16 does not reproduce."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    mask = attention_mask.float() if attention_mask is not None and attention_mask.is_floating_point() else attention_mask
    out, weights = sdpa_attention_forward(module, query.float(), key.float(), value.float(), mask, **kwargs)
    return out.to(query.dtype), weights


def reference_model(name):
    from transformers import AttentionInterface

    spec = MODELS[name]
    model = build(spec)
    sha = state_sha(model)
    AttentionInterface.register("tilequant_fp32_sdpa", _fp32_attention)
    model.set_attn_implementation("tilequant_fp32_sdpa")
    cfg = SimpleNamespace(tile_m=64, tile_n=64, pad_to_tile=True, quant_style="gi", dtype_out="fp16")
    keep = {}
    for parent, attr, full, lin in iter_target_linears(model, cfg, model_type=spec["arch"]):
        w = lin.weight.detach()
        n_tr, n_tc = (w.shape[0] + 63) // 64, (w.shape[1] + 63) // 64
        ids16 = keep_ids_for(name, full, n_tr, n_tc)
        keep[full] = ids16
        mask = torch.zeros(n_tr * n_tc, dtype=torch.bool)
        mask[ids16.long()] = True
        ids8 = torch.nonzero(~mask).reshape(-1).to(torch.int32)
        pack = pack_weight_from_tile_ids(w, n_tr=n_tr, n_tc=n_tc, int8_tile_ids=ids8, fp16_tile_ids=ids16, cfg=cfg)
        bias = None if lin.bias is None else lin.bias.detach()
        setattr(parent, attr, ref_ml.MixedLinear(pack, bias, cfg))
    return model, keep, sha


@torch.inference_mode()
def greedy(model, prompt):
    out = model(input_ids=prompt, use_cache=True)
    tokens, margins, all_logits = [], [], []
    cache = out.past_key_values
    logits = out.logits[:, -1].float()
    for step in range(NEW_TOKENS):
        tok = logits.argmax(-1)
        tokens.append(tok)
        margins.append(margin_ulps(logits.topk(2, dim=-1).values))
        all_logits.append(logits.to(DTYPE))
        if step + 1 == NEW_TOKENS:
            break
        out = model(input_ids=tok[:, None], past_key_values=cache, use_cache=True)
        cache = out.past_key_values
        logits = out.logits[:, -1].float()
    return torch.stack(tokens, 1), torch.stack(margins, 1), torch.stack(all_logits, 1)


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref_ml.gemm_mixed_rows_splitk = interp_gemm
    out = {}
    for name, spec in MODELS.items():
        t0 = time.time()
        model, keep, sha = reference_model(name)
        prompt = torch.randint(0, spec["vocab"], (BATCH, PROMPT_LEN), generator=torch.Generator().manual_seed(spec["seed"] + 5))
        tokens, margins, logits = greedy(model, prompt)
        out[f"{name}__prompt"] = prompt.numpy()
        out[f"{name}__tokens"] = tokens.numpy()
        out[f"{name}__margins"] = margins.numpy()
        out[f"{name}__logits"] = logits.numpy()
        out[f"{name}__rows"] = np.flatnonzero((margins >= MIN_MARGIN_ULPS).all(1).numpy()).astype(np.int64)
        out[f"{name}__state_sha"] = np.array(sha)
        for full, ids in keep.items():
            out[f"{name}__keep__{full}"] = ids.numpy()
        print(f"{name}: {time.time() - t0:.1f} s, per-row min margin (FP16 ulps) {margins.min(1).values.tolist()}, "
              f"rows kept {out[f'{name}__rows'].tolist()}")
    np.savez_compressed(HERE / "tokens.npz", **out)
    print("tokens.npz written")


if __name__ == "__main__":
    main()
