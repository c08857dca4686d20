"""Tiny seeded decoders shared by the greedy-token fixture generator (make_tokens.py)
and the GPU test that checks this repository's decoder against those fixtures.

The weights come from a CPU ``torch.manual_seed`` before the Hugging Face constructor,
so the same torch build gives the same bits on any machine (``state_sha`` checks it).
Tile maps: 10 % of every projection's 64x64 tiles kept 16-bit, drawn from a generator
seeded by the model and the module name.

The models run in FP16: a greedy token can only be expected to match across two
implementations when the top logit leads by more than the rounding either one may
introduce, and FP16's 10-bit mantissa makes that slack 8x finer than BF16's.  The
fixture marks the prompt rows whose reference margin is at least MIN_MARGIN_ULPS FP16
ulps at every step.
"""

from __future__ import annotations

import hashlib
import math
import zlib

import torch

PROMPT_LEN, BATCH, NEW_TOKENS, KEEP = 16, 8, 32, 0.10
DTYPE = torch.float16  # the reference MixedLinear's default output type; 10 mantissa bits
MIN_MARGIN_ULPS = 4    # a fixture row counts when its top-1 logit leads by this many FP16 ulps at every step

MODELS = {
    "llama": dict(arch="llama", hidden=256, inter=512, layers=2, heads=4, kv_heads=2, head_dim=64, vocab=512,
                  rope_theta=500000.0, seed=11),
    "qwen2": dict(arch="qwen2", hidden=256, inter=640, layers=2, heads=4, kv_heads=2, head_dim=64, vocab=512,
                  rope_theta=1000000.0, seed=12),
}


def build(spec, device="cpu"):
    """The seeded random-init model (FP16, eval) on the CPU, then moved to `device`."""
    common = dict(hidden_size=spec["hidden"], intermediate_size=spec["inter"], num_hidden_layers=spec["layers"],
                  num_attention_heads=spec["heads"], num_key_value_heads=spec["kv_heads"], vocab_size=spec["vocab"],
                  tie_word_embeddings=False, rope_theta=spec["rope_theta"], max_position_embeddings=256,
                  initializer_range=0.1, attn_implementation="sdpa")
    if spec["arch"] == "llama":
        from transformers import LlamaConfig as Cfg, LlamaForCausalLM as Model

        common["head_dim"] = spec["head_dim"]
    else:
        from transformers import Qwen2Config as Cfg, Qwen2ForCausalLM as Model
    torch.manual_seed(spec["seed"])
    model = Model(Cfg(**common)).to(DTYPE).eval()
    return model.to(device)


def state_sha(model) -> str:
    h = hashlib.sha256()
    for name, t in sorted(model.state_dict().items()):
        h.update(name.encode())
        h.update(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def margin_ulps(logits_top2):
    """(top1 - top2) in FP16 ulps of top1, for a [..., 2] tensor of the two largest logits."""
    top1, top2 = logits_top2[..., 0].float(), logits_top2[..., 1].float()
    ulp = torch.exp2(torch.floor(torch.log2(top1.abs().clamp_min(2.0 ** -14))) - 10)
    return (top1 - top2) / ulp


def keep_ids_for(model_name: str, module: str, n_tr: int, n_tc: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(MODELS[model_name]["seed"] * 1000003 + zlib.crc32(module.encode()))
    total = n_tr * n_tc
    n_keep = int(math.ceil(KEEP * total))
    return torch.randperm(total, generator=g)[:n_keep].sort().values.to(torch.int32)
