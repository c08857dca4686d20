"""Which ``nn.Linear`` modules of a decoder become MixedLinear.

Same contract as the reference's src/models/rules.py:9-76: the Q/K/V/O and
gate/up/down projections of Llama- and Qwen2-style decoders, optionally narrowed by
``cfg.module_filters`` (fnmatch patterns over full module names).
"""

from __future__ import annotations

import fnmatch
from typing import Any, List, Tuple

import torch.nn as nn

TARGET_SUFFIXES = ("q_proj", "k_proj", "v_proj", "o_proj", "up_proj", "down_proj", "gate_proj")
LLAMA_TARGET_SUFFIXES = TARGET_SUFFIXES
QWEN_TARGET_SUFFIXES = TARGET_SUFFIXES


def _cfg_get(cfg: Any, key: str, default=None):
    if isinstance(cfg, dict):
        return cfg.get(key, default)
    return getattr(cfg, key, default)


def should_quantize_name(full_name: str, cfg: Any) -> bool:
    patterns = _cfg_get(cfg, "module_filters", None)
    return not patterns or any(fnmatch.fnmatch(full_name, p) for p in patterns)


def iter_target_linears(model: nn.Module, cfg: Any, model_type: str = "llama") -> List[Tuple[nn.Module, str, str, nn.Linear]]:
    """(parent, attribute, full name, linear) for every target projection."""
    suffixes = QWEN_TARGET_SUFFIXES if "qwen" in model_type.lower() else LLAMA_TARGET_SUFFIXES
    modules = dict(model.named_modules())
    found = []
    for name, mod in model.named_modules():
        if not isinstance(mod, nn.Linear) or not name.endswith(suffixes) or not should_quantize_name(name, cfg):
            continue
        parent_name, _, attr = name.rpartition(".")
        found.append((modules[parent_name] if parent_name else model, attr, name, mod))
    return found
