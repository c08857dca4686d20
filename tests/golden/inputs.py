"""Seeded synthetic inputs shared by the fixture generator, the tests and bench.py.

Every tensor comes from a CPU ``torch.Generator`` so the same seed gives the same
bits on any machine with this torch build.  The shapes and value distributions
follow the benchmark configurations of the mixed tile GEMM path:

* config 1 -- one MixedLinear with the Llama-3.2-3B q_proj shape: X (16, 3072) BF16
  N(0, 1) with 8 seeded outlier channels scaled x20; W (3072, 3072) BF16 N(0, 0.02);
  1 % of the 48x48 64x64 tiles kept BF16, chosen uniformly.
"""

from __future__ import annotations

import hashlib
import math

import numpy as np
import torch


def gen(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))
    return g


def activations(rows: int, k: int, seed: int, *, outliers: int = 0, outlier_scale: float = 20.0,
                dtype=torch.bfloat16) -> torch.Tensor:
    g = gen(seed)
    x = torch.randn((rows, k), generator=g, dtype=torch.float32)
    if outliers:
        ch = torch.randperm(k, generator=g)[:outliers]
        x[:, ch] *= outlier_scale
    return x.to(dtype)


def weight(m: int, k: int, seed: int, *, std: float = 0.02, dtype=torch.bfloat16) -> torch.Tensor:
    g = gen(seed)
    return (torch.randn((m, k), generator=g, dtype=torch.float32) * std).to(dtype)


def keep_ids(n_tr: int, n_tc: int, keep_frac: float, seed: int) -> torch.Tensor:
    """Uniformly chosen BF16 keep tile ids, ceil(keep_frac * T) of them, ascending."""
    total = n_tr * n_tc
    n_keep = int(math.ceil(keep_frac * total)) if keep_frac > 0 else 0
    g = gen(seed)
    return torch.randperm(total, generator=g)[:n_keep].sort().values.to(torch.int32)


def complement_ids(fp16_ids: torch.Tensor, total: int) -> torch.Tensor:
    mask = torch.zeros((total,), dtype=torch.bool)
    if fp16_ids.numel():
        mask[fp16_ids.long()] = True
    return torch.nonzero(~mask, as_tuple=False).reshape(-1).to(torch.int32)


def config1(seed: int = 0):
    """(x, W, fp16_ids, int8_ids, n_tr, n_tc) of benchmark config 1."""
    x = activations(16, 3072, seed, outliers=8)
    w = weight(3072, 3072, seed + 1)
    fp16 = keep_ids(48, 48, 0.01, seed + 2)
    return x, w, fp16, complement_ids(fp16, 48 * 48), 48, 48


def bits(t: torch.Tensor) -> np.ndarray:
    """Raw uint16 bit pattern of a 16-bit float tensor."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def sha256(a) -> str:
    if isinstance(a, torch.Tensor):
        a = a.contiguous().view(torch.uint8).numpy() if a.dtype in (torch.bfloat16, torch.float16) else a.contiguous().numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
