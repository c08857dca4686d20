"""Tensor parallelism of the mixed tile GEMM path across the GPUs of one node.

The reference runs on one GPU; this is the split the path shards by (the 64x64 tiles
are independent, and a 64-column tile's activation scale depends only on its own
columns):

* Q/K/V and gate/up are column-parallel: every rank owns a contiguous range of output
  row tiles (attention: whole heads, so 128-row = 2-tile units), packs only those
  tiles, and its output is final for those features;
* O and down are row-parallel: every rank owns a contiguous range of input column
  tiles (attention: the columns of its own heads), packs only those tiles with their
  unchanged per-tile scales, quantizes only those activation columns (the same codes
  and scales the full GEMM computes for them), and the partial outputs are summed
  with one NCCL all-reduce per layer; a bias is added once, after the sum.  With a
  ``PeerExchange`` (``peer.py``), decode-sized calls (1..64 rows) sum the partials
  inside the decode GEMM instead, over NVLink, in FP32 and in rank order.

Attention heads: rank r of t owns query heads [q0, q1) and the KV heads they read.
When there are fewer KV heads than ranks (Qwen2.5-7B: 4 KV heads at TP 8), each KV
head is replicated on t / kv ranks and the query heads of its group are dealt out
among them (7 query heads per KV head -> 3 + 4), so ranks hold 3 or 4 query heads.

The tile maps of the full model are restricted to each rank's tiles, so a rank's pack
holds exactly the tiles (and scales) of the single-GPU pack.  Numerics: the
column-parallel outputs are bit-identical to the single-GPU ones; row-parallel outputs
sum BF16 partials in NCCL's order, so they agree to within a few BF16 ulps.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from .trace import traced

TILE = 64


@dataclass(frozen=True)
class HeadShard:
    q_heads: Tuple[int, int]   # [q0, q1) query heads of this rank
    kv_heads: Tuple[int, int]  # [k0, k1) KV heads of this rank


def split_range(n: int, parts: int, index: int) -> Tuple[int, int]:
    """Contiguous near-equal split of range(n): part `index` of `parts`."""
    return (n * index) // parts, (n * (index + 1)) // parts


def head_shard(n_heads: int, n_kv: int, rank: int, world: int) -> HeadShard:
    """Query and KV heads rank `rank` of `world` owns (grouped-query attention)."""
    if n_heads % n_kv:
        raise ValueError("query heads must be a multiple of KV heads")
    group = n_heads // n_kv
    if world <= n_kv:
        if n_kv % world:
            raise ValueError(f"{n_kv} KV heads do not split over {world} ranks")
        k0, k1 = split_range(n_kv, world, rank)
        return HeadShard((k0 * group, k1 * group), (k0, k1))
    if world % n_kv:
        raise ValueError(f"{world} ranks do not replicate {n_kv} KV heads evenly")
    reps = world // n_kv
    kv = rank // reps
    g0, g1 = split_range(group, reps, rank % reps)
    if g1 <= g0:
        raise ValueError(f"rank {rank} would own no query head")
    return HeadShard((kv * group + g0, kv * group + g1), (kv, kv + 1))


def restrict_keep_ids(keep: torch.Tensor, n_tc: int, rows: Optional[Tuple[int, int]] = None,
                      cols: Optional[Tuple[int, int]] = None) -> Tuple[torch.Tensor, int, int]:
    """Kept 16-bit tile ids of a sub-grid: row tiles [r0, r1) x column tiles [c0, c1) of
    a grid with n_tc column tiles, renumbered within the sub-grid.  Returns (ids, n_tr,
    n_tc) of the sub-grid."""
    keep = keep.to(torch.int64).reshape(-1)
    r, c = keep // n_tc, keep % n_tc
    r0, r1 = rows if rows is not None else (0, int(r.max()) + 1 if keep.numel() else 0)
    c0, c1 = cols if cols is not None else (0, n_tc)
    sel = (r >= r0) & (r < r1) & (c >= c0) & (c < c1)
    sub_tc = c1 - c0
    ids = ((r[sel] - r0) * sub_tc + (c[sel] - c0)).sort().values.to(torch.int32)
    return ids, r1 - r0, sub_tc


def _slice_linear(lin: nn.Linear, rows: Optional[Tuple[int, int]] = None,
                  cols: Optional[Tuple[int, int]] = None, keep_bias: bool = True) -> nn.Linear:
    w = lin.weight.detach()
    if rows is not None:
        w = w[rows[0]:rows[1]]
    if cols is not None:
        w = w[:, cols[0]:cols[1]]
    out = nn.Linear(w.shape[1], w.shape[0], bias=lin.bias is not None and keep_bias, device=w.device, dtype=w.dtype)
    with torch.no_grad():
        out.weight.copy_(w)
        if out.bias is not None:
            b = lin.bias.detach()
            out.bias.copy_(b[rows[0]:rows[1]] if rows is not None else b)
    return out


class PeerReduceSum(nn.Module):
    """Row-parallel ``MixedLinear`` whose decode-sized calls (1..64 rows) sum the ranks'
    partials inside the GEMM through a ``PeerExchange``; larger calls, and shapes whose
    decode grid does not fit the exchange's slots or the GPU at once (the kernel refuses
    those on the host, before any launch, the same way on every rank; the answer is kept
    per shape), take the NCCL all-reduce of ``AllReduceSum``.  The bias is added once,
    after the sum, either way.  Every rank sees the same row counts, so all ranks take
    the same path."""

    MAX_ROWS = 64

    def __init__(self, inner: nn.Module, exchange, group=None, bias: Optional[torch.Tensor] = None):
        super().__init__()
        self.inner = inner
        self.exchange = exchange
        self.group = group
        self.bias = None if bias is None else nn.Parameter(bias.detach().clone(), requires_grad=False)
        self._peer_fits: Dict[int, bool] = {}  # rows -> the peer-sum grid fits

    @traced("tq.PeerReduceSum")
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        from ._native import TileQuantError
        from .peer import gemm_mixed_peer_sum
        from .quant_utils import quantize_activation_tile_absmax

        inner = self.inner
        rows = x.numel() // max(1, x.shape[-1])
        if 0 < rows <= self.MAX_ROWS and x.dim() in (2, 3) and self._peer_fits.get(rows, True):
            x2d = x.reshape(-1, x.shape[-1]).contiguous()
            if x2d.shape[1] != inner.K_orig:
                raise ValueError(f"Input K mismatch: got {x2d.shape[1]}, expected {inner.K_orig}")
            out_dtype = inner._out_dtype()
            bias = None if self.bias is None else self.bias.to(dtype=out_dtype).contiguous()
            x_int8, sx = quantize_activation_tile_absmax(x2d, tile_n=inner.tile_n)
            try:
                y = gemm_mixed_peer_sum(x_fp=x2d, x_int8=x_int8, sx=sx, out_dtype=out_dtype, exchange=self.exchange,
                                        bias=bias, **inner._weights())
                self._peer_fits[rows] = True
                return y.reshape(*x.shape[:-1], inner.M_orig)
            except (ValueError, TileQuantError) as e:
                too_big = any(m in str(e) for m in ("more decode CTAs than exchange slots",
                                                    "does not fit on the GPU at once"))
                if not too_big or rows in self._peer_fits:
                    raise
                self._peer_fits[rows] = False  # this shape's grid does not fit: NCCL from now on
        y = inner(x)
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.all_reduce(y, group=self.group)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y


class AllReduceSum(nn.Module):
    """Row-parallel projection: the wrapped module's partial output summed over the
    process group (NCCL all-reduce, in place), then the bias once."""

    def __init__(self, inner: nn.Module, group=None, bias: Optional[torch.Tensor] = None):
        super().__init__()
        self.inner = inner
        self.group = group
        self.bias = None if bias is None else nn.Parameter(bias.detach().clone(), requires_grad=False)

    @traced("tq.AllReduceSum")
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        y = self.inner(x)
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.all_reduce(y, group=self.group)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y


@dataclass
class LinearShard:
    """How one projection of the full model is sharded on this rank."""

    name: str
    rows: Optional[Tuple[int, int]]  # output features [o0, o1) (column-parallel)
    cols: Optional[Tuple[int, int]]  # input features [i0, i1) (row-parallel)
    bias: Optional[torch.Tensor] = None  # row-parallel bias, added once after the sum


def shard_decoder_(model: nn.Module, rank: int, world: int) -> Dict[str, LinearShard]:
    """Shard a Llama/Qwen2-style decoder in place for tensor parallelism.

    Every attention and MLP projection is replaced by this rank's slice (dense, still
    ``nn.Linear``; row-parallel slices without their bias).  Then pack the slices
    (``apply_sharded_tile_maps``) and wrap the row-parallel ones in ``AllReduceSum``
    (``wrap_row_parallel_``).  Embeddings, norms and the LM head stay replicated.
    Returns the shard of every projection by its full name.
    """
    cfg = model.config.get_text_config(decoder=True)
    n_heads, n_kv = cfg.num_attention_heads, cfg.num_key_value_heads
    head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // n_heads
    if head_dim % TILE:
        raise ValueError("head_dim must be a multiple of the 64-wide tile")
    hs = head_shard(n_heads, n_kv, rank, world)
    inter = cfg.intermediate_size
    if inter % TILE:
        raise ValueError("intermediate size must be a multiple of the 64-wide tile")
    i0, i1 = (TILE * v for v in split_range(inter // TILE, world, rank))
    q_rows = (hs.q_heads[0] * head_dim, hs.q_heads[1] * head_dim)
    kv_rows = (hs.kv_heads[0] * head_dim, hs.kv_heads[1] * head_dim)
    shards: Dict[str, LinearShard] = {}
    for name, mod in list(model.named_modules()):
        attn = getattr(mod, "q_proj", None)
        if isinstance(attn, nn.Linear) and hasattr(mod, "o_proj"):
            for proj, rows in (("q_proj", q_rows), ("k_proj", kv_rows), ("v_proj", kv_rows)):
                setattr(mod, proj, _slice_linear(getattr(mod, proj), rows=rows))
                shards[f"{name}.{proj}"] = LinearShard(f"{name}.{proj}", rows, None)
            o = mod.o_proj
            mod.o_proj = _slice_linear(o, cols=q_rows, keep_bias=False)
            shards[f"{name}.o_proj"] = LinearShard(f"{name}.o_proj", None, q_rows,
                                                   None if o.bias is None else o.bias.detach().clone())
            if hasattr(mod, "num_key_value_groups"):
                mod.num_key_value_groups = (hs.q_heads[1] - hs.q_heads[0]) // (hs.kv_heads[1] - hs.kv_heads[0]) or 1
        gate = getattr(mod, "gate_proj", None)
        if isinstance(gate, nn.Linear) and hasattr(mod, "down_proj"):
            for proj in ("gate_proj", "up_proj"):
                setattr(mod, proj, _slice_linear(getattr(mod, proj), rows=(i0, i1)))
                shards[f"{name}.{proj}"] = LinearShard(f"{name}.{proj}", (i0, i1), None)
            d = mod.down_proj
            mod.down_proj = _slice_linear(d, cols=(i0, i1), keep_bias=False)
            shards[f"{name}.down_proj"] = LinearShard(f"{name}.down_proj", None, (i0, i1),
                                                      None if d.bias is None else d.bias.detach().clone())
    if not shards:
        raise RuntimeError("no attention / MLP projections found to shard")
    return shards


def shard_keep_ids(full_keep: torch.Tensor, full_shape: Tuple[int, int], shard: LinearShard) -> torch.Tensor:
    """The full projection's kept 16-bit tile ids restricted to this rank's shard."""
    m, k = full_shape
    n_tc = (k + TILE - 1) // TILE
    rows = None if shard.rows is None else (shard.rows[0] // TILE, (shard.rows[1] + TILE - 1) // TILE)
    cols = None if shard.cols is None else (shard.cols[0] // TILE, (shard.cols[1] + TILE - 1) // TILE)
    if rows is None:
        rows = (0, (m + TILE - 1) // TILE)
    ids, _, _ = restrict_keep_ids(full_keep, n_tc, rows=rows, cols=cols)
    return ids


def apply_sharded_tile_maps(model: nn.Module, shards: Dict[str, LinearShard], full_keep: Callable,
                            full_shapes: Dict[str, Tuple[int, int]], cfg=None, model_type: str = "llama",
                            iaa_channel_stats: Optional[Dict[str, torch.Tensor]] = None):
    """Pack this rank's projection slices with the full model's tile maps restricted to
    them.  ``full_keep(name, n_tr, n_tc)`` gives the full projection's kept ids (the same
    on every rank); ``full_shapes[name]`` its (out, in) features; ``iaa_channel_stats``
    the full projections' IAA channel means (sliced here to a row-parallel shard's input
    columns)."""
    from .apply import apply_tile_maps

    stats = None
    if iaa_channel_stats is not None:
        stats = {}
        for name, sh in shards.items():
            s = iaa_channel_stats[name]
            stats[name] = s[sh.cols[0]:sh.cols[1]] if sh.cols is not None else s

    def keep_for(name: str, n_tr: int, n_tc: int) -> torch.Tensor:
        m, k = full_shapes[name]
        full = full_keep(name, (m + TILE - 1) // TILE, (k + TILE - 1) // TILE)
        return shard_keep_ids(torch.as_tensor(full), (m, k), shards[name])

    return apply_tile_maps(model, keep_for, cfg, model_type=model_type, iaa_channel_stats=stats, fuse_groups=True)


def wrap_row_parallel_(model: nn.Module, shards: Dict[str, LinearShard], group=None, exchange=None) -> int:
    """Wrap every row-parallel projection (whatever module now holds it) in
    ``AllReduceSum``, or in ``PeerReduceSum`` when a ``PeerExchange`` is given and the
    projection is a ``MixedLinear``; returns how many were wrapped."""
    from .mixed_linear import MixedLinear

    modules = dict(model.named_modules())
    n = 0
    for name, sh in shards.items():
        if sh.cols is None:
            continue
        parent_name, _, attr = name.rpartition(".")
        parent = modules[parent_name] if parent_name else model
        inner = getattr(parent, attr)
        if isinstance(inner, (AllReduceSum, PeerReduceSum)):
            continue
        bias = None if sh.bias is None else sh.bias.to(next(inner.buffers(), sh.bias).device)
        if exchange is not None and isinstance(inner, MixedLinear):
            setattr(parent, attr, PeerReduceSum(inner, exchange, group, bias))
        else:
            setattr(parent, attr, AllReduceSum(inner, group, bias))
        n += 1
    return n


def tensor_parallel_(model: nn.Module, rank: int, world: int, full_keep: Callable, cfg=None, group=None,
                     model_type: str = "llama",
                     iaa_channel_stats: Optional[Dict[str, torch.Tensor]] = None,
                     exchange=None) -> Dict[str, LinearShard]:
    """Shard, pack and wire a dense decoder for tensor parallelism in one call: the
    full model's tile maps ``full_keep(name, n_tr, n_tc)`` (identical on every rank)
    are restricted to this rank's slices.  ``exchange`` (a connected ``PeerExchange``)
    moves the decode-sized row-parallel sums into the GEMM."""
    shapes = projection_shapes(model)
    shards = shard_decoder_(model, rank, world)
    apply_sharded_tile_maps(model, shards, full_keep, shapes, cfg, model_type=model_type,
                            iaa_channel_stats=iaa_channel_stats)
    wrap_row_parallel_(model, shards, group, exchange)
    return shards


def projection_shapes(model: nn.Module) -> Dict[str, Tuple[int, int]]:
    """(out, in) features of every q/k/v/o/gate/up/down ``nn.Linear`` by full name."""
    out: Dict[str, Tuple[int, int]] = {}
    for name, mod in model.named_modules():
        if isinstance(mod, nn.Linear) and name.rsplit(".", 1)[-1] in (
                "q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
            out[name] = (mod.out_features, mod.in_features)
    return out


def seeded_random_keep(fraction: float, seed: int, names: List[str]) -> Callable:
    """Per-projection random tile maps that every rank reproduces: the map of each name
    is drawn from a generator seeded by (seed, the name's index in `names`)."""
    from .apply import random_keep_ids

    index = {n: i for i, n in enumerate(sorted(names))}

    def keep(name: str, n_tr: int, n_tc: int) -> torch.Tensor:
        g = torch.Generator(device="cpu")
        g.manual_seed(int(seed) * 100003 + index[name])
        return random_keep_ids(n_tr, n_tc, fraction, g)

    return keep
