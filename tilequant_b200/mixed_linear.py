"""``MixedLinear``: drop-in ``nn.Linear`` replacement over a mixed INT8/16-bit pack.

Public surface of the reference module family (src/models/mixed_linear.py of
HanzhiZhang-Ulrica/TileQuant), kept so models and state dicts interchange: the classes
``MixedLinear`` (:114-254), ``MixedLinearGroup`` (:265-333), ``MixedLinearSlice``
(:336-350), ``fuse_projection_groups`` / ``reset_projection_groups`` (:353-392), the
buffer names (the ``Pack`` fields), the cfg keys ``dtype_out`` (default fp16) and
``activation_row_chunk_size``, the group submodule names and the ``ValueError`` messages.

How a forward runs here, by activation row count N (rows = tokens):

* N <= the chunk size: one quantization (per-64-column scales over all N rows, then the
  INT8 codes) and one mixed GEMM launch; the GEMM picks its kernel by N (the decode
  kernel up to 16 rows, the split-K row kernel up to 64, the tcgen05 kernel above);
* N > the chunk size: the scales over all N rows first, then quantize + GEMM per chunk
  of rows, each chunk writing its row slice of one output.
The scales are global over the call's rows either way, so both give the same bits.

Work shared between modules that read the same activation is remembered on the
activation tensor itself (``_Memo``): an entry records a fingerprint of the tensor (its
storage address, offset, shape, strides, dtype, version counter when it has one, and
the CUDA stream) and which consumers it has served; an entry whose fingerprint no
longer matches, or that a consumer asks for a second time, is recomputed.  Two things
use it:

* sibling ``MixedLinear`` modules (Q/K/V or gate/up that were not stacked) quantize a
  shared activation once -- only in inference mode, on CUDA, from 32 rows up (the
  reference's threshold: below it the quantization is a single small launch);
* a ``MixedLinearGroup`` (stacked siblings) runs its one GEMM when the first member
  slice asks and serves the other members from the same output.
The entry lives exactly as long as the activation tensor, so nothing outlives the
tensor it was derived from.
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from .gemm import gemm_mixed_rows_splitk
from .pack import Pack, concat_packs_along_rows
from .quant_utils import (
    activation_tile_absmax_scales,
    quantize_activation_tile_absmax,
    quantize_activation_tile_with_scales,
)
from .trace import traced

# Rows per quantize + GEMM chunk of a large call (the reference's knob and default name;
# results do not depend on it).  B200's 180 GB lets prefill run in larger launches.
DEFAULT_ACTIVATION_ROW_CHUNK_SIZE = 16384
ACTIVATION_QUANT_CACHE_MIN_ROWS = 32

_PACK_BUFFERS = ("int8_tiles", "int8_scales", "int8_tile_ids", "int8_row_ptr", "int8_row_indices", "fp16_tiles",
                 "fp16_tile_ids", "fp16_row_ptr", "fp16_row_indices")


def _cfg_value(cfg: Any, key: str, default=None):
    """cfg may be a mapping or an attribute namespace (both occur in the reference)."""
    return cfg.get(key, default) if isinstance(cfg, dict) else getattr(cfg, key, default)


# --------------------------------------------------------------------------- memos

class _Memo:
    """Work derived from one activation tensor, stored on that tensor.

    ``lookup`` returns the value stored under ``key`` if the tensor still matches the
    fingerprint taken when it was stored and ``consumer`` has not been served from it
    yet (a module called twice on the same tensor object -- possibly changed in place
    under inference mode, where tensors carry no version counter -- recomputes)."""

    ATTR = "_tilequant_memo"

    @staticmethod
    def fingerprint(x: torch.Tensor) -> Tuple[Any, ...]:
        try:
            version = int(x._version)
        except RuntimeError:  # inference tensors have no version counter
            version = None
        stream = torch.cuda.current_stream(x.device).cuda_stream if x.is_cuda else 0
        return (x.data_ptr(), x.storage_offset(), tuple(x.shape), x.stride(), x.dtype, version, stream)

    @classmethod
    def _table(cls, x: torch.Tensor, create: bool) -> Optional[Dict[Any, list]]:
        table = getattr(x, cls.ATTR, None)
        if table is None and create:
            try:
                table = {}
                setattr(x, cls.ATTR, table)
            except (AttributeError, RuntimeError):  # tensors that take no attributes: no memo
                return None
        return table

    @classmethod
    def lookup(cls, x: torch.Tensor, key: Any, consumer: Any):
        table = cls._table(x, create=False)
        entry = table.get(key) if table else None
        if entry is None or entry[0] != cls.fingerprint(x) or consumer in entry[1]:
            return None
        entry[1].add(consumer)
        return entry[2]

    @classmethod
    def store(cls, x: torch.Tensor, key: Any, consumer: Any, value: Any) -> None:
        table = cls._table(x, create=True)
        if table is not None:
            table[key] = [cls.fingerprint(x), {consumer}, value]

    @classmethod
    def forget(cls, x: torch.Tensor, key: Any) -> None:
        table = cls._table(x, create=False)
        if table:
            table.pop(key, None)


def _quantize(source: torch.Tensor, x2d: torch.Tensor, tile_n: int, consumer: Any):
    """INT8 codes and per-tile scales of ``x2d`` (a 2-D view of ``source``), shared between
    the consumers of ``source`` where that is allowed (see the module docstring)."""
    shareable = (x2d.shape[0] >= ACTIVATION_QUANT_CACHE_MIN_ROWS and x2d.is_cuda
                 and torch.is_inference_mode_enabled())
    if not shareable:
        return quantize_activation_tile_absmax(x2d, tile_n=tile_n)
    key = ("quant", int(tile_n), x2d.data_ptr(), tuple(x2d.shape), x2d.stride())
    hit = _Memo.lookup(source, key, consumer)
    if hit is None:
        hit = quantize_activation_tile_absmax(x2d, tile_n=tile_n)
        _Memo.store(source, key, consumer, hit)
    return hit


# ---------------------------------------------------------------------- MixedLinear

class MixedLinear(nn.Module):
    """``y = x @ W^T (+ bias)`` with W held as a packed mixed INT8/16-bit tile arena."""

    def __init__(self, pack: Pack, bias: Optional[torch.Tensor], cfg: Any):
        super().__init__()
        self.cfg = cfg
        self.M_orig, self.K_orig = int(pack.M_orig), int(pack.K_orig)
        self.M, self.K = int(pack.M), int(pack.K)
        self.tile_m, self.tile_n = int(pack.tile_m), int(pack.tile_n)
        self.n_tr, self.n_tc = int(pack.n_tr), int(pack.n_tc)
        for name in _PACK_BUFFERS:
            self.register_buffer(name, getattr(pack, name), persistent=True)
        if bias is None:
            self.register_parameter("bias", None)
        else:
            self.bias = nn.Parameter(bias.detach().clone(), requires_grad=False)

    in_features = property(lambda self: self.K_orig)
    out_features = property(lambda self: self.M_orig)

    def to_pack(self) -> Pack:
        dims = dict(M_orig=self.M_orig, K_orig=self.K_orig, M=self.M, K=self.K, tile_m=self.tile_m,
                    tile_n=self.tile_n, n_tr=self.n_tr, n_tc=self.n_tc)
        return Pack(**dims, **{name: getattr(self, name) for name in _PACK_BUFFERS})

    def _out_dtype(self) -> torch.dtype:
        """cfg ``dtype_out``: bf16 or, by default, fp16 (the reference's default)."""
        return torch.bfloat16 if _cfg_value(self.cfg, "dtype_out", "fp16") in ("bf16", torch.bfloat16) else torch.float16

    def _row_chunk(self) -> int:
        return max(1, int(_cfg_value(self.cfg, "activation_row_chunk_size", DEFAULT_ACTIVATION_ROW_CHUNK_SIZE)))

    def _weights(self) -> Dict[str, Any]:
        """The pack arguments of ``gemm_mixed_rows_splitk``."""
        return dict(int8_tiles=self.int8_tiles, int8_scales=self.int8_scales, int8_tile_ids=self.int8_tile_ids,
                    int8_row_ptr=self.int8_row_ptr, fp16_tiles=self.fp16_tiles, fp16_tile_ids=self.fp16_tile_ids,
                    fp16_row_ptr=self.fp16_row_ptr, M=self.M_orig, K=self.K_orig, n_tr=self.n_tr, n_tc=self.n_tc)

    def _launch(self, x_fp: torch.Tensor, x_int8: torch.Tensor, sx: torch.Tensor,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        dtype = self._out_dtype()
        bias = self.bias
        if bias is not None and (bias.dtype != dtype or not bias.is_contiguous()):
            bias = bias.to(dtype=dtype).contiguous()  # the GEMM adds a bias of the output type
        return gemm_mixed_rows_splitk(x_fp=x_fp, x_int8=x_int8, sx=sx, out_dtype=dtype, bias=bias, out=out,
                                      **self._weights())

    def _as_rows(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() not in (2, 3):
            raise ValueError(f"Expected input rank 2 or 3, got shape={tuple(x.shape)}")
        if x.shape[-1] != self.K_orig:
            raise ValueError(f"Input K mismatch: got {x.shape[-1]}, expected {self.K_orig}")
        return x.reshape(-1, self.K_orig).contiguous()

    @traced("tq.MixedLinear")
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        rows = self._as_rows(x)
        n, chunk = rows.shape[0], self._row_chunk()
        if n <= chunk:
            x_int8, sx = _quantize(x, rows, self.tile_n, id(self))
            y = self._launch(rows, x_int8, sx)
        else:  # scales over every row first, so each chunk quantizes like the whole call
            sx = activation_tile_absmax_scales(rows, tile_n=self.tile_n)
            y = torch.empty((n, self.M_orig), device=rows.device, dtype=self._out_dtype())
            for lo in range(0, n, chunk):
                part = rows[lo:lo + chunk]
                self._launch(part, quantize_activation_tile_with_scales(part, sx=sx, tile_n=self.tile_n), sx,
                             out=y[lo:lo + chunk])
        return y.reshape(*x.shape[:-1], self.M_orig)


# --------------------------------------------------------------- stacked projections

class MixedLinearGroup(nn.Module):
    """Sibling projections of one activation (Q/K/V, gate/up) stacked along the output
    rows into one ``MixedLinear``: one quantization and one GEMM for all members, every
    output element from the same tile sequence and arithmetic as the member's own."""

    def __init__(self, members: List[MixedLinear]):
        super().__init__()
        if len(members) < 2:
            raise ValueError("A projection group needs at least two members")
        with_bias = {m.bias is not None for m in members}
        if len(with_bias) > 1:
            raise ValueError("Projection group members must all have or all lack bias")
        bias = torch.cat([m.bias.detach() for m in members]) if with_bias == {True} else None
        self.linear = MixedLinear(concat_packs_along_rows([m.to_pack() for m in members]), bias, members[0].cfg)
        widths = torch.tensor([m.M_orig for m in members])
        ends = widths.cumsum(0).tolist()
        self.bounds = tuple((e - w, e) for e, w in zip(ends, widths.tolist()))
        self._epoch = 0  # bumped by reset_pending: outputs stored before it are not served

    def output_for(self, x: torch.Tensor, index: int) -> torch.Tensor:
        """The stacked output for activation ``x``, computed when the first member asks and
        served once to each member; a member asking again recomputes."""
        key = ("group", id(self), self._epoch)
        out = _Memo.lookup(x, key, index)
        if out is None:
            out = self.linear(x)
            _Memo.store(x, key, index, out)
        return out

    def reset_pending(self) -> None:
        self._epoch += 1


class MixedLinearSlice(nn.Module):
    """Member ``index`` of a group: its column range of the group's stacked output."""

    def __init__(self, group: MixedLinearGroup, index: int):
        super().__init__()
        # the group module is registered on the parent (state dict key tilequant_*); the
        # slice only refers to it
        self.__dict__["group"] = group
        self.index = int(index)
        self.start, self.stop = group.bounds[self.index]
        self.in_features, self.out_features = group.linear.K_orig, self.stop - self.start

    @traced("tq.MixedLinearSlice")
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.group.output_for(x, self.index)[..., self.start:self.stop]


# (group submodule name, member attribute names): the reference's names, which appear in
# state-dict keys of fused models
PROJECTION_GROUPS = (
    ("tilequant_qkv", ("q_proj", "k_proj", "v_proj")),
    ("tilequant_gate_up", ("gate_proj", "up_proj")),
)


def _stackable(members: List[Any]) -> bool:
    """Members can share one stacked pack: all MixedLinear on one device, one input width,
    one tile shape, whole row tiles (a stacked arena has no ragged rows between members),
    and bias on all or none."""
    if not all(isinstance(m, MixedLinear) for m in members):
        return False
    shape = {(m.K_orig, m.tile_m, m.tile_n, m.int8_tiles.device, m.bias is None) for m in members}
    return len(shape) == 1 and all(m.M_orig % m.tile_m == 0 for m in members)


def fuse_projection_groups(model: nn.Module) -> int:
    """Stack every parent module's Q/K/V and gate/up ``MixedLinear`` siblings into a
    ``MixedLinearGroup`` (registered on the parent under its group name, the members
    replaced by slices); returns the number of groups formed."""
    formed = 0
    for parent in list(model.modules()):
        for group_name, names in PROJECTION_GROUPS:
            members = [getattr(parent, n, None) for n in names]
            if not _stackable(members):
                continue
            group = MixedLinearGroup(members)
            parent.add_module(group_name, group)
            for i, n in enumerate(names):
                setattr(parent, n, MixedLinearSlice(group, i))
            formed += 1
    return formed


def reset_projection_groups(model: nn.Module) -> None:
    """Forget every group's stored outputs (the next member call recomputes)."""
    for m in model.modules():
        if isinstance(m, MixedLinearGroup):
            m.reset_pending()
