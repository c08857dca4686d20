"""``MixedLinear``: drop-in ``nn.Linear`` replacement over a mixed INT8/16-bit pack.

Mirrors the reference module family (src/models/mixed_linear.py of
HanzhiZhang-Ulrica/TileQuant): the same classes, buffer names (so state dicts
interchange), cfg keys and errors, calling the sm_100a kernels of this package:

* ``MixedLinear``            -- mixed_linear.py:114-254
* ``MixedLinearGroup``       -- mixed_linear.py:265-333
* ``MixedLinearSlice``       -- mixed_linear.py:336-350
* ``fuse_projection_groups`` -- mixed_linear.py:359-386
* activation-quantization sharing between siblings -- mixed_linear.py:37-111

Forward, by activation row count N:
* N <= activation_row_chunk_size: quantize once (shared with sibling projections of
  the same activation when N >= 32 in inference mode), then the GEMM -- up to 16 rows
  the decode kernel, up to 64 the split-K row kernel, above that the tcgen05 kernel
  (the quantizer-fused GEMM, ``gemm_mixed_fused_quant``, stays available; quantizing
  once in its own launch is faster on B200 because the fused form repeats the
  quantization in every CTA);
* larger: tile scales over all rows first, then quantize + GEMM per row chunk, each
  chunk writing its row slice of one output.
All three give identical results: the scales are global over the call's rows.
"""

from __future__ import annotations

import weakref
from dataclasses import dataclass
from typing import Any, Dict, Optional, Tuple

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

# Rows per quantize+GEMM chunk of a large call (the reference's knob; the results do
# not depend on it).  B200's 180 GB lets prefill run in far fewer, larger launches.
DEFAULT_ACTIVATION_ROW_CHUNK_SIZE = 16384
ACTIVATION_QUANT_CACHE_MIN_ROWS = 32


@dataclass
class _SharedQuant:
    source_ref: "weakref.ReferenceType[torch.Tensor]"
    signature: Tuple[Any, ...]
    consumers: set
    x_int8: torch.Tensor
    sx: torch.Tensor


# One inference-only entry per (device, stream): Q/K/V (or gate/up) modules fed the
# same activation reuse one quantization.
_SHARED_QUANT: Dict[Tuple[int, int], _SharedQuant] = {}


def _cfg_get(cfg: Any, key: str, default=None):
    if isinstance(cfg, dict):
        return cfg.get(key, default)
    return getattr(cfg, key, default)


def _version(x: torch.Tensor) -> Optional[int]:
    try:
        return int(x._version)
    except RuntimeError:  # inference tensors carry no version counter
        return None


def _signature(x: torch.Tensor, extra: Tuple[Any, ...] = ()) -> Tuple[Any, ...]:
    return (int(x.data_ptr()), int(x.storage_offset()), tuple(x.shape), tuple(x.stride()), x.dtype, x.device,
            _version(x)) + extra


def _quantize_shared_activation(source: torch.Tensor, x_work: torch.Tensor, tile_n: int, consumer_id: int):
    if int(x_work.shape[0]) < ACTIVATION_QUANT_CACHE_MIN_ROWS or not (
        torch.is_inference_mode_enabled() and x_work.is_cuda
    ):
        return quantize_activation_tile_absmax(x_work, tile_n=tile_n)
    slot = (int(x_work.device.index or 0), int(torch.cuda.current_stream(x_work.device).cuda_stream))
    sig = _signature(x_work, (int(tile_n), _version(source)))
    hit = _SHARED_QUANT.get(slot)
    if hit is not None and hit.source_ref() is source and hit.signature == sig and consumer_id not in hit.consumers:
        hit.consumers.add(consumer_id)
        return hit.x_int8, hit.sx
    _SHARED_QUANT.pop(slot, None)  # do not keep an unrelated activation alive
    x_int8, sx = quantize_activation_tile_absmax(x_work, tile_n=tile_n)
    try:
        def _drop(dead, slot=slot):
            cur = _SHARED_QUANT.get(slot)
            if cur is not None and cur.source_ref is dead:
                _SHARED_QUANT.pop(slot, None)

        ref = weakref.ref(source, _drop)
    except TypeError:
        return x_int8, sx
    _SHARED_QUANT[slot] = _SharedQuant(ref, sig, {consumer_id}, x_int8, sx)
    return x_int8, sx


_BUFFERS = ("int8_tiles", "int8_scales", "int8_tile_ids", "int8_row_ptr", "int8_row_indices", "fp16_tiles",
            "fp16_tile_ids", "fp16_row_ptr", "fp16_row_indices")


class MixedLinear(nn.Module):
    def __init__(self, pack: Pack, bias: Optional[torch.Tensor], cfg: Any):
        super().__init__()
        self.cfg = cfg
        self.M_orig = int(pack.M_orig)
        self.K_orig = int(pack.K_orig)
        self.M = int(pack.M)
        self.K = int(pack.K)
        self.tile_m = int(pack.tile_m)
        self.tile_n = int(pack.tile_n)
        self.n_tr = int(pack.n_tr)
        self.n_tc = int(pack.n_tc)
        for name in _BUFFERS:
            self.register_buffer(name, getattr(pack, name), persistent=True)
        if bias is not None:
            self.bias = nn.Parameter(bias.detach().clone(), requires_grad=False)
        else:
            self.register_parameter("bias", None)

    @property
    def in_features(self) -> int:
        return self.K_orig

    @property
    def out_features(self) -> int:
        return self.M_orig

    def to_pack(self) -> Pack:
        return Pack(M_orig=self.M_orig, K_orig=self.K_orig, M=self.M, K=self.K, tile_m=self.tile_m,
                    tile_n=self.tile_n, n_tr=self.n_tr, n_tc=self.n_tc, **{n: getattr(self, n) for n in _BUFFERS})

    def _out_dtype(self) -> torch.dtype:
        dtype_out = _cfg_get(self.cfg, "dtype_out", "fp16")
        if dtype_out in ("bf16", torch.bfloat16):
            return torch.bfloat16
        return torch.float16

    def _activation_row_chunk_size(self) -> int:
        return max(1, int(_cfg_get(self.cfg, "activation_row_chunk_size", DEFAULT_ACTIVATION_ROW_CHUNK_SIZE)))

    def _out_bias(self, out_dtype: torch.dtype) -> Optional[torch.Tensor]:
        bias = self.bias
        if bias is None:
            return None
        if bias.dtype != out_dtype or not bias.is_contiguous():
            bias = bias.to(dtype=out_dtype).contiguous()
        return bias

    def _weights(self) -> Dict[str, Any]:
        return dict(int8_tiles=self.int8_tiles, int8_scales=self.int8_scales, int8_tile_ids=self.int8_tile_ids,
                    int8_row_ptr=self.int8_row_ptr, fp16_tiles=self.fp16_tiles, fp16_tile_ids=self.fp16_tile_ids,
                    fp16_row_ptr=self.fp16_row_ptr, M=self.M_orig, K=self.K_orig, n_tr=self.n_tr, n_tc=self.n_tc)

    def _gemm_bias(self, x_fp: torch.Tensor, x_int8: torch.Tensor, sx: torch.Tensor,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
        out_dtype = self._out_dtype()
        return gemm_mixed_rows_splitk(x_fp=x_fp, x_int8=x_int8, sx=sx, out_dtype=out_dtype,
                                      bias=self._out_bias(out_dtype), out=out, **self._weights())

    def _forward_chunk(self, x_chunk: torch.Tensor, sx: torch.Tensor, out: torch.Tensor) -> None:
        x_int8 = quantize_activation_tile_with_scales(x_chunk, sx=sx, tile_n=self.tile_n)
        self._gemm_bias(x_fp=x_chunk, x_int8=x_int8, sx=sx, out=out)

    @traced("tq.MixedLinear")
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        in_shape = x.shape
        if x.dim() == 3:
            x2d = x.reshape(-1, x.shape[-1])
        elif x.dim() == 2:
            x2d = x
        else:
            raise ValueError(f"Expected input rank 2 or 3, got shape={tuple(x.shape)}")
        n_rows, k_in = x2d.shape
        if k_in != self.K_orig:
            raise ValueError(f"Input K mismatch: got {k_in}, expected {self.K_orig}")
        x_work = x2d.contiguous()
        out_dtype = self._out_dtype()
        if n_rows <= self._activation_row_chunk_size():
            x_int8, sx = _quantize_shared_activation(x, x_work, self.tile_n, id(self))
            y = self._gemm_bias(x_fp=x_work, x_int8=x_int8, sx=sx)
        else:
            chunk = self._activation_row_chunk_size()
            sx = activation_tile_absmax_scales(x_work, tile_n=self.tile_n)
            y = torch.empty((n_rows, self.M_orig), device=x_work.device, dtype=out_dtype)
            for start in range(0, n_rows, chunk):
                self._forward_chunk(x_work[start:start + chunk], sx, y[start:start + chunk])
        if x.dim() == 3:
            y = y.reshape(in_shape[0], in_shape[1], self.M_orig)
        return y


@dataclass
class _Pending:
    source_ref: "weakref.ReferenceType[torch.Tensor]"
    signature: Tuple[Any, ...]
    consumed: set
    output: torch.Tensor


class MixedLinearGroup(nn.Module):
    """Sibling projections of one activation run as one stacked GEMM (Q/K/V,
    gate/up): one quantization, one launch; every output element comes from the same
    tile sequence and arithmetic as the member's own MixedLinear."""

    def __init__(self, members: "list[MixedLinear]"):
        super().__init__()
        if len(members) < 2:
            raise ValueError("A projection group needs at least two members")
        has_bias = [m.bias is not None for m in members]
        if any(has_bias) and not all(has_bias):
            raise ValueError("Projection group members must all have or all lack bias")
        bias = torch.cat([m.bias.detach() for m in members]) if all(has_bias) else None
        self.linear = MixedLinear(concat_packs_along_rows([m.to_pack() for m in members]), bias, members[0].cfg)
        edges = [0]
        for m in members:
            edges.append(edges[-1] + m.M_orig)
        self.bounds = tuple(zip(edges[:-1], edges[1:]))
        self._pending: Optional[_Pending] = None

    def output_for(self, x: torch.Tensor, index: int) -> torch.Tensor:
        sig = _signature(x)
        p = self._pending
        if p is not None and p.source_ref() is x and p.signature == sig and index not in p.consumed:
            p.consumed.add(index)
            if len(p.consumed) == len(self.bounds):
                self._pending = None
            return p.output
        self._pending = None
        output = self.linear(x)
        try:
            ref = weakref.ref(x)
        except TypeError:
            return output
        self._pending = _Pending(ref, sig, {index}, output)
        return output

    def reset_pending(self) -> None:
        self._pending = None


class MixedLinearSlice(nn.Module):
    """One member projection, served as a column slice of its group's output."""

    def __init__(self, group: MixedLinearGroup, index: int):
        super().__init__()
        object.__setattr__(self, "group", group)  # owned (and counted) by the parent module
        self.index = int(index)
        self.start, self.stop = group.bounds[self.index]
        self.out_features = self.stop - self.start
        self.in_features = group.linear.K_orig

    @traced("tq.MixedLinearSlice")
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.group.output_for(x, self.index)[..., self.start:self.stop]


PROJECTION_GROUPS = (
    ("tilequant_qkv", ("q_proj", "k_proj", "v_proj")),
    ("tilequant_gate_up", ("gate_proj", "up_proj")),
)


def fuse_projection_groups(model: nn.Module) -> int:
    """Replace Q/K/V and gate/up MixedLinear siblings by stacked groups; returns the
    number of groups formed."""
    fused = 0
    for parent in list(model.modules()):
        for group_name, names in PROJECTION_GROUPS:
            members = [getattr(parent, n, None) for n in names]
            if not all(isinstance(m, MixedLinear) for m in members):
                continue
            first = members[0]
            if any(m.K_orig != first.K_orig or m.M_orig % m.tile_m != 0 or m.tile_m != first.tile_m
                   or m.tile_n != first.tile_n or m.int8_tiles.device != first.int8_tiles.device for m in members):
                continue
            if len({m.bias is None for m in members}) != 1:
                continue
            group = MixedLinearGroup(members)
            parent.add_module(group_name, group)
            for i, n in enumerate(names):
                setattr(parent, n, MixedLinearSlice(group, i))
            fused += 1
    return fused


def reset_projection_groups(model: nn.Module) -> None:
    for module in model.modules():
        if isinstance(module, MixedLinearGroup):
            module.reset_pending()
