"""One greedy decode step of a Llama/Qwen2-style decoder through fused kernels.

The reference decodes by running the transformers model forward inside its CUDA graph
(src/runtime/graph_decode.py:428-452): every RMSNorm, residual add, RoPE, cache update,
activation and quantization is its own framework operator, about forty launches per
layer, and its attention is ``aten._flash_attention_forward`` over a token-major cache
(src/runtime/graph_decode.py:58-70).  ``FusedDecodeStep`` computes the same step from
the same modules' parameters with the kernels of ``csrc/decode_ops.cu``:

    add_rmsnorm       residual add + RMSNorm                      (1 launch)
    QKV projection    quantizer + mixed tile GEMM                 (2)
    attn_decode       RoPE, cache write, split-KV attention over
                      the valid prefix, merge + O-input quantizer (2)
    O projection      mixed tile GEMM on those codes              (1)
    add_rmsnorm                                                   (1)
    gate/up           quantizer + mixed tile GEMM                 (2)
    silu_mul_quant    SiLU(gate) * up + down-input quantizer      (1)
    down projection   mixed tile GEMM on those codes              (1)

Projections that are not plain ``MixedLinear`` (tensor-parallel wrappers, or anything
else with the module interface) are called as modules on the 16-bit activations.  The
KV cache is the transformers ``StaticCache`` the prefill filled (head-major
[batch, kv_heads, max_len, head_dim]); the step writes slot ``position`` itself.
"""

from __future__ import annotations

import ctypes
import math
from typing import List, Optional

import torch
import torch.nn as nn

from . import _native as N
from .mixed_linear import MixedLinear, MixedLinearGroup
from .trace import traced

SUPPORTED_MODEL_TYPES = ("llama", "qwen2")


def add_rmsnorm(resid: torch.Tensor, delta: Optional[torch.Tensor], weight: torch.Tensor, eps: float,
                resid_out: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = weight * rmsnorm(resid + delta) (2-D, 16-bit); with ``delta`` the sum is also
    written to ``resid_out`` (may be ``resid`` itself)."""
    N.require_cuda(resid, delta, weight, resid_out, out)
    rows, hidden = resid.shape
    if out is None:
        out = torch.empty_like(resid)
    if delta is not None and resid_out is None:
        raise ValueError("resid_out is required with delta")
    for t in (resid, delta, resid_out, out):
        if t is not None and (t.dim() != 2 or t.stride(1) != 1 or t.shape != resid.shape or t.dtype != resid.dtype):
            raise ValueError("add_rmsnorm: 2-D tensors of one shape and dtype with unit column stride")
    if weight.numel() != hidden or weight.dtype != resid.dtype or not weight.is_contiguous():
        raise ValueError("add_rmsnorm: weight must be a contiguous [hidden] tensor of the activation dtype")
    lib = N.load()
    N.check(lib.tq_add_rmsnorm(resid.data_ptr(), resid.stride(0), N.ptr(delta), 0 if delta is None else delta.stride(0),
                               weight.data_ptr(), N.ptr(resid_out), 0 if resid_out is None else resid_out.stride(0),
                               out.data_ptr(), out.stride(0), rows, hidden, float(eps), N.dtype_code(resid.dtype),
                               N.stream_of(resid)), "add_rmsnorm")
    return out


def silu_mul_quant(gate: torch.Tensor, up: torch.Tensor, h: Optional[torch.Tensor] = None,
                   q: Optional[torch.Tensor] = None, sx: Optional[torch.Tensor] = None):
    """h = silu(gate) * up (16-bit, each op rounded) and h's INT8 codes and per-64-column
    scales.  gate/up: 2-D views sharing one row stride (the two halves of a stacked
    gate/up output, or two tensors of one layout)."""
    N.require_cuda(gate, up, h, q, sx)
    rows, k = gate.shape
    if up.shape != gate.shape or up.stride() != gate.stride() or gate.stride(1) != 1 or up.dtype != gate.dtype:
        raise ValueError("silu_mul_quant: gate and up must share shape, strides and dtype")
    h = torch.empty((rows, k), device=gate.device, dtype=gate.dtype) if h is None else h
    q = torch.empty((rows, k), device=gate.device, dtype=torch.int8) if q is None else q
    sx = torch.empty(((k + 63) // 64,), device=gate.device, dtype=torch.float32) if sx is None else sx
    lib = N.load()
    N.check(lib.tq_silu_mul_quant(gate.data_ptr(), up.data_ptr(), gate.stride(0), rows, k, h.data_ptr(), h.stride(0),
                                  q.data_ptr(), q.stride(0), sx.data_ptr(), N.dtype_code(gate.dtype),
                                  N.stream_of(gate)), "silu_mul_quant")
    return h, q, sx


def attn_decode_splits(batch: int, kv_heads: int, max_len: int, device: torch.device) -> int:
    with torch.cuda.device(device):
        return int(N.load().tq_attn_decode_splits(int(batch), int(kv_heads), int(max_len)))


class AttnWorkspace:
    """Split partials of ``attn_decode`` for one (batch, query heads, head_dim, splits)."""

    def __init__(self, batch: int, q_heads: int, head_dim: int, splits: int, device: torch.device):
        self.splits = int(splits)
        n = batch * q_heads * self.splits
        self.m = torch.empty(n, device=device, dtype=torch.float32)
        self.l = torch.empty(n, device=device, dtype=torch.float32)
        self.o = torch.empty(n * head_dim, device=device, dtype=torch.float32)
        self.err = torch.zeros(1, device=device, dtype=torch.int32)


def attn_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                k_cache: torch.Tensor, v_cache: torch.Tensor, position: torch.Tensor, scale: float,
                ws: AttnWorkspace, out: Optional[torch.Tensor] = None, q_out: Optional[torch.Tensor] = None,
                sx: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention of one new token per sequence (q/k/v: [B, heads * D] views, unrotated)
    over cache slots [0, position]: RoPE with ``cos``/``sin`` ([D] of the position), the
    token's K/V written into slot ``position``, output [B, Hq * D]; with ``q_out``/``sx``
    also its INT8 codes and tile scales."""
    N.require_cuda(q, k, v, cos, sin, k_cache, v_cache, position, out, q_out, sx)
    B, Hkv, L, D = k_cache.shape
    if v_cache.shape != k_cache.shape or not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("attn_decode: K and V caches must be contiguous [B, Hkv, L, D] tensors")
    for t in (q, k, v):
        if t.dim() != 2 or t.shape[0] != B or t.stride(1) != 1 or t.dtype != k_cache.dtype:
            raise ValueError("attn_decode: q/k/v must be [B, heads * D] with unit column stride")
    Hq = q.shape[1] // D
    if q.shape[1] != Hq * D or k.shape[1] != Hkv * D or v.shape[1] != Hkv * D:
        raise ValueError("attn_decode: q/k/v widths do not match the cache's heads")
    if cos.numel() != D or sin.numel() != D or position.dtype != torch.int64:
        raise ValueError("attn_decode: cos/sin need head_dim values, position an int64 tensor")
    if ws.m.numel() < B * Hq * ws.splits or ws.o.numel() < B * Hq * ws.splits * D:
        raise ValueError("attn_decode: workspace too small")
    out = torch.empty((B, Hq * D), device=q.device, dtype=q.dtype) if out is None else out
    a = N.AttnArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), cos=cos.data_ptr(), sin=sin.data_ptr(),
                   k_cache=k_cache.data_ptr(), v_cache=v_cache.data_ptr(), pos=position.data_ptr(),
                   ws_m=ws.m.data_ptr(), ws_l=ws.l.data_ptr(), ws_o=ws.o.data_ptr(), err=ws.err.data_ptr(),
                   ld_q=q.stride(0), ld_k=k.stride(0), ld_v=v.stride(0), B=B, Hq=Hq, Hkv=Hkv, D=D, L=L,
                   S=ws.splits, scale_log2=float(scale) * math.log2(math.e), reserved=0)
    lib = N.load()
    N.check(lib.tq_attn_decode(ctypes.byref(a), out.data_ptr(), out.stride(0), N.ptr(q_out),
                               0 if q_out is None else q_out.stride(0), N.ptr(sx), N.dtype_code(q.dtype),
                               N.stream_of(q)), "attn_decode")
    return out


def greedy_pick(logits: torch.Tensor, keys: torch.Tensor, position: torch.Tensor, prompt_tokens: int,
                next_ids: Optional[torch.Tensor] = None, token: Optional[torch.Tensor] = None,
                generated: Optional[torch.Tensor] = None) -> None:
    """The greedy decode step's pick and bookkeeping in two kernels: argmax of every row
    of ``logits`` [B, V] (first index of the maximum, as ``torch.argmax``) into
    ``next_ids`` and ``token`` ([B, 1] int64), into ``generated[:, position - prompt + 1]``,
    then ``position += 1``.  ``keys``: [B] int64 scratch, zero before the first call and
    left zero by every call."""
    N.require_cuda(logits, keys, position, next_ids, token, generated)
    B, V = logits.shape
    if logits.stride(1) != 1 or keys.dtype != torch.int64 or keys.numel() < B or position.dtype != torch.int64:
        raise ValueError("greedy_pick: unit-stride logits, int64 keys and position")
    for t in (next_ids, token):
        if t is not None and (t.dtype != torch.int64 or t.numel() != B or not t.is_contiguous()):
            raise ValueError("greedy_pick: next/token must be contiguous int64 [B] tensors")
    if generated is not None and (generated.dtype != torch.int64 or generated.shape[0] != B or generated.stride(1) != 1):
        raise ValueError("greedy_pick: generated must be int64 [B, T] with unit column stride")
    lib = N.load()
    N.check(lib.tq_greedy_pick(logits.data_ptr(), logits.stride(0), B, V, N.dtype_code(logits.dtype), keys.data_ptr(),
                               N.ptr(next_ids), N.ptr(token), N.ptr(generated),
                               0 if generated is None else generated.stride(0),
                               0 if generated is None else generated.shape[1], position.data_ptr(), int(prompt_tokens),
                               N.stream_of(logits)), "greedy_pick")


def _proj(mod: nn.Module, x: torch.Tensor, q: Optional[torch.Tensor] = None,
          sx: Optional[torch.Tensor] = None) -> torch.Tensor:
    """A projection of 2-D activations; a plain MixedLinear takes the given codes."""
    if q is not None and type(mod) is MixedLinear:
        return mod._launch(x, q, sx)
    return mod(x)


class _Layer:
    """The modules and shapes of one decoder layer, resolved once."""

    def __init__(self, layer: nn.Module, cache_layer, dtype: torch.dtype):
        attn, mlp = layer.self_attn, layer.mlp
        self.norm1, self.norm2 = layer.input_layernorm, layer.post_attention_layernorm
        self.eps1, self.eps2 = float(self.norm1.variance_epsilon), float(self.norm2.variance_epsilon)
        self.D = int(attn.head_dim)
        self.scale = float(attn.scaling)
        qkv = getattr(attn, "tilequant_qkv", None)
        self.qkv = qkv.linear if isinstance(qkv, MixedLinearGroup) else None
        self.q_proj, self.k_proj, self.v_proj, self.o_proj = attn.q_proj, attn.k_proj, attn.v_proj, attn.o_proj
        gu = getattr(mlp, "tilequant_gate_up", None)
        self.gate_up = gu.linear if isinstance(gu, MixedLinearGroup) else None
        self.gate_proj, self.up_proj, self.down_proj = mlp.gate_proj, mlp.up_proj, mlp.down_proj
        self.k_cache, self.v_cache = cache_layer.keys, cache_layer.values
        _, self.Hkv, self.L, D = self.k_cache.shape
        if D != self.D or not (self.k_cache.is_contiguous() and self.v_cache.is_contiguous()):
            raise ValueError("the KV cache is not a contiguous head-major [B, Hkv, L, D] tensor")
        self.Hq = int(self.q_proj.out_features) // self.D
        self.inter = int(self.gate_proj.out_features)
        for m in (self.qkv, self.gate_up, self.q_proj, self.o_proj, self.down_proj):
            if type(m) is MixedLinear and m._out_dtype() != dtype:
                raise ValueError("MixedLinear output dtype differs from the model's")


class FusedDecodeStep:
    """``step(token [B, 1] int64, position [1] int64) -> logits [B, 1, vocab]`` for a
    decoder whose KV cache (``cache``) holds the first ``position`` tokens."""

    @staticmethod
    def unsupported_reason(model: nn.Module) -> Optional[str]:
        cfg = model.config.get_text_config(decoder=True)
        if getattr(cfg, "model_type", None) not in SUPPORTED_MODEL_TYPES:
            return f"model type {getattr(cfg, 'model_type', None)!r} (supported: {', '.join(SUPPORTED_MODEL_TYPES)})"
        if getattr(cfg, "hidden_act", None) not in ("silu", "swish"):
            return f"activation {getattr(cfg, 'hidden_act', None)!r}"
        inner = getattr(model, "model", None)
        for name in ("embed_tokens", "layers", "norm", "rotary_emb"):
            if not hasattr(inner, name):
                return f"no {name}"
        if not hasattr(model, "lm_head"):
            return "no lm_head"
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        if head_dim not in (64, 128):
            return f"head_dim {head_dim}"
        if cfg.num_attention_heads // cfg.num_key_value_heads > 8:
            return "more than 8 query heads per KV head"
        if cfg.hidden_size % 8:
            return "hidden size not a multiple of 8"
        return None

    def __init__(self, model: nn.Module, cache, batch_size: int, device: torch.device):
        reason = self.unsupported_reason(model)
        if reason:
            raise ValueError(f"FusedDecodeStep: unsupported model: {reason}")
        if not 1 <= batch_size <= 64:
            raise ValueError("FusedDecodeStep: batch size must be in 1..64")
        self.model = model
        inner = model.model
        self.dtype = inner.embed_tokens.weight.dtype
        if self.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("FusedDecodeStep: the model must be in float16 or bfloat16")
        if len(cache.layers) < len(inner.layers):
            raise ValueError("FusedDecodeStep: the cache has fewer layers than the model")
        self.layers: List[_Layer] = [_Layer(layer, cl, self.dtype) for layer, cl in zip(inner.layers, cache.layers)]
        B, H = int(batch_size), int(inner.embed_tokens.weight.shape[1])
        first = self.layers[0]
        if first.k_cache.shape[0] != B:
            raise ValueError("FusedDecodeStep: cache batch differs from batch_size")
        self.batch, self.hidden = B, H
        dev = torch.device(device)
        splits = attn_decode_splits(B, first.Hkv, first.L, dev)
        self.ws = AttnWorkspace(B, max(l.Hq for l in self.layers), max(l.D for l in self.layers), splits, dev)
        width = max(l.Hq * l.D for l in self.layers)
        self.resid = torch.empty((B, H), device=dev, dtype=self.dtype)
        self.x = torch.empty((B, H), device=dev, dtype=self.dtype)
        self.attn = torch.empty((B, width), device=dev, dtype=self.dtype)
        self.attn_q = torch.empty((B, width), device=dev, dtype=torch.int8)
        self.attn_sx = torch.empty((width // 64,), device=dev, dtype=torch.float32)
        inter = max(l.inter for l in self.layers)
        self.h = torch.empty((B, inter), device=dev, dtype=self.dtype)
        self.h_q = torch.empty((B, inter), device=dev, dtype=torch.int8)
        self.h_sx = torch.empty(((inter + 63) // 64,), device=dev, dtype=torch.float32)

    def _norm(self, resid, delta, weight, eps):
        """The layer input: residual add (with delta) and RMSNorm."""
        return add_rmsnorm(resid, delta, weight, eps, resid_out=self.resid, out=self.x), None, None

    def status(self) -> int:
        """The attention kernel's error word (0, or TQ_ERR_TIMEOUT); synchronises."""
        return int(self.ws.err.item())

    def reset_status(self) -> None:
        """Clear the attention kernel's error word (stream-ordered)."""
        self.ws.err.zero_()

    @traced("tq.FusedDecodeStep")
    @torch.inference_mode()
    def __call__(self, token: torch.Tensor, position: torch.Tensor) -> torch.Tensor:
        inner = self.model.model
        B = self.batch
        emb = inner.embed_tokens(token).reshape(B, self.hidden)
        cos, sin = inner.rotary_emb(emb, position.view(1, 1))
        cos, sin = cos.reshape(-1), sin.reshape(-1)
        resid, delta = emb, None
        for L in self.layers:
            # residual add (from the second layer on) + input RMSNorm (+ the QKV input's codes)
            x, xq, xsx = self._norm(resid, delta, L.norm1.weight, L.eps1)
            resid = self.resid if delta is not None else resid
            qd, kd = L.Hq * L.D, L.Hkv * L.D
            if L.qkv is not None:
                y = _proj(L.qkv, x, xq, xsx)
                q, k, v = y[:, :qd], y[:, qd:qd + kd], y[:, qd + kd:qd + 2 * kd]
            else:
                q, k, v = _proj(L.q_proj, x), _proj(L.k_proj, x), _proj(L.v_proj, x)
            a_out, a_q, a_sx = self.attn[:, :qd], self.attn_q[:, :qd], self.attn_sx[:qd // 64]
            attn_decode(q, k, v, cos, sin, L.k_cache, L.v_cache, position, L.scale, self.ws, out=a_out, q_out=a_q,
                        sx=a_sx)
            delta = _proj(L.o_proj, a_out, a_q, a_sx)
            x, xq, xsx = self._norm(resid, delta, L.norm2.weight, L.eps2)
            resid = self.resid
            if L.gate_up is not None:
                gu = _proj(L.gate_up, x, xq, xsx)
                gate, up = gu[:, :L.inter], gu[:, L.inter:2 * L.inter]
            else:
                gate, up = _proj(L.gate_proj, x), _proj(L.up_proj, x)
                if gate.stride() != up.stride():
                    gate, up = gate.contiguous(), up.contiguous()
            h, h_q, h_sx = self.h[:, :L.inter], self.h_q[:, :L.inter], self.h_sx[:(L.inter + 63) // 64]
            silu_mul_quant(gate, up, h, h_q, h_sx)
            delta = _proj(L.down_proj, h, h_q, h_sx)
        x = add_rmsnorm(resid, delta, inner.norm.weight, float(inner.norm.variance_epsilon), resid_out=self.resid,
                        out=self.x)
        return self.model.lm_head(x).unsqueeze(1)
