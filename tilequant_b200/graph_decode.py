"""Fixed-shape CUDA-graph greedy decoding over a model whose projections are MixedLinear.

Same interface as the reference's ``CudaGraphGreedyDecoder``
(src/runtime/graph_decode.py:96-479): ``prepare`` (allocate the static KV cache, warm
up, capture), ``prefill`` (copy a prompt in, replay the reset-and-prefill graph,
return the first token), ``decode`` (replay the one-token graph ``steps`` times, return
a GPU view of the generated ids), ``generate``, ``generate_timed`` (synchronised
host timestamps: TTFT and decode time) and ``close``.

How the graphs are built here:

* one prefill graph and one decode graph per (batch, prompt, output) shape; the KV
  cache is a transformers ``StaticCache`` whose storage never moves, and the decode
  graph keeps the current token and position on the GPU, so replays need no host
  input at all;
* prefill runs the transformers forward with a registered attention function (causal
  SDPA over the prompt prefix of the cache) and the mixed tile GEMM kernels of this
  package (quantizer + tcgen05 kernel) for the projections;
* decode runs ``FusedDecodeStep`` (decode_step.py) for Llama/Qwen2 decoders: per layer
  a fused residual-add + RMSNorm, the QKV GEMM, one decode-attention kernel pair (RoPE,
  cache write, split-KV attention over the valid prefix only, the O projection's input
  quantization), the O GEMM, the second norm, the gate/up GEMM, SiLU * up with the down
  projection's input quantization and the down GEMM -- the reference's flash-attention
  decode (src/runtime/graph_decode.py:58-70) reads the valid prefix the same way.
  Other models (or ``fused_decode=False``) decode through the transformers forward with
  SDPA of the single query over the whole static cache and an additive mask built on
  the GPU from the position tensor;
* one replay launches exactly the kernels of one eager body.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Optional, Sequence, Union

import torch
import torch.nn.functional as F

from .trace import traced

_ATTENTION_NAME = "tilequant_b200_static_graph"
_DECODER_ATTRIBUTE = "_tilequant_b200_graph_decoder"
# Prompts of more tokens than this (batch x prompt) prefill eagerly into the cache: the
# launch overhead a graph removes is negligible there, and a captured prefill would
# keep all of its activations in the graph's memory pool.
MAX_CAPTURED_PREFILL_TOKENS = 16384


def _graph_attention(module, query, key, value, attention_mask, dropout: float = 0.0, scaling=None, **_):
    """query (B, H, q, D); key/value the layer's whole static cache (B, Hkv, L, D)."""
    dec = getattr(module, _DECODER_ATTRIBUTE)
    if dec._in_prefill:
        if query.shape[2] != dec.prompt_tokens:
            raise RuntimeError("captured prefill query length changed")
        p = dec.prompt_tokens
        out = F.scaled_dot_product_attention(query, key[:, :, :p], value[:, :, :p], is_causal=True, scale=scaling,
                                             enable_gqa=True)
    else:
        if query.shape[2] != 1:
            raise RuntimeError("captured decode takes one query token")
        out = F.scaled_dot_product_attention(query, key, value, attn_mask=dec._decode_mask, scale=scaling,
                                             enable_gqa=True)
    return out.transpose(1, 2).contiguous(), None


def _no_mask(*_, **__):
    return None


@dataclass(frozen=True)
class GreedyGenerationTiming:
    """Host timestamps around one synchronised fixed-length request."""

    start_s: float
    first_token_s: float
    end_s: float

    @property
    def ttft_ms(self) -> float:
        return (self.first_token_s - self.start_s) * 1e3

    @property
    def decode_ms(self) -> float:
        return (self.end_s - self.first_token_s) * 1e3


class CudaGraphGreedyDecoder:
    """Reusable fixed-batch greedy decoder over a ``StaticCache``.

    ``eager=True`` runs the same prefill/decode bodies without graphs (the same kernels
    in the same order), for checking the captured path.
    """

    def __init__(self, model: torch.nn.Module, *, prompt_tokens: int, max_new_tokens: int, batch_size: int = 1,
                 device: Union[torch.device, str] = "cuda", prefill_only: bool = False, eager: bool = False,
                 fused_decode: bool = True) -> None:
        from transformers import StaticCache

        if prompt_tokens < 1:
            raise ValueError("prompt_tokens must be positive")
        if batch_size < 1:
            raise ValueError("batch_size must be positive")
        if max_new_tokens < (0 if prefill_only else 1):
            raise ValueError(f"max_new_tokens must be at least {0 if prefill_only else 1}")
        self.model = model
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("CudaGraphGreedyDecoder requires a CUDA device")
        cfg = model.config.get_text_config(decoder=True)
        if model.training or getattr(cfg, "attention_dropout", 0.0) != 0.0:
            raise ValueError("CudaGraphGreedyDecoder requires eval-mode zero-dropout attention")
        if getattr(cfg, "sliding_window", None) is not None and getattr(cfg, "use_sliding_window", False):
            raise ValueError("CudaGraphGreedyDecoder requires full causal attention")
        if cfg.num_attention_heads % cfg.num_key_value_heads:
            raise ValueError("CudaGraphGreedyDecoder requires grouped-query attention")
        index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        devices = {(p.device.type, p.device.index) for p in model.parameters()}
        devices |= {(b.device.type, b.device.index) for b in model.buffers()}
        if devices != {("cuda", index)}:
            raise ValueError("CudaGraphGreedyDecoder requires a single-device CUDA model")
        self.prompt_tokens = int(prompt_tokens)
        self.batch_size = int(batch_size)
        self.max_new_tokens = int(max_new_tokens)
        self.max_cache_len = self.prompt_tokens + (0 if prefill_only else self.max_new_tokens)
        self._prefill_only = prefill_only
        self._eager = eager
        self._fused_decode = fused_decode
        self._step = None  # FusedDecodeStep, built once the prefill has allocated the cache
        self._pick_keys = None  # greedy_pick scratch of the fused step
        self.cache = StaticCache(config=model.config, max_cache_len=self.max_cache_len)
        self._in_prefill = True
        dev = self.device
        # graph inputs and outputs: fixed storage, never reassigned
        self._prompt = torch.zeros((self.batch_size, self.prompt_tokens), dtype=torch.long, device=dev)
        self._prefill_pos = torch.arange(self.prompt_tokens, dtype=torch.long, device=dev)
        self._slots = torch.arange(self.max_cache_len, dtype=torch.long, device=dev)
        self._decode_mask = torch.zeros((1, 1, 1, self.max_cache_len), dtype=self._dtype(), device=dev)
        self._token = torch.zeros((self.batch_size, 1), dtype=torch.long, device=dev)
        self._position = torch.zeros((1,), dtype=torch.long, device=dev)
        self._next = torch.zeros((self.batch_size, 1), dtype=torch.long, device=dev)
        self._generated = torch.zeros((self.batch_size, max(1, self.max_new_tokens)), dtype=torch.long, device=dev)
        self._prefill_graph: Optional[torch.cuda.CUDAGraph] = None
        self._decode_graph: Optional[torch.cuda.CUDAGraph] = None
        self._prefill_logits: Optional[torch.Tensor] = None
        self._decode_logits: Optional[torch.Tensor] = None
        self.last_logits: Optional[torch.Tensor] = None
        self.prefill_captured = False
        # kernels of this library in one replay of each graph (counted during capture)
        self.captured_launches = {"prefill": 0, "decode": 0}
        # peer-sum exchanges of tensor-parallel row-parallel projections: their error
        # words are read at the synchronised points (check_peer_status)
        self._exchanges = list({id(ex): ex for ex in (getattr(m, "exchange", None) for m in model.modules())
                                if ex is not None and hasattr(ex, "status")}.values())
        self._prepared = False
        self._attach()

    def _dtype(self) -> torch.dtype:
        for p in self.model.parameters():
            if p.is_floating_point():
                return p.dtype if p.dtype in (torch.float16, torch.bfloat16) else torch.bfloat16
        return torch.bfloat16

    # ------------------------------------------------------------------ binding
    def _attach(self) -> None:
        from transformers import AttentionInterface
        from transformers.masking_utils import AttentionMaskInterface

        AttentionInterface.register(_ATTENTION_NAME, _graph_attention)
        # the function reads no mask; transformers would otherwise build one, with host
        # synchronisation that graph capture forbids
        AttentionMaskInterface.register(_ATTENTION_NAME, _no_mask)
        mods = [m for m in self.model.modules() if hasattr(m, "num_key_value_groups") and hasattr(m, "layer_idx")]
        if not mods:
            raise ValueError("model has no compatible attention modules")
        if any(hasattr(m, _DECODER_ATTRIBUTE) for m in mods):
            raise RuntimeError("model already has a CudaGraphGreedyDecoder attached")
        self._previous_attention = getattr(self.model.config, "_attn_implementation", "sdpa") or "sdpa"
        for m in mods:
            setattr(m, _DECODER_ATTRIBUTE, self)
        self.model.set_attn_implementation(_ATTENTION_NAME)

    def close(self, attn_implementation: Optional[str] = None) -> None:
        """Detach from the model; release the graphs and the cache."""
        for m in self.model.modules():
            if getattr(m, _DECODER_ATTRIBUTE, None) is self:
                delattr(m, _DECODER_ATTRIBUTE)
        self.model.set_attn_implementation(attn_implementation or self._previous_attention)
        self._prefill_graph = self._decode_graph = None
        self._step = None
        self.cache = None
        self._prefill_logits = self._decode_logits = self.last_logits = None

    # ------------------------------------------------------------------ capture
    @classmethod
    @torch.inference_mode()
    def prepare(cls, model: torch.nn.Module, *, prompt_tokens: int = 128, max_new_tokens: int = 512,
                batch_size: int = 1, device: Union[torch.device, str] = "cuda", prefill_only: bool = False,
                eager: bool = False, fused_decode: bool = True) -> "CudaGraphGreedyDecoder":
        """Allocate, warm up and capture the prefill and decode graphs (outside any
        request timing)."""
        dec = cls(model, prompt_tokens=prompt_tokens, max_new_tokens=max_new_tokens, batch_size=batch_size,
                  device=device, prefill_only=prefill_only, eager=eager, fused_decode=fused_decode)
        try:
            dec._capture()
        except BaseException:
            dec.close()
            raise
        return dec

    @torch.inference_mode()
    def _capture(self) -> None:
        decode = not self._prefill_only and self.max_new_tokens > 1
        # eager warm-up: the cache's storage and every kernel's lazy state exist before capture
        self._prefill_body()
        if decode and self._fused_decode:
            from .decode_step import FusedDecodeStep

            if FusedDecodeStep.unsupported_reason(self.model) is None:
                self._step = FusedDecodeStep(self.model, self.cache, self.batch_size, self.device)
                self._pick_keys = torch.zeros(self.batch_size, dtype=torch.long, device=self.device)
        if decode:
            self._decode_body()
        torch.cuda.synchronize(self.device)
        if self._eager:
            self._prepared = True
            return
        torch.cuda.empty_cache()
        self.prefill_captured = self.batch_size * self.prompt_tokens <= MAX_CAPTURED_PREFILL_TOKENS
        from ._native import kernel_launches

        if self.prefill_captured:
            g = torch.cuda.CUDAGraph()
            n0 = kernel_launches()
            with torch.cuda.graph(g):
                self._prefill_body()
            self.captured_launches["prefill"] = kernel_launches() - n0
            self._prefill_graph = g
        else:
            self._prefill_body()
        if decode:
            g = torch.cuda.CUDAGraph()
            n0 = kernel_launches()
            with torch.cuda.graph(g):
                self._decode_body()
            self.captured_launches["decode"] = kernel_launches() - n0
            self._decode_graph = g
        torch.cuda.synchronize(self.device)
        self._prepared = True

    @torch.inference_mode()
    def _prefill_body(self) -> None:
        self._in_prefill = True
        self.cache.reset()
        if not self._prefill_only:
            self._generated.zero_()
            self._position.fill_(self.prompt_tokens)
        out = self.model(input_ids=self._prompt, attention_mask=None, position_ids=self._prefill_pos.view(1, -1),
                         past_key_values=self.cache, cache_position=self._prefill_pos, use_cache=True,
                         logits_to_keep=1)
        self._prefill_logits = out.logits
        if not self._prefill_only:
            self._token.copy_(out.logits[:, -1:].argmax(dim=-1))
            self._generated[:, :1].copy_(self._token)

    @torch.inference_mode()
    def _decode_body(self) -> None:
        self._in_prefill = False
        if self._step is not None:
            from .decode_step import greedy_pick

            self._decode_logits = self._step(self._token, self._position)
            # argmax + next token + generated ids + position, in two kernels
            greedy_pick(self._decode_logits.view(self.batch_size, -1), self._pick_keys, self._position,
                        self.prompt_tokens, self._next, self._token, self._generated)
            return
        else:
            # additive mask over the static cache: slots past the current position are hidden
            self._decode_mask.copy_(torch.where(self._slots <= self._position, 0.0, float("-inf"))
                                    .to(self._decode_mask.dtype).view(1, 1, 1, -1))
            out = self.model(input_ids=self._token, attention_mask=None, position_ids=self._position.view(1, 1),
                             past_key_values=self.cache, cache_position=self._position, use_cache=True,
                             logits_to_keep=1)
            self._decode_logits = out.logits
        self._next.copy_(self._decode_logits[:, -1:].argmax(dim=-1))
        # position P consumes generated token P - prompt and produces token P - prompt + 1
        idx = (self._position - self.prompt_tokens + 1).view(1, 1).expand(self.batch_size, 1)
        self._generated.scatter_(1, idx, self._next)
        self._token.copy_(self._next)
        self._position.add_(1)

    # ------------------------------------------------------------------ requests
    def _prompt_from(self, prompt_ids: Union[torch.Tensor, Sequence[int]]) -> torch.Tensor:
        prompt = prompt_ids.to(torch.long) if isinstance(prompt_ids, torch.Tensor) else torch.tensor(prompt_ids,
                                                                                                   dtype=torch.long)
        if prompt.ndim == 1:
            prompt = prompt.unsqueeze(0)
        if tuple(prompt.shape) != (self.batch_size, self.prompt_tokens):
            raise ValueError(f"expected {(self.batch_size, self.prompt_tokens)}, got {tuple(prompt.shape)}")
        return prompt

    @traced("tq.prefill")
    @torch.inference_mode()
    def prefill(self, prompt_ids: Union[torch.Tensor, Sequence[int]]) -> torch.Tensor:
        """Copy the prompt in, replay the reset-and-prefill graph; returns the first
        generated token (or, with ``prefill_only``, the last position's logits)."""
        if not self._prepared:
            raise RuntimeError("call CudaGraphGreedyDecoder.prepare() before prefill")
        prompt = self._prompt_from(prompt_ids)
        self._prompt.copy_(prompt, non_blocking=prompt.device.type == "cpu" and prompt.is_pinned())
        if self._prefill_graph is not None:
            self._prefill_graph.replay()
        else:
            self._prefill_body()
        self.last_logits = self._prefill_logits
        return self._prefill_logits if self._prefill_only else self._token

    @traced("tq.decode")
    @torch.inference_mode()
    def decode(self, steps: Optional[int] = None) -> torch.Tensor:
        """Replay the decode graph ``steps`` times (default: up to the prepared bound);
        returns a GPU view of the ids generated so far (overwritten by the next prefill)."""
        if not self._prepared:
            raise RuntimeError("call CudaGraphGreedyDecoder.prepare() before decoding")
        if self._prefill_only:
            raise RuntimeError("decode() is unavailable after prepare(prefill_only=True)")
        if steps is None:
            steps = self.max_new_tokens - 1
        if not 0 <= steps <= self.max_new_tokens - 1:
            raise ValueError(f"steps must be in [0, {self.max_new_tokens - 1}]")
        for _ in range(steps):
            if self._decode_graph is not None:
                self._decode_graph.replay()
            else:
                self._decode_body()
        if steps:
            self.last_logits = self._decode_logits
        return self._generated[:, : steps + 1]

    @torch.inference_mode()
    def generate(self, prompt_ids, *, new_tokens: Optional[int] = None) -> torch.Tensor:
        """One request; greedy ids on the GPU, without synchronising."""
        new_tokens = self.max_new_tokens if new_tokens is None else new_tokens
        if not 1 <= new_tokens <= self.max_new_tokens:
            raise ValueError(f"new_tokens must be in [1, {self.max_new_tokens}]")
        self.prefill(prompt_ids)
        return self.decode(new_tokens - 1)

    @torch.inference_mode()
    def generate_timed(self, prompt_ids, *, new_tokens: Optional[int] = None):
        """``generate`` with synchronised host timestamps (TTFT, decode time)."""
        new_tokens = self.max_new_tokens if new_tokens is None else new_tokens
        torch.cuda.synchronize(self.device)
        start = time.perf_counter()
        self.prefill(prompt_ids)
        torch.cuda.synchronize(self.device)
        first = time.perf_counter()
        ids = self.decode(new_tokens - 1)
        torch.cuda.synchronize(self.device)
        end = time.perf_counter()
        self.check_peer_status()
        self.check_step_status()
        return ids, GreedyGenerationTiming(start, first, end)

    def check_step_status(self) -> None:
        """Raise ``TileQuantError`` if a bounded wait of the fused decode step's attention
        kernel gave up (a chunk of the KV cache never reached shared memory, so that
        step's logits, and the ids after it, are undefined).  Reads the step's error word,
        which synchronises, and clears it; no-op without a fused step."""
        from ._native import TQ_OK, TileQuantError

        step = getattr(self, "_step", None)
        if step is None:
            return
        st = step.status()
        if st != TQ_OK:
            step.reset_status()
            raise TileQuantError(f"decode attention: a wait for a KV-cache chunk ran out (status {st}); the "
                                 "request's ids are undefined")

    def check_peer_status(self) -> None:
        """Raise ``TileQuantError`` if a row-parallel peer sum of the model gave up
        waiting for a peer (its outputs, and so the generated ids, are then undefined;
        every rank must reset its exchange before the next request).  Reads each
        exchange's error word, which synchronises; no-op without exchanges."""
        from ._native import TQ_OK, TileQuantError

        for ex in self._exchanges:
            st = ex.status()
            if st != TQ_OK:
                raise TileQuantError(f"peer sum: a wait for a peer rank ran out (status {st}); reset the exchange "
                                     "on every rank before the next request")
