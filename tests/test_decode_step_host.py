"""Host-side checks of the fused decode step (CPU, no kernel launches): which decoders
``FusedDecodeStep`` takes, how it resolves a layer's modules and KV cache, the errors
it raises before touching a GPU, and that every decode-step operator refuses CPU
tensors instead of computing on the host."""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from tilequant_b200 import decode_step as D


def _llama(**kw):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
               num_key_value_heads=2, head_dim=64, vocab_size=128)
    cfg.update(kw)
    torch.manual_seed(0)
    return LlamaForCausalLM(LlamaConfig(**cfg)).to(torch.bfloat16).eval()


def _qwen2(**kw):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
               num_key_value_heads=2, vocab_size=128)
    cfg.update(kw)
    torch.manual_seed(0)
    return Qwen2ForCausalLM(Qwen2Config(**cfg)).to(torch.bfloat16).eval()


def _cache(model, batch=2, max_len=32, dtype=torch.bfloat16, contiguous=True):
    cfg = model.config
    hd = cfg.head_dim if getattr(cfg, "head_dim", None) else cfg.hidden_size // cfg.num_attention_heads
    layers = []
    for _ in range(cfg.num_hidden_layers):
        if contiguous:
            k = torch.zeros(batch, cfg.num_key_value_heads, max_len, hd, dtype=dtype)
        else:  # token-major storage seen through a head-major view
            k = torch.zeros(batch, max_len, cfg.num_key_value_heads, hd, dtype=dtype).transpose(1, 2)
        layers.append(SimpleNamespace(keys=k, values=k.clone() if contiguous else k))
    return SimpleNamespace(layers=layers)


def test_llama_and_qwen2_decoders_are_supported():
    assert D.FusedDecodeStep.unsupported_reason(_llama()) is None
    assert D.FusedDecodeStep.unsupported_reason(_qwen2()) is None
    assert D.FusedDecodeStep.unsupported_reason(_llama(head_dim=128, num_attention_heads=2)) is None


@pytest.mark.parametrize("kw,needle", [
    (dict(head_dim=32, num_attention_heads=8), "head_dim 32"),
    (dict(hidden_act="gelu"), "activation"),
    (dict(num_attention_heads=16, num_key_value_heads=1, head_dim=64), "more than 8 query heads"),
])
def test_unsupported_decoders_are_named(kw, needle):
    reason = D.FusedDecodeStep.unsupported_reason(_llama(**kw))
    assert reason is not None and needle in reason
    with pytest.raises(ValueError, match="unsupported model"):
        D.FusedDecodeStep(_llama(**kw), _cache(_llama()), 2, torch.device("cpu"))


def test_other_architectures_are_refused_by_type():
    from transformers import GPT2Config, GPT2LMHeadModel

    model = GPT2LMHeadModel(GPT2Config(n_embd=64, n_layer=1, n_head=2, vocab_size=64))
    reason = D.FusedDecodeStep.unsupported_reason(model)
    assert reason is not None and "gpt2" in reason


def test_layer_resolution_reads_shapes_from_modules_and_cache():
    model = _qwen2()
    cache = _cache(model, batch=3, max_len=40)
    layer = D._Layer(model.model.layers[0], cache.layers[0], torch.bfloat16)
    assert (layer.Hq, layer.Hkv, layer.L, layer.D, layer.inter) == (4, 2, 40, 64, 512)
    assert layer.qkv is None and layer.gate_up is None  # plain nn.Linear projections
    assert layer.scale == pytest.approx(64 ** -0.5)
    assert layer.eps1 == pytest.approx(model.config.rms_norm_eps)


def test_layer_resolution_rejects_a_token_major_cache():
    model = _llama()
    with pytest.raises(ValueError, match="head-major"):
        D._Layer(model.model.layers[0], _cache(model, contiguous=False).layers[0], torch.bfloat16)


def test_step_construction_errors_come_before_any_device_work():
    model = _llama()
    with pytest.raises(ValueError, match="batch size"):
        D.FusedDecodeStep(model, _cache(model), 0, torch.device("cpu"))
    with pytest.raises(ValueError, match="float16 or bfloat16"):
        D.FusedDecodeStep(_llama().float(), _cache(model), 2, torch.device("cpu"))
    short = _cache(model)
    short.layers = short.layers[:1]
    with pytest.raises(ValueError, match="fewer layers"):
        D.FusedDecodeStep(model, short, 2, torch.device("cpu"))
    with pytest.raises(ValueError, match="cache batch"):
        D.FusedDecodeStep(model, _cache(model, batch=3), 2, torch.device("cpu"))


def test_operators_refuse_cpu_tensors():
    x = torch.zeros(2, 256, dtype=torch.bfloat16)
    w = torch.ones(256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="no CPU path"):
        D.add_rmsnorm(x, None, w, 1e-6)
    with pytest.raises(ValueError, match="no CPU path"):
        D.silu_mul_quant(x, x)
    cache = torch.zeros(2, 2, 16, 64, dtype=torch.bfloat16)
    ws = SimpleNamespace(m=torch.zeros(1), l=torch.zeros(1), o=torch.zeros(1), err=torch.zeros(1), splits=1)
    pos = torch.zeros(1, dtype=torch.int64)
    cs = torch.zeros(64)
    with pytest.raises(ValueError, match="no CPU path"):
        D.attn_decode(x[:, :256], x[:, :128], x[:, :128], cs, cs, cache, cache.clone(), pos, 0.125, ws)
    with pytest.raises(ValueError, match="no CPU path"):
        D.greedy_pick(torch.zeros(2, 128), torch.zeros(2, dtype=torch.int64), pos, 16)
