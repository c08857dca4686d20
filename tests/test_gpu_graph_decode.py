"""CUDA-graph greedy decoding over MixedLinear projections (a small Llama-architecture
model with random weights and random 64x64 tile maps)."""

from __future__ import annotations

import pytest
import torch

import tilequant_b200 as tq
from tilequant_b200.apply import apply_random_tile_maps
from tilequant_b200.graph_decode import CudaGraphGreedyDecoder

DEV = "cuda:0"


def _tiny_llama(seed=0, layers=2, tie=True):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(hidden_size=256, intermediate_size=640, num_hidden_layers=layers, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=64, vocab_size=1000, max_position_embeddings=1024,
                      rope_theta=500000.0, tie_word_embeddings=tie, attn_implementation="sdpa")
    torch.manual_seed(seed)
    with torch.device(DEV):
        model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    return model


@pytest.mark.gpu
def test_projections_become_mixed_linear(cuda_device):
    model = _tiny_llama()
    swapped = apply_random_tile_maps(model, 0.1, seed=3)
    assert len(swapped) == 2 * 7
    n_mixed = sum(isinstance(m, (tq.MixedLinear, tq.MixedLinearSlice)) for m in model.modules())
    assert n_mixed >= 2 * 7
    ids = torch.randint(0, 1000, (2, 24), device=DEV)
    with torch.inference_mode():
        logits = model(input_ids=ids).logits
    assert torch.isfinite(logits.float()).all()


@pytest.mark.gpu
@pytest.mark.parametrize("batch,prompt,new", [(1, 16, 40), (3, 33, 35)])
def test_graph_decode_matches_eager_bodies(cuda_device, batch, prompt, new):
    """Replaying the captured graphs gives the same greedy tokens (and logits) as running
    the same prefill/decode bodies eagerly, for the first 32+ steps."""
    model = _tiny_llama(seed=batch)
    apply_random_tile_maps(model, 0.05, seed=7)
    gen = torch.Generator().manual_seed(11)
    ids = torch.randint(0, 1000, (batch, prompt), generator=gen)
    eager = CudaGraphGreedyDecoder.prepare(model, prompt_tokens=prompt, max_new_tokens=new, batch_size=batch,
                                           device=DEV, eager=True)
    ref = eager.generate(ids).clone()
    ref_logits = eager.last_logits.clone()
    eager.close()
    graph = CudaGraphGreedyDecoder.prepare(model, prompt_tokens=prompt, max_new_tokens=new, batch_size=batch,
                                           device=DEV)
    assert graph._decode_graph is not None and graph.prefill_captured
    for _ in range(2):  # replays are independent requests
        out = graph.generate(ids).clone()
        assert out.shape == (batch, new)
        assert torch.equal(out, ref)
    assert torch.equal(graph.last_logits, ref_logits)
    ids2, timing = graph.generate_timed(ids, new_tokens=8)
    assert torch.equal(ids2, ref[:, :8]) and timing.ttft_ms > 0 and timing.decode_ms > 0
    graph.close()


@pytest.mark.gpu
def test_graph_decode_first_token_matches_plain_forward(cuda_device):
    """The first generated token is the argmax of an ordinary full forward."""
    model = _tiny_llama(seed=5)
    apply_random_tile_maps(model, 0.02, seed=9)
    ids = torch.randint(0, 1000, (2, 20), generator=torch.Generator().manual_seed(2))
    with torch.inference_mode():
        want = model(input_ids=ids.to(DEV)).logits[:, -1].argmax(-1)
    dec = CudaGraphGreedyDecoder.prepare(model, prompt_tokens=20, max_new_tokens=4, batch_size=2, device=DEV)
    first = dec.prefill(ids)
    assert torch.equal(first.view(-1), want)
    dec.close()


@pytest.mark.gpu
def test_decoder_argument_checks(cuda_device):
    model = _tiny_llama()
    with pytest.raises(ValueError):
        CudaGraphGreedyDecoder(model, prompt_tokens=0, max_new_tokens=4, device=DEV)
    dec = CudaGraphGreedyDecoder.prepare(model, prompt_tokens=8, max_new_tokens=4, device=DEV)
    with pytest.raises(ValueError):
        dec.prefill(torch.zeros((2, 8), dtype=torch.long))
    with pytest.raises(ValueError):
        dec.decode(9)
    with pytest.raises(RuntimeError):
        CudaGraphGreedyDecoder(model, prompt_tokens=8, max_new_tokens=4, device=DEV)  # already attached
    dec.close()
