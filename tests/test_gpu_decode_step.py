"""The fused decode-step kernels (csrc/decode_ops.cu) against the decoder's own torch
arithmetic, and the fused decode step against the transformers forward it replaces.

* add_rmsnorm: the residual add bit-exact; the normalised output equal to the torch
  RMSNorm's except where the f32 sum of squares, summed in another order, moves a
  rounding boundary of the normalised value (1 ulp, which the weight multiply can make
  2 ulps of the output), in well under 1 % of the outputs;
* silu_mul_quant: h bit-exact against torch's bf16/f16 silu then multiply, and its
  codes and scales bit-exact against the activation quantizer applied to h;
* attn_decode: the rotated K and the V of the new token in the cache bit-exact against
  the decoder's apply_rotary_pos_emb; the output within 2 % (relative to the largest
  output) of an f32 softmax attention over the valid prefix (the kernel rounds P to
  16 bits before P V, as flash attention does); its codes bit-exact against the
  quantizer applied to the output; slots past the position never read.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import tilequant_b200 as tq
from tilequant_b200.decode_step import AttnWorkspace, add_rmsnorm, attn_decode, attn_decode_splits, silu_mul_quant
from tests.helpers import greedy_steps, tracking

pytestmark = pytest.mark.gpu
DTYPES = [torch.bfloat16, torch.float16]


def _ulps(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    def ordered(t):
        i = t.contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
        return torch.where(i >= 0x8000, 0x8000 - i, i)

    return (ordered(a) - ordered(b)).abs()


def _torch_rmsnorm(h, w, eps):
    x = h.float()
    var = x.pow(2).mean(-1, keepdim=True)
    return w * (x * torch.rsqrt(var + eps)).to(h.dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,hidden", [(1, 256), (4, 3072), (16, 5120), (64, 3584)])
def test_add_rmsnorm_matches_torch(cuda_device, dtype, rows, hidden):
    g = torch.Generator(device=cuda_device).manual_seed(rows * 7 + hidden)
    resid = torch.randn(rows, hidden, device=cuda_device, generator=g).to(dtype)
    delta = (torch.randn(rows, hidden, device=cuda_device, generator=g) * 0.5).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, device=cuda_device, generator=g)).to(dtype)
    h_ref = resid + delta
    y_ref = _torch_rmsnorm(h_ref, w, 1e-5)
    out_resid = torch.empty_like(resid)
    y = add_rmsnorm(resid, delta, w, 1e-5, resid_out=out_resid)
    assert torch.equal(out_resid.view(torch.int16), h_ref.view(torch.int16))
    d = _ulps(y, y_ref)
    assert int(d.max()) <= 2 and float((d > 0).float().mean()) < 0.01
    # no delta: plain RMSNorm, residual untouched; in place on the residual
    y0 = add_rmsnorm(resid, None, w, 1e-5)
    assert int(_ulps(y0, _torch_rmsnorm(resid, w, 1e-5)).max()) <= 2
    r2 = resid.clone()
    add_rmsnorm(r2, delta, w, 1e-5, resid_out=r2)
    assert torch.equal(r2.view(torch.int16), h_ref.view(torch.int16))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,inter", [(1, 512), (4, 8192), (16, 18944), (128, 640), (3, 100)])
def test_silu_mul_quant_matches_torch_and_quantizer(cuda_device, dtype, rows, inter):
    g = torch.Generator(device=cuda_device).manual_seed(rows + inter)
    gu = (torch.randn(rows, 2 * inter, device=cuda_device, generator=g) * 3).to(dtype)
    gate, up = gu[:, :inter], gu[:, inter:]
    h_ref = F.silu(gate) * up
    h, q, sx = silu_mul_quant(gate, up)
    assert torch.equal(h.view(torch.int16), h_ref.view(torch.int16))
    q_ref, sx_ref = tq.quantize_activation_tile_absmax(h_ref.contiguous())
    assert torch.equal(sx, sx_ref)
    assert torch.equal(q, q_ref)


def _rope_torch(x, cos, sin):
    """The decoder's apply_rotary_pos_emb on [.., D] 16-bit tensors."""
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return (x * cos) + (rot * sin)


def _attn_case(dev, dtype, B, Hq, Hkv, D, L, pos, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    k_cache = torch.randn(B, Hkv, L, D, device=dev, generator=g).to(dtype)
    v_cache = torch.randn(B, Hkv, L, D, device=dev, generator=g).to(dtype)
    qkv = torch.randn(B, (Hq + 2 * Hkv) * D, device=dev, generator=g).to(dtype)
    ang = torch.rand(D // 2, device=dev, generator=g) * 6.28
    cos = torch.cat([ang.cos(), ang.cos()]).to(dtype)
    sin = torch.cat([ang.sin(), ang.sin()]).to(dtype)
    return k_cache, v_cache, qkv, cos, sin, torch.tensor([pos], device=dev, dtype=torch.int64)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("B,Hq,Hkv,D,L,pos,splits", [
    (4, 24, 8, 128, 2304, 2047, None),  # config 3 (Llama-3.2-3B), first decode step
    (4, 24, 8, 128, 2304, 2303, None),  # last slot
    (1, 4, 2, 64, 100, 0, None),        # the first token only
    (2, 28, 4, 128, 300, 64, 3),        # 7 query heads per KV head; pos at a chunk start
    (3, 8, 8, 64, 129, 63, 64),         # more splits than chunks (empty splits)
    (16, 40, 8, 128, 1280, 1100, None),  # Qwen2.5-14B heads, batch 16
    (2, 8, 1, 128, 4096, 3000, 1),      # one split over the whole prefix
])
def test_attn_decode_matches_f32_attention(cuda_device, dtype, B, Hq, Hkv, D, L, pos, splits):
    dev = cuda_device
    k_cache, v_cache, qkv, cos, sin, position = _attn_case(dev, dtype, B, Hq, Hkv, D, L, pos, B * 1000 + L)
    q, k, v = qkv[:, :Hq * D], qkv[:, Hq * D:(Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:]
    # the reference: the decoder's RoPE in 16-bit ops, cache update, f32 softmax attention
    q_rot = _rope_torch(q.view(B, Hq, D), cos, sin)
    k_rot = _rope_torch(k.view(B, Hkv, D), cos, sin)
    kc_ref, vc_ref = k_cache.clone(), v_cache.clone()
    kc_ref[:, :, pos] = k_rot
    vc_ref[:, :, pos] = v.view(B, Hkv, D)
    rep = Hq // Hkv
    kk = kc_ref[:, :, :pos + 1].float().repeat_interleave(rep, dim=1)
    vv = vc_ref[:, :, :pos + 1].float().repeat_interleave(rep, dim=1)
    scale = D ** -0.5
    p = torch.softmax(torch.einsum("bhd,bhsd->bhs", q_rot.float(), kk) * scale, dim=-1)
    ref = torch.einsum("bhs,bhsd->bhd", p, vv).reshape(B, Hq * D)

    # slots past pos hold garbage that must not be read
    k_cache[:, :, pos + 1:] = float("nan")
    v_cache[:, :, pos + 1:] = float("nan")
    S = splits or attn_decode_splits(B, Hkv, L, dev)
    ws = AttnWorkspace(B, Hq, D, S, dev)
    q_out = torch.empty(B, Hq * D, device=dev, dtype=torch.int8)
    sx = torch.empty(Hq * D // 64, device=dev, dtype=torch.float32)
    out = attn_decode(q, k, v, cos, sin, k_cache, v_cache, position, scale, ws, q_out=q_out, sx=sx)
    torch.cuda.synchronize()
    assert int(ws.err.item()) == 0
    assert torch.equal(k_cache[:, :, pos].view(torch.int16), k_rot.view(torch.int16))
    assert torch.equal(v_cache[:, :, pos].view(torch.int16), v.view(B, Hkv, D).view(torch.int16))
    assert torch.equal(k_cache[:, :, :pos].view(torch.int16), kc_ref[:, :, :pos].view(torch.int16))
    assert torch.isfinite(out.float()).all()
    err = float((out.float() - ref).abs().max() / ref.abs().max())
    assert err < 2e-2, err
    q_ref, sx_ref = tq.quantize_activation_tile_absmax(out)
    assert torch.equal(sx, sx_ref) and torch.equal(q_out, q_ref)


def test_attn_decode_in_cuda_graph_follows_position(cuda_device):
    """One captured launch serves successive positions: the position is read on the
    device at every replay."""
    dev, dtype = cuda_device, torch.bfloat16
    B, Hq, Hkv, D, L = 2, 8, 2, 128, 512
    k_cache, v_cache, qkv, cos, sin, position = _attn_case(dev, dtype, B, Hq, Hkv, D, L, 100, 5)
    q, k, v = qkv[:, :Hq * D], qkv[:, Hq * D:(Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:]
    ws = AttnWorkspace(B, Hq, D, attn_decode_splits(B, Hkv, L, dev), dev)
    out = torch.empty(B, Hq * D, device=dev, dtype=dtype)
    attn_decode(q, k, v, cos, sin, k_cache, v_cache, position, D ** -0.5, ws, out=out)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        attn_decode(q, k, v, cos, sin, k_cache, v_cache, position, D ** -0.5, ws, out=out)
    for p in (101, 300, 511):
        position.fill_(p)
        graph.replay()
        want = torch.empty_like(out)
        k2, v2 = k_cache.clone(), v_cache.clone()
        attn_decode(q, k, v, cos, sin, k2, v2, position, D ** -0.5, ws, out=want)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), want.view(torch.int16)), p
        assert torch.equal(k_cache[:, :, p].view(torch.int16), k2[:, :, p].view(torch.int16))


# ------------------------------------------------------------------ the whole step

@pytest.mark.parametrize("arch", ["llama", "qwen2"])
def test_fused_step_tracks_transformers_forward(cuda_device, arch):
    """The graph decoder with the fused step against the same decoder running the
    transformers forward (masked SDPA over the static cache) for 32 steps, teacher-forced
    on the latter's tokens: the logits stay within 6 % of their scale (the attention's
    summation order and the RMSNorm's, amplified by the INT8 re-quantization of every
    projection input as in the CPU/GPU comparison of the token tests) and the picks agree
    wherever the transformers path's top-1 leads by at least 32 FP16 ulps."""
    from tests.golden import tiny_models as T
    from tilequant_b200.apply import apply_random_tile_maps, default_cfg
    from tilequant_b200.graph_decode import CudaGraphGreedyDecoder

    spec = dict(T.MODELS[arch])
    model = T.build(dict(spec, seed=31)).to(cuda_device)
    apply_random_tile_maps(model, 0.1, seed=4, model_type=spec["arch"], cfg=default_cfg(dtype_out="fp16"))
    prompt = torch.randint(0, spec["vocab"], (4, 40), generator=torch.Generator().manual_seed(3))
    dec = CudaGraphGreedyDecoder.prepare(model, prompt_tokens=40, max_new_tokens=4, batch_size=4, device=cuda_device)
    assert dec._step is not None, "the fused step was not used"
    dec.close()
    hf, hf_logits = greedy_steps(model, prompt, cuda_device, 32, eager=False, fused_decode=False)
    _, ours = greedy_steps(model, prompt, cuda_device, 32, eager=False, forced=hf)
    drift, sure, bad, agree = tracking(hf, hf_logits, ours)
    print(f"{arch}: drift {drift:.4f}, steps with a sure pick {sure:.2f}, agree {agree:.3f}, differing picks {bad}")
    assert drift <= 0.06, drift
    assert sure >= 0.6, sure
    assert not bad, bad


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("B,V", [(1, 512), (4, 128256), (16, 152064), (3, 5000)])
def test_greedy_pick_matches_torch_argmax_and_bookkeeping(cuda_device, dtype, B, V):
    """argmax (first index of the maximum, ties included), the next token, the generated
    id at position - prompt + 1 and the advanced position, over three calls in a row
    (the scratch keys are left zero by each)."""
    from tilequant_b200.decode_step import greedy_pick

    g = torch.Generator(device=cuda_device).manual_seed(B + V)
    prompt, T = 10, 5
    keys = torch.zeros(B, dtype=torch.long, device=cuda_device)
    position = torch.tensor([prompt], dtype=torch.long, device=cuda_device)
    nxt = torch.zeros(B, 1, dtype=torch.long, device=cuda_device)
    tok = torch.zeros(B, 1, dtype=torch.long, device=cuda_device)
    gen = torch.full((B, T), -1, dtype=torch.long, device=cuda_device)
    for call in range(3):
        logits = (torch.randn(B, V, device=cuda_device, generator=g) * 4).to(dtype)
        logits[0, V // 3] = logits[0, V // 2] = logits[0].max() + 1  # a tie: the first index wins
        if B > 1:
            logits[1] = -logits[1].abs()  # an all-negative row
        want = logits.argmax(dim=-1)
        greedy_pick(logits, keys, position, prompt, nxt, tok, gen)
        torch.cuda.synchronize()
        assert torch.equal(nxt.view(-1), want) and torch.equal(tok.view(-1), want), call
        assert int(want[0]) == V // 3
        assert torch.equal(gen[:, call + 1], want), call
        assert int(position.item()) == prompt + call + 1
        assert int(keys.abs().sum().item()) == 0
