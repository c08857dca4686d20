"""Comparison helpers shared by the tests (bit patterns, BF16 ulp distance)."""

from __future__ import annotations

import numpy as np


def ordered16(bits: np.ndarray) -> np.ndarray:
    """Map 16-bit float bit patterns to integers that are monotonic in value."""
    b = np.asarray(bits, np.uint16).astype(np.int32)
    return np.where(b & 0x8000, 0x8000 - b, b)


def ulp_dist16(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    return np.abs(ordered16(a_bits) - ordered16(b_bits))


def assert_within_ulp(a_bits, b_bits, ulp: int = 1, what: str = ""):
    d = ulp_dist16(a_bits, b_bits)
    worst = int(d.max()) if d.size else 0
    assert worst <= ulp, f"{what}: max BF16 ulp distance {worst} > {ulp} ({int((d > ulp).sum())} elements)"
    return d


def to_torch16(bits: np.ndarray, dtype, device=None):
    """uint16 bit pattern -> 16-bit float tensor (no value conversion)."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(dtype)
    return t.to(device) if device is not None else t


def from_torch16(t) -> np.ndarray:
    import torch

    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def f16bits_to_f32(bits, dtype_code: int = 0) -> np.ndarray:
    b = np.asarray(bits, np.uint16)
    if dtype_code == 0:
        return (b.astype(np.uint32) << 16).view(np.float32)
    return b.view(np.float16).astype(np.float32)


def ulp_bf16(v: np.ndarray) -> np.ndarray:
    """Size of one BF16 ulp at |v| (8 significant bits)."""
    a = np.maximum(np.abs(v).astype(np.float64), 1e-30)
    return np.exp2(np.floor(np.log2(a)) - 7)


def assert_close_with_bias(y_bits, ref_bits, bias_bits, what: str = "", dtype_code: int = 0):
    """Outputs with bias: out = round(f32(round(acc)) + bias) rounds twice, so one ulp
    of the pre-bias value can be many ulps of a cancelled sum.  Allowed error: one ulp
    of the pre-bias value plus one ulp of the result."""
    y = f16bits_to_f32(y_bits, dtype_code)
    r = f16bits_to_f32(ref_bits, dtype_code)
    b = f16bits_to_f32(bias_bits, dtype_code)[None, :]
    tol = ulp_bf16(r - b) + ulp_bf16(r)
    bad = np.abs(y - r) > tol
    assert not bad.any(), f"{what}: {int(bad.sum())} elements beyond one pre-bias ulp"


def assert_close_gemm(y_bits, ref_bits, what: str = "", rms_frac: float = 1e-3, dtype_code: int = 0):
    """GEMM outputs whose 16-bit tile dots were summed in another order: within one
    BF16 ulp of the reference, except near zero where cancellation makes ulps tiny;
    there the difference must stay below rms_frac of the output's RMS magnitude."""
    y = f16bits_to_f32(y_bits, dtype_code).astype(np.float64)
    r = f16bits_to_f32(ref_bits, dtype_code).astype(np.float64)
    rms = float(np.sqrt(np.mean(r * r))) if r.size else 0.0
    tol = np.maximum(ulp_bf16(r), rms_frac * rms)
    bad = np.abs(y - r) > tol
    if bad.any():
        idx = np.argwhere(bad)[:5]
        detail = ", ".join(f"{tuple(i)}: got {y[tuple(i)]:.6g} ref {r[tuple(i)]:.6g}" for i in idx)
        raise AssertionError(f"{what}: {int(bad.sum())} elements beyond tolerance (rms {rms:.4g}): {detail}")
    return np.abs(y - r)


def greedy_steps(model, prompt, device, new_tokens: int, eager: bool, forced=None, **prepare_kwargs):
    """Greedy decoding through CudaGraphGreedyDecoder: the prompt, then new_tokens - 1
    one-token steps.  With ``forced`` (ids [batch, new_tokens]) each step's input is the
    forced token instead of the decoder's own pick (teacher forcing), so two arms can be
    compared over the same history.  ``prepare_kwargs`` go to ``prepare``.  Returns (ids
    [batch, new_tokens] numpy, logits [batch, new_tokens, vocab] on the CPU)."""
    import torch

    from tilequant_b200.graph_decode import CudaGraphGreedyDecoder

    dec = CudaGraphGreedyDecoder.prepare(model, prompt_tokens=prompt.shape[1], max_new_tokens=new_tokens,
                                         batch_size=prompt.shape[0], device=device, eager=eager, **prepare_kwargs)
    logits = []
    try:
        dec.prefill(prompt)
        logits.append(dec.last_logits.reshape(prompt.shape[0], -1).clone())
        for step in range(new_tokens - 1):
            if forced is not None:
                with torch.inference_mode():
                    dec._token.copy_(torch.from_numpy(np.ascontiguousarray(forced[:, step:step + 1])).to(device))
            dec.decode(1)
            logits.append(dec.last_logits.reshape(prompt.shape[0], -1).clone())
        ids = dec._generated.clone()
    finally:
        dec.close()
    return ids.cpu().numpy(), torch.stack(logits, 1).cpu()


def tracking(ref_ids, ref_logits, our_logits, sure_ulps: float = 32):
    """How closely teacher-forced logits follow a reference run: the per-step drift
    max|ours - ref| / max|ref| (over prompts and vocabulary, worst step), the fraction of
    (prompt, step) whose reference top-1 leads by at least ``sure_ulps`` FP16 ulps, the
    (prompt, step, lead) of those where the two picks differ, and the fraction of all
    (prompt, step) where the picks agree."""
    from tests.golden.tiny_models import margin_ulps

    rl, ol = ref_logits.float(), our_logits.float()
    drift = (ol - rl).abs().amax(dim=(0, 2)) / rl.abs().amax(dim=(0, 2))
    margin = margin_ulps(rl.topk(2, dim=-1).values).numpy()
    sure = margin >= sure_ulps
    picks = ol.argmax(dim=-1).numpy()
    bad = [(int(r), int(t), float(margin[r, t])) for r, t in zip(*np.nonzero(sure & (picks != ref_ids)))]
    return float(drift.max()), float(sure.mean()), bad, float((picks == ref_ids).mean())
