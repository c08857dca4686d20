"""End-to-end greedy decoding: this repository's CUDA-graph decoder over its sm_100a
kernels, against the same model decoded with every projection computed by the
reference's arithmetic.

The reference arm: the same seeded tiny decoders (a Llama and a Qwen2 with Q/K/V bias,
``tests/golden/tiny_models.py``) and the same tile maps, each projection's GEMM computed
on the CPU by the restatement in ``oracle/`` -- pinned bit-exactly to the reference's own
quantizer and Triton kernel by ``tests/test_oracle_golden.py`` -- at the split and
rounding the reference kernel would use for that call (a fused multiply-add per INT8
tile at prefill, a multiply then an add at the split the decode kernels run), decoded
step by step by the same decoder (eager mode: the same attention, norms and LM head).

With every tile INT8 the arithmetic of the path is fully specified, so the two arms must
give bit-identical logits at every one of the 32 steps, and so identical tokens.  With
16-bit tiles the reference's BF16/FP16 tile dot has no fixed summation order (the kernel
hands it to the tensor cores), so a last-bit difference there is allowed; our decoder is
then teacher-forced on the reference arm's tokens and compared step by step where the
reference's top logit leads by more than the drift such bits leave.

(``tests/golden/tokens.npz`` also holds 32 greedy tokens and their logits from the
reference's own Python model path run on the CPU; ``test_reference_cpu_run_teacher_forced``
follows them.  There a CPU attention and a GPU attention differ in the last FP16 bit of
~16 % of their outputs, and every projection re-quantizes its input to INT8, which turns
such one-ulp differences into ~1 % output differences a layer later, so the picks are
compared where the reference's margin exceeds that drift.)
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import tilequant_b200 as tq
from tests.golden import tiny_models as T
from tests.helpers import greedy_steps, tracking
from oracle import oracle as O

pytestmark = pytest.mark.gpu
FIX = np.load(Path(__file__).resolve().parent / "golden" / "tokens.npz")


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


class OracleProjection(torch.nn.Module):
    """A MixedLinear's pack, multiplied by the CPU restatement of the reference (oracle/)
    at the split and rounding the GPU kernels use for the same row count."""

    def __init__(self, lin: tq.MixedLinear):
        super().__init__()
        self.lin = lin
        self.code = O.BF16 if lin._out_dtype() == torch.bfloat16 else O.F16
        self.pk = dict(n_tr=lin.n_tr, n_tc=lin.n_tc, int8_tiles=lin.int8_tiles.cpu().numpy(),
                       int8_scales=lin.int8_scales.cpu().numpy(), int8_tile_ids=lin.int8_tile_ids.cpu().numpy(),
                       int8_row_ptr=lin.int8_row_ptr.cpu().numpy(), fp16_tiles=_bits(lin.fp16_tiles),
                       fp16_tile_ids=lin.fp16_tile_ids.cpu().numpy(), fp16_row_ptr=lin.fp16_row_ptr.cpu().numpy())
        self.bias = None if lin.bias is None else _bits(lin.bias.to(lin._out_dtype()))

    def forward(self, x):
        lin = self.lin
        rows = x.reshape(-1, lin.K_orig)
        n = rows.shape[0]
        prefill = n > 64  # the tcgen05 kernel: split 1, one FMA per INT8 tile
        split = 1 if prefill else tq.select_split_k(n_tr=lin.n_tr, n_tc=lin.n_tc, n_rows=n, device=x.device)
        xb = _bits(rows)
        q, sx = O.quantize_act(xb, self.code)
        y = O.gemm(q, sx, self.pk, xb, lin.M_orig, lin.K_orig, split_k=split, bias_bits=self.bias, xdtype=self.code,
                   odtype=self.code, use_fma=prefill)
        out = torch.from_numpy(y.view(np.int16)).view(x.dtype).to(x.device)
        return out.reshape(*x.shape[:-1], lin.M_orig)


def _model(name, keep_frac, device, oracle: bool):
    from tilequant_b200.apply import apply_tile_maps, default_cfg

    spec = T.MODELS[name]
    model = T.build(spec)
    assert T.state_sha(model) == str(FIX[f"{name}__state_sha"]), "the seeded model differs from the fixture's"
    model = model.to(device)
    if keep_frac == 0:
        keep = lambda n, n_tr, n_tc: torch.zeros(0, dtype=torch.int32)  # noqa: E731
    else:
        prefix = f"{name}__keep__"
        keep = {k[len(prefix):]: torch.from_numpy(FIX[k]) for k in FIX.files if k.startswith(prefix)}
    apply_tile_maps(model, keep, default_cfg(dtype_out="fp16"), model_type=spec["arch"])
    if oracle:
        for parent in list(model.modules()):
            for attr, child in list(parent.named_children()):
                if isinstance(child, tq.MixedLinear):
                    setattr(parent, attr, OracleProjection(child))
    return model


def _decode(model, prompt, device, eager, forced=None):
    return greedy_steps(model, prompt, device, T.NEW_TOKENS, eager, forced)


@pytest.mark.parametrize("name", sorted(T.MODELS))
def test_int8_tiles_bit_identical_to_reference_arithmetic(cuda_device, name):
    prompt = torch.from_numpy(FIX[f"{name}__prompt"])
    ours, our_logits = _decode(_model(name, 0, cuda_device, oracle=False), prompt, cuda_device, eager=False)
    ref, ref_logits = _decode(_model(name, 0, cuda_device, oracle=True), prompt, cuda_device, eager=True)
    np.testing.assert_array_equal(ours, ref)
    assert torch.equal(our_logits.view(torch.int16), ref_logits.view(torch.int16))


@pytest.mark.parametrize("name", sorted(T.MODELS))
def test_mixed_tiles_track_reference_arithmetic(cuda_device, name):
    """10 % 16-bit tiles.  A single GEMM agrees with the oracle to 1 ulp in <2 % of its
    outputs (the 16-bit tile dot's order), but every projection re-quantizes its input
    to INT8, so such a bit moves whole quantization steps a layer later and the KV cache
    carries it forward: free-running, the two arms part at the first near-tie.  So our
    decoder is teacher-forced on the reference arm's tokens (same history at every step)
    and must keep its logits within 4 % of the logit scale of the reference's (measured
    <= 2.2 %) and pick the reference's token wherever the reference's top-1 leads by at
    least 32 FP16 ulps (measured: the picks differed only at leads of <= 9 ulps)."""
    prompt = torch.from_numpy(FIX[f"{name}__prompt"])
    ref, ref_logits = _decode(_model(name, 0.1, cuda_device, oracle=True), prompt, cuda_device, eager=True)
    _, our_logits = _decode(_model(name, 0.1, cuda_device, oracle=False), prompt, cuda_device, eager=False,
                            forced=ref)
    drift, sure, bad, agree = tracking(ref, ref_logits, our_logits)
    assert drift <= 0.04, drift
    assert sure >= 0.6, sure
    assert not bad, f"(prompt, step, reference lead in ulps) where the tokens differ: {bad}"


@pytest.mark.parametrize("name", sorted(T.MODELS))
def test_reference_cpu_run_teacher_forced(cuda_device, name):
    """Against the reference's own Python model path (run on the CPU to make the
    fixture), our decoder teacher-forced on the reference's 32 tokens: the logits stay
    within 6 % of the logit scale of the reference's (measured <= 5 %: the CPU/GPU
    attention and norm drift on top of the 16-bit tile bits), the picks agree at 95 % of
    the steps or more, and everywhere the reference's top-1 leads by at least 64 FP16
    ulps (about two thirds of the steps of these fixtures; the largest lead at which the
    picks were seen to differ was 52 ulps)."""
    prompt = torch.from_numpy(FIX[f"{name}__prompt"])
    ref, ref_logits = FIX[f"{name}__tokens"], torch.from_numpy(FIX[f"{name}__logits"])
    _, our_logits = _decode(_model(name, 0.1, cuda_device, oracle=False), prompt, cuda_device, eager=False,
                            forced=ref)
    drift, sure, bad, agree = tracking(ref, ref_logits, our_logits, sure_ulps=64)
    print(f"{name}: drift {drift:.4f}, sure {sure:.2f}, agree {agree:.3f}")
    assert drift <= 0.06, drift
    assert sure >= 0.5, sure
    assert agree >= 0.95, agree
    assert not bad, f"(prompt, step, reference lead in ulps) where the tokens differ: {bad}"
