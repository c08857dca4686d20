"""Observable behaviour of MixedLinear's work sharing on the GPU, counted with the
library's launch counter (every kernel this library starts):

* unstacked sibling projections (Q/K/V) fed the same activation quantize it once -- in
  inference mode, from 32 rows up -- and give the same bits as when each quantizes
  alone;
* below 32 rows, or outside inference mode, each quantizes for itself;
* a stacked group runs one quantization and one GEMM per activation, served to every
  member slice; a member asking again (a new forward on the same tensor) recomputes,
  and so does any member after the tensor changes in place.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

import tilequant_b200 as tq
from tilequant_b200 import _native as N
from tests.golden import inputs as I

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _cfg():
    return SimpleNamespace(tile_m=64, tile_n=64, pad_to_tile=True, quant_style="gi", dtype_out="bf16")


def _linear(m, k, seed):
    w = I.weight(m, k, seed).to(DEV)
    n_tr, n_tc = m // 64, k // 64
    keep = I.keep_ids(n_tr, n_tc, 0.1, seed + 1)
    p = tq.pack_weight_from_tile_ids(w, n_tr=n_tr, n_tc=n_tc, int8_tile_ids=I.complement_ids(keep, n_tr * n_tc),
                                     fp16_tile_ids=keep, cfg=_cfg())
    return tq.MixedLinear(p, None, _cfg())


def _launches(fn):
    torch.cuda.synchronize()
    n0 = N.kernel_launches()
    out = fn()
    torch.cuda.synchronize()
    return N.kernel_launches() - n0, out


def _siblings():
    return [_linear(256, 192, 10), _linear(128, 192, 20), _linear(128, 192, 30)]


@pytest.mark.parametrize("rows", [16, 64])
def test_siblings_share_one_quantization_from_32_rows(cuda_device, rows):
    mods = _siblings()
    x = I.activations(rows, 192, 40).to(DEV)
    q_launches = _launches(lambda: tq.quantize_activation_tile_absmax(x))[0]
    with torch.inference_mode():
        alone = [m(x.clone()) for m in mods]  # separate tensors: no sharing
        n, shared = _launches(lambda: [m(x) for m in mods])
    for a, b in zip(alone, shared):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    quantizations = 1 if rows >= 32 else 3
    assert n == 3 + quantizations * q_launches


def test_no_sharing_outside_inference_mode(cuda_device):
    mods = _siblings()
    x = I.activations(64, 192, 41).to(DEV)
    q_launches = _launches(lambda: tq.quantize_activation_tile_absmax(x))[0]
    with torch.no_grad():
        n, _ = _launches(lambda: [m(x) for m in mods])
    assert n == 3 + 3 * q_launches


def test_stacked_group_one_quantization_one_gemm(cuda_device):
    mods = _siblings()
    group = tq.MixedLinearGroup(mods)
    slices = [tq.MixedLinearSlice(group, i) for i in range(3)]
    x = I.activations(64, 192, 42).to(DEV)
    q_launches = _launches(lambda: tq.quantize_activation_tile_absmax(x))[0]
    with torch.inference_mode():
        separate = [m(x.clone()) for m in mods]
        n, outs = _launches(lambda: [s(x) for s in slices])
        assert n == q_launches + 1
        for a, b in zip(separate, outs):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16))
        # the next forward on the same tensor: every member is served again, once more
        n2, _ = _launches(lambda: [s(x) for s in slices])
        assert n2 == q_launches + 1
    # in-place change between members (outside inference mode the version counter moves)
    with torch.no_grad():
        y0 = slices[0](x)
        x.mul_(2.0)
        n3, y1 = _launches(lambda: slices[1](x))
        assert n3 == q_launches + 1
        assert not torch.equal(y1, outs[1])
    del y0
