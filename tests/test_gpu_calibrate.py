"""GI / IAA calibration on the GPU: the reduction kernels against the reference's own
outputs (tests/golden/calib.npz), the collectors against a torch FP32 restatement of
the reference's arithmetic, and checkpoint resume."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from tilequant_b200 import calibrate as C

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
CALIB = np.load(Path(__file__).resolve().parent / "golden" / "calib.npz")
TARGETS = sorted({k.split("__")[1] for k in CALIB.files if k.startswith("gi__")})


def _bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.float32).to(torch.bfloat16)


@pytest.mark.parametrize("name", TARGETS)
def test_gi_kernel_matches_reference(cuda_device, name):
    w = CALIB[f"gi__{name}__w"]
    m, k = w.shape
    scores = torch.zeros(((m + 63) // 64, (k + 63) // 64), device=DEV)
    wt = _bf16(w).to(DEV) if w.dtype != np.uint16 else torch.from_numpy(w.view(np.int16)).view(torch.bfloat16).to(DEV)
    for b in range(3):
        g = CALIB[f"gi__{name}__grad{b}"]
        gt = _bf16(g).to(DEV) if g.dtype != np.uint16 else torch.from_numpy(g.view(np.int16)).view(torch.bfloat16).to(DEV)
        C.gi_accumulate(scores, wt, gt)
    np.testing.assert_allclose(scores.cpu().numpy(), CALIB[f"gi__{name}__scores"], rtol=2e-5, atol=1e-30)


@pytest.mark.parametrize("name", TARGETS)
def test_iaa_kernels_match_reference(cuda_device, name):
    x = CALIB[f"iaa__{name}__x"]
    w = CALIB[f"gi__{name}__w"]
    tobf = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16) if a.dtype == np.uint16 else _bf16(a)  # noqa: E731
    xt, wt = tobf(x).to(DEV), tobf(w).to(DEV)
    acc = torch.zeros((x.shape[1],), dtype=torch.float64, device=DEV)
    rows = C.iaa_channel_accumulate(acc, xt)
    assert rows == x.shape[0]
    mean, scores = C.iaa_tile_scores(wt, acc, rows)
    np.testing.assert_array_equal(mean.cpu().numpy(), CALIB[f"iaa__{name}__mean"])
    np.testing.assert_allclose(scores.cpu().numpy(), CALIB[f"iaa__{name}__scores"], rtol=2e-5)


def _tiny(seed=0):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(hidden_size=256, intermediate_size=640, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=64, vocab_size=300, attn_implementation="sdpa")
    torch.manual_seed(seed)
    with torch.device(DEV):
        return LlamaForCausalLM(cfg).to(torch.bfloat16)


def _batches(n, seed=1):
    g = torch.Generator().manual_seed(seed)
    return [{"input_ids": torch.randint(0, 300, (2, 40), generator=g)} for _ in range(n)]


def _is_target(name):
    return name.endswith(("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"))


def _tile_sum(s):
    m, k = s.shape
    return torch.nn.functional.pad(s, (0, (-k) % 64, 0, (-m) % 64)).reshape(
        (m + 63) // 64, 64, (k + 63) // 64, 64).sum(dim=(1, 3))


def test_iaa_collector_matches_torch_restatement(cuda_device):
    model = _tiny()
    scores, stats = C.collect_iaa_tile_scores_with_channel_stats(model, _batches(3), _is_target, {"calib": {}})
    # restatement: f64 sum of |x| per channel over all rows, mean in f32, tile sums of |W| * mean
    sums, counts = {}, {}

    def hook(mod, inp, name):
        x2 = inp[0].reshape(-1, inp[0].shape[-1])
        sums[name] = sums.get(name, 0) + x2.double().abs().sum(0)
        counts[name] = counts.get(name, 0) + x2.shape[0]

    hooks = [m.register_forward_pre_hook(lambda mod, inp, n=n: hook(mod, inp, n)) for n, m in model.named_modules()
             if _is_target(n)]
    with torch.no_grad():
        for b in _batches(3):
            model(input_ids=b["input_ids"].to(DEV))
    for h in hooks:
        h.remove()
    assert set(scores) == set(sums) and len(scores) == 14
    for n, m in model.named_modules():
        if not _is_target(n):
            continue
        mean = (sums[n] / counts[n]).float()
        torch.testing.assert_close(stats[n], mean.cpu(), rtol=1e-6, atol=0)
        want = _tile_sum(m.weight.float().abs() * mean.view(1, -1)).cpu()
        torch.testing.assert_close(scores[n], want, rtol=2e-5, atol=1e-6)


def test_gi_collector_matches_torch_restatement(cuda_device):
    model = _tiny(1)
    got = C.collect_gi_tile_scores(model, _batches(2, 5), _is_target, {"calib": {}})
    want = {}
    for b in _batches(2, 5):
        model.zero_grad(set_to_none=True)
        ids = b["input_ids"].to(DEV)
        C._next_token_ce_loss(model(input_ids=ids), ids).backward()
        for n, m in model.named_modules():
            if _is_target(n):
                want[n] = want.get(n, 0) + _tile_sum((m.weight.float() * m.weight.grad.float()).abs())
    model.zero_grad(set_to_none=True)
    for n in want:
        torch.testing.assert_close(got[n], want[n].cpu(), rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("kind", ["gi", "iaa"])
def test_collectors_resume_from_checkpoint(cuda_device, tmp_path, kind):
    fn = C.collect_gi_tile_scores if kind == "gi" else C.collect_iaa_tile_scores
    full = fn(_tiny(2), _batches(4, 9), _is_target, {"calib": {}})
    part_cfg = {"calib": {"checkpoint_dir": str(tmp_path), "checkpoint_every_batches": 1, "num_samples": 2}}
    fn(_tiny(2), _batches(4, 9), _is_target, part_cfg)
    assert any(tmp_path.iterdir())
    resumed = fn(_tiny(2), _batches(4, 9), _is_target,
                 {"calib": {"checkpoint_dir": str(tmp_path), "resume_from_checkpoint": True}})
    for n in full:
        torch.testing.assert_close(resumed[n], full[n], rtol=1e-6, atol=0)
