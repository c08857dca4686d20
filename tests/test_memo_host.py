"""The per-activation memo behind MixedLinear's shared quantization and stacked-group
outputs (no GPU): an entry is served once per consumer, and not at all once the tensor
it was derived from has changed."""

from __future__ import annotations

import torch

from tilequant_b200.mixed_linear import _Memo


def test_served_once_per_consumer():
    x = torch.randn(4, 8)
    _Memo.store(x, "k", "a", 123)
    assert _Memo.lookup(x, "k", "a") is None  # the storing consumer already has it
    assert _Memo.lookup(x, "k", "b") == 123
    assert _Memo.lookup(x, "k", "b") is None  # b was served
    assert _Memo.lookup(x, "k", "c") == 123
    assert _Memo.lookup(x, "other", "d") is None


def test_changed_tensor_invalidates():
    x = torch.randn(4, 8)
    _Memo.store(x, "k", "a", 1)
    x.add_(1.0)  # version counter moves
    assert _Memo.lookup(x, "k", "b") is None


def test_views_and_inference_tensors():
    base = torch.randn(4, 8)
    v = base[:, :4]
    _Memo.store(v, "k", "a", 2)
    assert _Memo.lookup(base, "k", "b") is None  # the memo belongs to the view object
    with torch.inference_mode():
        t = torch.randn(3, 3)
        _Memo.store(t, "k", "a", 3)
        assert _Memo.lookup(t, "k", "b") == 3
    _Memo.forget(t, "k")
    assert _Memo.lookup(t, "k", "c") is None
