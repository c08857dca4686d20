"""NVTX ranges are off by default (no calls into NVTX) and, when on, bracket the
decorated host steps, also when they raise."""

from __future__ import annotations

import pytest
import torch

from tilequant_b200 import trace


def test_ranges_follow_the_switch(monkeypatch):
    calls = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda name: calls.append(("push", name)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: calls.append(("pop", None)))

    @trace.traced("tq.test")
    def step(x):
        if x < 0:
            raise ValueError("negative")
        return x + 1

    was = trace.enabled()
    try:
        trace.set_enabled(False)
        assert step(1) == 2 and calls == []
        with trace.nvtx_range("tq.off"):
            pass
        assert calls == []
        trace.set_enabled(True)
        assert step(2) == 3
        assert calls == [("push", "tq.test"), ("pop", None)]
        with pytest.raises(ValueError):
            step(-1)
        assert calls[-2:] == [("push", "tq.test"), ("pop", None)]
        with trace.nvtx_range("tq.block"):
            pass
        assert calls[-2:] == [("push", "tq.block"), ("pop", None)]
    finally:
        trace.set_enabled(was)


def test_entry_points_are_traced():
    from tilequant_b200.graph_decode import CudaGraphGreedyDecoder
    from tilequant_b200.loader import load_mixed_precision_model_from_masks
    from tilequant_b200.mixed_linear import MixedLinear
    from tilequant_b200.parallel import AllReduceSum, PeerReduceSum

    for fn in (CudaGraphGreedyDecoder.prefill, CudaGraphGreedyDecoder.decode, load_mixed_precision_model_from_masks,
               MixedLinear.forward, AllReduceSum.forward, PeerReduceSum.forward):
        assert hasattr(fn, "__wrapped__"), fn
