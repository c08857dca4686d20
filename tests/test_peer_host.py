"""Host logic of the row-parallel peer sum (no GPU): which path ``PeerReduceSum`` takes,
and how it learns, once per row count, that a shape's decode grid does not fit."""

from __future__ import annotations

import pytest
import torch

import tilequant_b200.peer as peer_mod
import tilequant_b200.quant_utils as qu
from tilequant_b200 import _native as N
from tilequant_b200.parallel import PeerReduceSum


class _Inner(torch.nn.Module):
    """Stands in for a row-parallel MixedLinear shard: K 128 in, M 64 out."""

    K_orig, M_orig, tile_n = 128, 64, 64

    def __init__(self):
        super().__init__()
        self.calls = 0

    def _out_dtype(self):
        return torch.bfloat16

    def _weights(self):
        return {}

    def forward(self, x):
        self.calls += 1
        return torch.full((*x.shape[:-1], self.M_orig), 2.0, dtype=torch.bfloat16)


@pytest.fixture
def fake_kernels(monkeypatch):
    state = {"peer_calls": 0, "error": None}

    def quantize(x, tile_n=64):
        return torch.zeros_like(x, dtype=torch.int8), torch.ones(x.shape[1] // tile_n)

    def peer_sum(*, x_fp, out_dtype, exchange, bias=None, **_):
        state["peer_calls"] += 1
        if state["error"] is not None:
            raise state["error"]
        return torch.full((x_fp.shape[0], 64), 3.0, dtype=out_dtype)

    monkeypatch.setattr(qu, "quantize_activation_tile_absmax", quantize)
    monkeypatch.setattr(peer_mod, "gemm_mixed_peer_sum", peer_sum)
    return state


def test_decode_sized_calls_take_the_peer_sum(fake_kernels):
    mod = PeerReduceSum(_Inner(), exchange=object(), bias=torch.ones(64))
    y = mod(torch.randn(2, 3, 128, dtype=torch.bfloat16))
    assert y.shape == (2, 3, 64) and float(y[0, 0, 0]) == 3.0  # the kernel added the bias itself
    assert fake_kernels["peer_calls"] == 1 and mod.inner.calls == 0
    y = mod(torch.randn(65, 128, dtype=torch.bfloat16))  # beyond 64 rows: the all-reduce path
    assert mod.inner.calls == 1 and float(y[0, 0]) == 3.0  # 2 from the shard + the bias once


def test_a_grid_that_does_not_fit_falls_back_once(fake_kernels):
    fake_kernels["error"] = ValueError("gemm_mixed_peer_sum: peer sum: more decode CTAs than exchange slots")
    mod = PeerReduceSum(_Inner(), exchange=object())
    x = torch.randn(64, 128, dtype=torch.bfloat16)
    assert float(mod(x)[0, 0]) == 2.0 and fake_kernels["peer_calls"] == 1
    assert float(mod(x)[0, 0]) == 2.0 and fake_kernels["peer_calls"] == 1  # not asked again
    assert mod._peer_fits == {64: False}
    fake_kernels["error"] = None
    mod(torch.randn(8, 128, dtype=torch.bfloat16))  # another row count is asked
    assert fake_kernels["peer_calls"] == 2 and mod._peer_fits[8] is True


def test_other_errors_are_not_swallowed(fake_kernels):
    mod = PeerReduceSum(_Inner(), exchange=object())
    fake_kernels["error"] = ValueError("bias must be a contiguous [M] tensor of out_dtype")
    with pytest.raises(ValueError, match="bias"):
        mod(torch.randn(4, 128, dtype=torch.bfloat16))
    fake_kernels["error"] = ValueError("gemm_mixed_peer_sum: peer sum: need 1 <= world <= 8 and 0 <= rank < world")
    with pytest.raises(ValueError, match="world"):  # a misconfigured exchange is not a size fallback
        mod(torch.randn(4, 128, dtype=torch.bfloat16))
    # a shape that worked before and then fails is an error, not a fallback
    fake_kernels["error"] = None
    mod(torch.randn(5, 128, dtype=torch.bfloat16))
    fake_kernels["error"] = N.TileQuantError("gemm_mixed_peer_sum: TQ_ERR_UNSUPPORTED: peer sum: the decode grid "
                                             "does not fit on the GPU at once")
    with pytest.raises(N.TileQuantError):
        mod(torch.randn(5, 128, dtype=torch.bfloat16))


def test_decoder_peer_status_raises_after_a_timeout():
    """The decoder's synchronised points read the exchanges' error words: a peer sum that
    gave up waiting surfaces as TileQuantError instead of silently wrong tokens."""
    from tilequant_b200 import _native as N
    from tilequant_b200.graph_decode import CudaGraphGreedyDecoder

    class Exchange:  # the error word of a PeerExchange, as status() reads it
        def __init__(self):
            self.word = N.TQ_OK

        def status(self):
            return self.word

    ex = Exchange()
    dec = CudaGraphGreedyDecoder.__new__(CudaGraphGreedyDecoder)
    dec._exchanges = [ex]
    dec.check_peer_status()
    ex.word = N.TQ_ERR_TIMEOUT
    with pytest.raises(N.TileQuantError, match="reset the exchange"):
        dec.check_peer_status()


def test_decoder_step_status_raises_and_clears_after_a_timeout():
    """The fused decode step's attention error word is read at the same synchronised
    point: a timed-out cache load surfaces as TileQuantError and the word is cleared."""
    from tilequant_b200 import _native as N
    from tilequant_b200.graph_decode import CudaGraphGreedyDecoder

    class Step:  # the attention error word of a FusedDecodeStep
        def __init__(self):
            self.word = N.TQ_OK

        def status(self):
            return self.word

        def reset_status(self):
            self.word = N.TQ_OK

    dec = CudaGraphGreedyDecoder.__new__(CudaGraphGreedyDecoder)
    dec._step = None
    dec.check_step_status()  # no fused step: nothing to read
    dec._step = Step()
    dec.check_step_status()
    dec._step.word = N.TQ_ERR_TIMEOUT
    with pytest.raises(N.TileQuantError, match="KV-cache chunk"):
        dec.check_step_status()
    dec.check_step_status()  # cleared
