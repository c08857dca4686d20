"""Tensor parallelism on 2 GPUs (skipped with fewer): the sharded MixedLinear decoder
against the unsharded one, eager forward and CUDA-graph greedy decoding with the NCCL
all-reduces captured in the graphs -- or, with a PeerExchange, the decode-sized
row-parallel sums done inside the decode GEMM over NVLink -- and a K-split GEMM
through the peer sum against the unsplit GEMM."""

from __future__ import annotations

import queue
import socket
import time
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _guarded(target, rank, world, port, out_q, *args):
    """Run one rank's `target`; its result, or the traceback of what it raised, goes to
    `out_q` as (rank, ok, payload) so the parent learns of a failed rank at once."""
    try:
        out_q.put((rank, True, target(rank, world, port, *args)))
    except BaseException:
        out_q.put((rank, False, traceback.format_exc()))
        raise


def _run_two_ranks(target, *args, deadline_s=400):
    """Spawn two ranks of `target(rank, world, port, *args)` and return their results in
    rank order.  A rank that raised fails the test with its traceback as soon as it is
    reported; ranks are never killed (the one still in a collective ends on its process
    group's timeout), and the parent waits no longer than `deadline_s` for results."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_guarded, args=(target, r, 2, port, q) + args) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    end = time.monotonic() + deadline_s
    while len(res) < 2 and time.monotonic() < end:
        try:
            rank, ok, payload = q.get(timeout=1.0)
        except queue.Empty:
            if all(p.exitcode is not None for p in procs):
                break
            continue
        res[rank] = (ok, payload)
        if not ok:
            break
    for p in procs:
        p.join(timeout=180)
    failed = {r: v[1] for r, v in res.items() if not v[0]}
    assert not failed, "\n".join(f"rank {r}:\n{tb}" for r, tb in failed.items())
    assert len(res) == 2, f"ranks without a result (exit codes {[p.exitcode for p in procs]})"
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return [res[r][1] for r in range(2)]


def _model(dev, qwen=False):
    if qwen:
        from transformers import Qwen2Config as Cfg, Qwen2ForCausalLM as Model

        cfg = Cfg(hidden_size=512, intermediate_size=1280, num_hidden_layers=2, num_attention_heads=8,
                  num_key_value_heads=2, vocab_size=500, attn_implementation="sdpa")
    else:
        from transformers import LlamaConfig as Cfg, LlamaForCausalLM as Model

        cfg = Cfg(hidden_size=512, intermediate_size=1280, num_hidden_layers=2, num_attention_heads=8,
                  num_key_value_heads=4, head_dim=64, vocab_size=500, attn_implementation="sdpa")
    torch.manual_seed(0)
    with torch.device(dev):
        return Model(cfg).to(torch.bfloat16).eval()


def _worker(rank, world, port, qwen, peer):
    import os

    import torch.distributed as dist

    from tilequant_b200.apply import apply_tile_maps
    from tilequant_b200.graph_decode import CudaGraphGreedyDecoder
    from tilequant_b200.parallel import projection_shapes, seeded_random_keep, tensor_parallel_
    from tilequant_b200.peer import PeerExchange

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    import datetime

    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    exchange = None
    try:
        if peer:
            exchange = PeerExchange(dev, world, rank).connect()
        mtype = "qwen2" if qwen else "llama"
        full = _model(dev, qwen)
        keep = seeded_random_keep(0.1, 5, list(projection_shapes(full)))
        apply_tile_maps(full, keep, model_type=mtype)
        ids = torch.randint(0, 500, (2, 24), generator=torch.Generator().manual_seed(1)).to(dev)
        with torch.inference_mode():
            want = full(input_ids=ids).logits.float()
        del full
        model = _model(dev, qwen)
        tensor_parallel_(model, rank, world, keep, model_type=mtype, exchange=exchange)
        with torch.inference_mode():
            got = model(input_ids=ids).logits.float()
        rel = float((got - want).abs().max() / want.abs().max())
        agree = float((got.argmax(-1) == want.argmax(-1)).float().mean())
        dec = CudaGraphGreedyDecoder.prepare(model, prompt_tokens=24, max_new_tokens=12, batch_size=2, device=dev)
        toks = dec.generate(ids.cpu()).clone()
        dec.close()
        gathered = [torch.empty_like(toks) for _ in range(world)]
        dist.all_gather(gathered, toks)
        same = all(torch.equal(g, toks) for g in gathered)
        status = 0 if exchange is None else exchange.status()
        return rel, agree, same, status
    finally:
        if exchange is not None:
            torch.cuda.synchronize()
            dist.barrier()
            exchange.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("qwen,peer", [(False, False), (True, False), (False, True), (True, True)])
def test_tensor_parallel_two_gpus(qwen, peer):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run_two_ranks(_worker, qwen, peer)
    for rank, (rel, agree, same, status) in enumerate(res):
        # row-parallel partials are summed in another order than the single-GPU K loop
        # (and rounded to BF16 first on the NCCL path), and the difference travels
        # through every later layer in BF16
        assert rel < 5e-2, (rank, rel)
        assert agree > 0.9, (rank, agree)
        assert same, rank  # every rank generates the same tokens
        assert status == 0, rank  # no peer wait ran out


def _gemm_worker(rank, world, port):
    import datetime
    import os
    from types import SimpleNamespace

    import torch.distributed as dist

    import tilequant_b200 as tq
    from tilequant_b200.apply import complement_ids
    from tilequant_b200.parallel import restrict_keep_ids
    from tilequant_b200.peer import PeerExchange, gemm_mixed_peer_sum
    from tests.golden import inputs as I
    from tests.helpers import assert_close_gemm, assert_close_with_bias, from_torch16

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    exchange = PeerExchange(dev, world, rank).connect()
    try:
        cfg = SimpleNamespace(tile_m=64, tile_n=64, pad_to_tile=True, quant_style="gi")
        m, k = 2048, 4096
        n_tr, n_tc = m // 64, k // 64
        w = I.weight(m, k, 40).to(dev)
        keep = I.keep_ids(n_tr, n_tc, 0.05, 41)
        full = tq.pack_weight_from_tile_ids(w, n_tr=n_tr, n_tc=n_tc, int8_tile_ids=complement_ids(keep, n_tr * n_tc),
                                            fp16_tile_ids=keep, cfg=cfg)
        c0, c1 = rank * n_tc // world, (rank + 1) * n_tc // world
        kk, _, _ = restrict_keep_ids(keep, n_tc, rows=(0, n_tr), cols=(c0, c1))
        part = tq.pack_weight_from_tile_ids(w[:, c0 * 64:c1 * 64].contiguous(), n_tr=n_tr, n_tc=c1 - c0,
                                            int8_tile_ids=complement_ids(kk, n_tr * (c1 - c0)), fp16_tile_ids=kk,
                                            cfg=cfg)

        def wts(p):
            return dict(int8_tiles=p.int8_tiles, int8_scales=p.int8_scales, int8_tile_ids=p.int8_tile_ids,
                        int8_row_ptr=p.int8_row_ptr, fp16_tiles=p.fp16_tiles, fp16_tile_ids=p.fp16_tile_ids,
                        fp16_row_ptr=p.fp16_row_ptr, M=p.M_orig, K=p.K_orig, n_tr=p.n_tr, n_tc=p.n_tc)

        bias_all = (torch.randn(m, generator=I.gen(42)) * 0.5).to(dev, torch.bfloat16)
        errors = []
        same = True
        for rows in (1, 7, 16):
            for call in range(2):
                bias = bias_all if call else None
                x = I.activations(rows, k, 50 + 10 * rows + call).to(dev)
                q, sx = tq.quantize_activation_tile_absmax(x)
                want = tq.gemm_mixed_rows_splitk(x_fp=x, x_int8=q, sx=sx, out_dtype=torch.bfloat16, bias=bias,
                                                 **wts(full))
                xs = x[:, c0 * 64:c1 * 64].contiguous()
                qs, ss = tq.quantize_activation_tile_absmax(xs)
                got = gemm_mixed_peer_sum(x_fp=xs, x_int8=qs, sx=ss, out_dtype=torch.bfloat16, bias=bias,
                                          exchange=exchange, **wts(part))
                torch.cuda.synchronize()
                try:  # FP32 partial sums in another association than the unsplit K loop
                    if bias is None:
                        assert_close_gemm(from_torch16(got), from_torch16(want), f"rows {rows}")
                    else:
                        assert_close_with_bias(from_torch16(got), from_torch16(want), from_torch16(bias),
                                               f"rows {rows} + bias")
                except AssertionError as e:
                    errors.append(str(e))
                gathered = [torch.empty_like(got) for _ in range(world)]
                dist.all_gather(gathered, got)
                same = same and all(torch.equal(g.view(torch.int16), got.view(torch.int16)) for g in gathered)
        return errors, same, exchange.status()
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        exchange.close()
        dist.destroy_process_group()


def test_peer_sum_gemm_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run_two_ranks(_gemm_worker)
    for rank, (errors, same, status) in enumerate(res):
        assert status == 0, rank
        assert same, rank  # the same bits on every rank
        assert not errors, (rank, errors)


def _token_worker(rank, world, port, name, peer):
    """TP1 (this GPU alone) against TP2 on the greedy-token fixture models: TP1 decodes
    freely, TP2 is teacher-forced on TP1's tokens."""
    import datetime
    import os
    from pathlib import Path

    import numpy as np
    import torch.distributed as dist

    from tests.golden import tiny_models as T
    from tests.helpers import greedy_steps, tracking
    from tilequant_b200.apply import apply_tile_maps, default_cfg
    from tilequant_b200.parallel import tensor_parallel_
    from tilequant_b200.peer import PeerExchange

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    exchange = None
    try:
        if peer:
            exchange = PeerExchange(dev, world, rank).connect()
        fix = np.load(Path(__file__).resolve().parent / "golden" / "tokens.npz")
        spec = T.MODELS[name]
        prefix = f"{name}__keep__"
        keep = {k[len(prefix):]: torch.from_numpy(fix[k]) for k in fix.files if k.startswith(prefix)}
        prompt = torch.from_numpy(fix[f"{name}__prompt"])
        cfg = default_cfg(dtype_out="fp16")
        one = T.build(spec, dev)
        apply_tile_maps(one, keep, cfg, model_type=spec["arch"])
        ref, ref_logits = greedy_steps(one, prompt, dev, T.NEW_TOKENS, eager=False)
        del one
        two = T.build(spec, dev)
        tensor_parallel_(two, rank, world, lambda n, n_tr, n_tc: keep[n], cfg=cfg, model_type=spec["arch"],
                         exchange=exchange)
        _, two_logits = greedy_steps(two, prompt, dev, T.NEW_TOKENS, eager=False, forced=ref)
        same = two_logits.view(torch.int16).to(dev, torch.int32)  # the logits' bits; NCCL has no int16
        gathered = [torch.empty_like(same) for _ in range(world)]
        dist.all_gather(gathered, same)
        identical = all(torch.equal(g, same) for g in gathered)
        status = 0 if exchange is None else exchange.status()
        return tracking(ref, ref_logits, two_logits), identical, status
    finally:
        if exchange is not None:
            torch.cuda.synchronize()
            dist.barrier()
            exchange.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("name,peer", [("llama", False), ("qwen2", False), ("llama", True), ("qwen2", True)])
def test_tensor_parallel_tokens_follow_tp1(name, peer):
    """Greedy tokens under TP2 against TP1 over 32 steps (the fixture's FP16 tiny Llama
    and Qwen2, 10 % 16-bit tiles): the row-parallel sums associate differently from the
    one-GPU K loop, so TP2 is teacher-forced on TP1's tokens and must keep its logits
    within 6 % of the logit scale and pick TP1's token wherever TP1's top-1 leads by at
    least 32 FP16 ulps; both ranks hold bit-identical logits."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run_two_ranks(_token_worker, name, peer)
    for rank, ((drift, sure, bad, agree), identical, status) in enumerate(res):
        print(f"{name} peer={peer} rank {rank}: drift {drift:.4f}, sure {sure:.2f}, agree {agree:.3f}, "
              f"differing picks {bad}")
        assert drift <= 0.06, (rank, drift)
        assert sure >= 0.6, (rank, sure)
        assert not bad, (rank, bad)
        assert identical, rank
        assert status == 0, rank
