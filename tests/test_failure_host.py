"""Failure detection without a GPU fault (host side, gloo ranks on the CPU).

A rank that dies between steps, or never joins, must surface on the surviving rank as
an error from its next collective within the process group's timeout -- not as a hang
-- and the tensor-parallel wiring must not swallow it.  Bad tile maps are rejected on
the host before anything runs.
"""

from __future__ import annotations

import datetime
import socket
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tilequant_b200.parallel import shard_decoder_, wrap_row_parallel_

TIMEOUT_S = 6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tiny():
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(hidden_size=128, intermediate_size=256, num_hidden_layers=1, num_attention_heads=2,
                      num_key_value_heads=2, head_dim=64, vocab_size=61, attn_implementation="sdpa")
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).eval()


def _worker(rank, world, port, mode, out_q):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=TIMEOUT_S))
    torch.set_num_threads(1)
    model = _tiny()
    shards = shard_decoder_(model, rank, world)
    wrap_row_parallel_(model, shards)
    ids = torch.randint(0, 61, (1, 5), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        model(input_ids=ids)  # one good step on every rank
    if rank == 1:
        out_q.put((rank, "left", 0.0))
        if mode == "exit":
            import os

            out_q.close()
            out_q.join_thread()  # the message is out before the process vanishes
            os._exit(0)  # dies between steps, with nothing in flight
        raise SystemExit(0)
    t0 = time.time()
    try:
        with torch.no_grad():
            model(input_ids=ids)  # its first row-parallel all-reduce has no partner
        out_q.put((rank, "no error", time.time() - t0))
    except Exception as e:  # noqa: BLE001 -- the collective's failure is the expected outcome
        out_q.put((rank, type(e).__name__, time.time() - t0))


@pytest.mark.parametrize("mode", ["exit", "raise"])
def test_dead_rank_surfaces_as_an_error_within_the_timeout(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, what, secs = q.get(timeout=240)
        res[rank] = (what, secs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    assert res[1][0] == "left"
    what, secs = res[0]
    assert what != "no error"
    assert secs < 10 * TIMEOUT_S


def test_out_of_range_tile_ids_are_rejected_before_anything_runs(tmp_path):
    from tilequant_b200.mask_io import load_fp16_keep_ids_for_layer

    np.savez_compressed(tmp_path / "fp16_keep_ids_tile64x64.npz", stems=np.asarray(["model_layers_0_mlp_up_proj"]),
                        shape_0=np.asarray([2, 2], np.int32), ids_0=np.asarray([1, 4], np.uint16))
    with pytest.raises(RuntimeError, match="Out-of-bound"):
        load_fp16_keep_ids_for_layer(tmp_path, "model.layers.0.mlp.up_proj")
    good = tmp_path / "good"
    good.mkdir()
    np.savez_compressed(good / "fp16_keep_ids_tile64x64.npz", stems=np.asarray(["model_layers_0_mlp_up_proj"]),
                        shape_0=np.asarray([2, 2], np.int32), ids_0=np.asarray([1, 3], np.uint16))
    assert load_fp16_keep_ids_for_layer(good, "model.layers.0.mlp.up_proj")[0].tolist() == [1, 3]
    with pytest.raises(FileNotFoundError, match="stem not found"):
        load_fp16_keep_ids_for_layer(good, "model.layers.9.mlp.up_proj")
