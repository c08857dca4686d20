"""Tensor-parallel sharding logic, on the CPU: head ownership, tile-map restriction, and
a 2-rank (gloo) forward of a sharded dense decoder against the unsharded one."""

from __future__ import annotations

import socket

import pytest
import torch
import torch.multiprocessing as mp

from tilequant_b200.parallel import (
    AllReduceSum,
    LinearShard,
    head_shard,
    projection_shapes,
    restrict_keep_ids,
    shard_decoder_,
    shard_keep_ids,
    split_range,
    wrap_row_parallel_,
)


@pytest.mark.parametrize("heads,kv,world", [(24, 8, 1), (24, 8, 2), (24, 8, 4), (24, 8, 8), (28, 4, 2), (28, 4, 4),
                                            (28, 4, 8), (40, 8, 8), (40, 8, 2)])
def test_head_shards_cover_every_head_once(heads, kv, world):
    seen_q = []
    for r in range(world):
        hs = head_shard(heads, kv, r, world)
        q0, q1 = hs.q_heads
        k0, k1 = hs.kv_heads
        assert q1 > q0 and k1 > k0
        group = heads // kv
        # every query head reads a KV head this rank holds
        assert all(k0 <= q // group < k1 for q in range(q0, q1))
        seen_q.extend(range(q0, q1))
    assert sorted(seen_q) == list(range(heads))


def test_qwen7b_tp8_heads_are_3_and_4():
    counts = [head_shard(28, 4, r, 8).q_heads for r in range(8)]
    assert [b - a for a, b in counts] == [3, 4, 3, 4, 3, 4, 3, 4]
    assert [head_shard(28, 4, r, 8).kv_heads for r in range(8)] == [(k, k + 1) for k in (0, 0, 1, 1, 2, 2, 3, 3)]


def test_head_shard_rejects_uneven():
    with pytest.raises(ValueError):
        head_shard(24, 8, 0, 3)
    with pytest.raises(ValueError):
        head_shard(28, 4, 0, 6)


def test_restrict_keep_ids_matches_mask():
    g = torch.Generator().manual_seed(0)
    n_tr, n_tc = 7, 9
    keep = torch.randperm(n_tr * n_tc, generator=g)[:20].sort().values
    mask = torch.zeros(n_tr, n_tc, dtype=torch.bool)
    mask.view(-1)[keep] = True
    for rows, cols in (((2, 5), None), (None, (3, 8)), ((0, 7), (0, 9)), ((6, 7), (8, 9))):
        ids, sr, sc = restrict_keep_ids(keep, n_tc, rows=rows or (0, n_tr), cols=cols)
        r0, r1 = rows or (0, n_tr)
        c0, c1 = cols or (0, n_tc)
        want = torch.nonzero(mask[r0:r1, c0:c1].reshape(-1)).reshape(-1).to(torch.int32)
        assert (sr, sc) == (r1 - r0, c1 - c0)
        assert torch.equal(ids, want)


def test_shard_keep_ids_row_and_column_parallel():
    keep = torch.tensor([0, 5, 9, 17, 40], dtype=torch.int32)  # 6 x 8 grid (384 x 512 features)
    col_par = shard_keep_ids(keep, (384, 512), LinearShard("q", (128, 320), None))  # row tiles 2..4
    assert col_par.tolist() == [17 - 16]
    row_par = shard_keep_ids(keep, (384, 512), LinearShard("o", None, (64, 384)))  # column tiles 1..5
    # kept tiles in columns 1..5: 5 (r0,c5), 9 (r1,c1), 17 (r2,c1) -> renumbered with 5 columns
    assert row_par.tolist() == [0 * 5 + 4, 1 * 5 + 0, 2 * 5 + 0]


def test_split_range_partitions():
    for n in (1, 7, 48, 296):
        for parts in (1, 2, 3, 8):
            bounds = [split_range(n, parts, i) for i in range(parts)]
            assert bounds[0][0] == 0 and bounds[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(bounds, bounds[1:]))


def _tiny_llama(qkv_bias=False):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=64, vocab_size=97, attention_bias=qkv_bias,
                      attn_implementation="sdpa")
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).eval()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, qkv_bias, out_q):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        torch.set_num_threads(1)
        full = _tiny_llama(qkv_bias)
        ids = torch.randint(0, 97, (2, 11), generator=torch.Generator().manual_seed(3))
        with torch.no_grad():
            want = full(input_ids=ids).logits
        model = _tiny_llama(qkv_bias)
        shapes = projection_shapes(model)
        shards = shard_decoder_(model, rank, world)
        assert set(shards) == set(shapes)
        assert wrap_row_parallel_(model, shards) == 4
        assert sum(isinstance(m, AllReduceSum) for m in model.modules()) == 4
        with torch.no_grad():
            got = model(input_ids=ids).logits
        out_q.put((rank, float((got - want).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("qkv_bias", [False, True])
def test_sharded_dense_decoder_matches_full_on_two_gloo_ranks(qkv_bias):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, qkv_bias, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err in results:
        assert err < 1e-4, (rank, err)
