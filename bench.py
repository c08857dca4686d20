#!/usr/bin/env python
"""Benchmark of the mixed INT8/BF16 64x64 tile GEMM path on B200 (one JSON line).

Workload (default, benchmark config 2): one Llama-3.2-3B decoder block at prefill,
4 x 2048 tokens (8192 activation rows), hidden 3072, intermediate 8192, 24/8 heads,
head_dim 128; random-init BF16 weights N(0, 0.02) with 5 % of each linear's 64x64
tiles kept BF16 (uniformly chosen), the rest INT8 with one scale per tile.

* a step = one pass of the hot path over the block: the four MixedLinear forwards
  (stacked Q/K/V, O, stacked gate/up, down), each = activation quantization + mixed
  GEMM, on the block's own activations (captured from one eager block forward);
* ``value`` = linear ops of the block (2 * rows * sum(out * in) = 1.649e12) / step
  time, TOPS; device time from CUDA events, L2 flushed (256 MB write) between steps;
* ``e2e`` = the same metric for the whole block forward through the public module
  API with the hidden states copied in from pinned host memory and the block output
  copied back every step;
* ``roofline`` = the dominant kernel (the stacked gate/up mixed GEMM) against the
  dense INT8 peak measured in this run (cuBLASLt INT8 8192^3 via ``torch._int_mm``);
* ``cpu_baseline`` = the CPU restatement of the reference (oracle/, C + OpenMP on all
  host threads) on windows of ``--cpu-rows`` consecutive rows of each linear, built
  from the same seeded weights and tile maps, for about ``--cpu-seconds``;
* outside the timed regions, the timed gate/up launch's output is checked against the
  CPU restatement on rows sampled from every 128-row block; no line is printed when it
  does not match.

``--impl reference`` times that CPU restatement alone, one window per step, without
loading this project's GPU library: the reference's own GEMM is a Triton GPU kernel
whose Python sources do not travel to the GPU box, and its CPU torch path covers only
the quantizer and the packer.  ``--workload decode`` measures config 1 (one
q_proj-shaped MixedLinear, 16 decode tokens) in GB/s instead; ``--workload gemm``
times one mixed GEMM launch of ``--shape`` (the case the kernel profiles capture).

The default line also carries ``decode`` (config 1: decode GEMM GB/s, fraction of HBM)
and ``generate`` (config 3: decode tokens/s, p50 TTFT and TPOT) sub-objects.

Multi-GPU (torchrun): the default workload is strong-scaled by tensor parallelism (the
same block and total work at every N: Q/K/V and gate/up column-parallel, O and down
row-parallel with an NCCL all-reduce of their partial outputs); the step time is the
max over ranks.  ``--workload decode``/``gemm`` run one replica per rank (weak scaling),
``--workload generate --tp`` shards the model over the ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path
from types import SimpleNamespace

import torch
import torch.nn.functional as F

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

LLAMA3B = dict(hidden=3072, inter=8192, heads=24, kv_heads=8, head_dim=128, rope_theta=500000.0)
TOKENS = (4, 2048)
KEEP = 0.05
METRIC_PREFILL = "tile-GEMM TOPS: Llama-3.2-3B decoder block prefill (4x2048 tokens), 4 MixedLinear forwards"
PREFILL_CONFIG = {"workload": "config2: Llama-3.2-3B decoder block prefill", "rows": TOKENS[0] * TOKENS[1],
                  "hidden": 3072, "intermediate": 8192, "heads": "24/8", "keep_bf16": KEEP, "tile": "64x64",
                  "l2": "flushed (256 MB write) between timed steps"}
GEMM_PROFILE = "umma_kernel_gate_up_8192x16384x3072.md"
DECODE_PROFILE = "gemv_kernel_config1_16x3072x3072.md"


def _peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


def _profile_traffic(summary: str):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) recorded by
    an ncu capture in profiles/<summary> as a line `traffic_bytes_per_launch: N`."""
    try:
        for line in (ROOT / "profiles" / summary).read_text().splitlines():
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip().split()[0]))
    except Exception:
        pass
    return None


# ---------------------------------------------------------------- workload pieces

def _cfg():
    return SimpleNamespace(tile_m=64, tile_n=64, pad_to_tile=True, quant_style="gi", dtype_out="bf16")


def _mixed_linear(out_f, in_f, seed, device, keep=KEEP):
    import tilequant_b200 as tq
    from tests.golden import inputs as I

    w = I.weight(out_f, in_f, seed).to(device)
    n_tr, n_tc = (out_f + 63) // 64, (in_f + 63) // 64
    fp16 = I.keep_ids(n_tr, n_tc, keep, seed + 1)
    pack = tq.pack_weight_from_tile_ids(w, n_tr=n_tr, n_tc=n_tc, int8_tile_ids=I.complement_ids(fp16, n_tr * n_tc),
                                        fp16_tile_ids=fp16, cfg=_cfg())
    return tq.MixedLinear(pack, None, _cfg())


class Block:
    """Llama decoder block with MixedLinear projections (RMSNorm, RoPE, causal GQA
    SDPA, SwiGLU), Q/K/V and gate/up stacked into one GEMM each."""

    def __init__(self, seed, device, dims=LLAMA3B, keep=KEEP):
        import tilequant_b200 as tq

        h, i, nh, nkv, hd = dims["hidden"], dims["inter"], dims["heads"], dims["kv_heads"], dims["head_dim"]
        self.dims = dims
        lin = lambda o, k, s: _mixed_linear(o, k, seed * 100 + s, device, keep)  # noqa: E731
        self.qkv = tq.MixedLinearGroup([lin(nh * hd, h, 1), lin(nkv * hd, h, 3), lin(nkv * hd, h, 5)]).linear
        self.o = lin(h, nh * hd, 7)
        self.gate_up = tq.MixedLinearGroup([lin(i, h, 9), lin(i, h, 11)]).linear
        self.down = lin(h, i, 13)
        self.ln1 = torch.ones(h, device=device, dtype=torch.bfloat16)
        self.ln2 = torch.ones(h, device=device, dtype=torch.bfloat16)
        inv = 1.0 / (dims["rope_theta"] ** (torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd))
        ang = torch.outer(torch.arange(TOKENS[1], device=device, dtype=torch.float32), inv)
        self.cos = torch.cat([ang, ang], -1).cos().to(torch.bfloat16)
        self.sin = torch.cat([ang, ang], -1).sin().to(torch.bfloat16)

    @staticmethod
    def _rms(x, w, eps=1e-5):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w

    def _rope(self, x):  # (B, H, S, D)
        d = x.shape[-1] // 2
        return x * self.cos + torch.cat([-x[..., d:], x[..., :d]], -1) * self.sin

    def forward(self, hidden, capture=None):
        d = self.dims
        B, S = TOKENS
        nh, nkv, hd = d["heads"], d["kv_heads"], d["head_dim"]
        x = self._rms(hidden, self.ln1)
        q, k, v = self.qkv(x).split([nh * hd, nkv * hd, nkv * hd], dim=-1)
        q = self._rope(q.view(B, S, nh, hd).transpose(1, 2))
        k = self._rope(k.view(B, S, nkv, hd).transpose(1, 2))
        v = v.view(B, S, nkv, hd).transpose(1, 2)
        attn = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        attn = attn.transpose(1, 2).reshape(B * S, nh * hd)
        h2 = hidden + self.o(attn)
        x2 = self._rms(h2, self.ln2)
        g, u = self.gate_up(x2).chunk(2, dim=-1)
        act = (F.silu(g.float()) * u.float()).to(torch.bfloat16)
        out = h2 + self.down(act)
        if capture is not None:
            capture.update(x_qkv=x, x_o=attn.contiguous(), x_gu=x2, x_down=act)
        return out

    def linear_ops(self, rows):
        d = self.dims
        h, i, nh, nkv, hd = d["hidden"], d["inter"], d["heads"], d["kv_heads"], d["head_dim"]
        return 2 * rows * ((nh + 2 * nkv) * hd * h + h * nh * hd + 2 * i * h + h * i)


# -------------------------------------------------------------------- helpers

class ClockSampler:
    """Polls SM clock and throttle reasons through NVML while the timed region runs."""

    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index, period=0.01):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.period = period
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM))
                mask = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                for name, bit in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def _dist():
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0"))


def _max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(ws):
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()


def _int8_peak(device):
    """cuBLASLt INT8 GEMM 8192^3 through torch._int_mm: best of 5, TOPS."""
    try:
        a = torch.randint(-127, 127, (8192, 8192), device=device, dtype=torch.int8)
        b = torch.randint(-127, 127, (8192, 8192), device=device, dtype=torch.int8).t()
        for _ in range(3):
            torch._int_mm(a, b)
        best = 0.0
        for _ in range(5):
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            best = max(best, 2 * 8192 ** 3 / (e0.elapsed_time(e1) * 1e-3) / 1e12)
        return best, "measured in this run: torch._int_mm (cuBLASLt) INT8 8192^3, best of 5"
    except Exception as exc:  # pragma: no cover - depends on the box
        return 4500.0, f"datasheet dense INT8 (torch._int_mm failed: {type(exc).__name__})"


def _bits16(t: torch.Tensor):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view("uint16")


def _pack_arrays(mod) -> dict:
    """A MixedLinear's packed buffers as host arrays in the oracle's layout."""
    pk = {}
    for key in ("int8_tiles", "int8_scales", "int8_tile_ids", "int8_row_ptr", "fp16_tiles", "fp16_tile_ids",
                "fp16_row_ptr"):
        v = getattr(mod, key)
        pk[key] = _bits16(v) if v.dtype == torch.bfloat16 else v.cpu().numpy()
    pk.update(n_tr=mod.n_tr, n_tc=mod.n_tc)
    return pk


def _verify_sample(x: torch.Tensor, y: torch.Tensor, mod, seed: int = 0, per_block: int = 1) -> int:
    """Checker (oracle/) for a full-size GEMM launch: rows sampled from every 128-row
    token block, quantized with the scales of the whole batch, multiplied by the CPU
    restatement and compared with the GPU output within one BF16 ulp (the tolerance of
    tests/helpers.py).  Raises on a mismatch, so no value is printed for a kernel
    whose output is wrong.  Returns the number of rows checked."""
    import numpy as np

    from oracle import oracle as O
    from tests.helpers import assert_close_gemm

    rows = int(x.shape[0])
    rng = np.random.default_rng(seed)
    sel = np.unique(np.concatenate([
        np.minimum(rows - 1, b * 128 + rng.integers(0, 128, per_block)) for b in range((rows + 127) // 128)]))
    xb = _bits16(x)
    sx = O.act_scales(xb)
    xs = np.ascontiguousarray(xb[sel])
    ref = O.gemm(O.quantize_with_scales(xs, sx), sx, _pack_arrays(mod), xs, mod.M_orig, mod.K_orig, split_k=1,
                 use_fma=True)
    got = _bits16(y[torch.from_numpy(sel).to(y.device)])
    assert_close_gemm(got, ref, f"{rows}x{mod.M_orig}x{mod.K_orig} sampled rows")
    return int(sel.size)


# The config-2 linears as the reference's packs: the same seeded weights and tile maps
# as Block(seed=7) (member seeds 7 * 100 + s), Q/K/V and gate/up stacked along the
# output rows the way concat_packs_along_rows stacks them.
REF_LINEARS = (("qkv", ((3072, 701), (1024, 703), (1024, 705)), 3072),
               ("o", ((3072, 707),), 3072),
               ("gate_up", ((8192, 709), (8192, 711)), 3072),
               ("down", ((3072, 713),), 8192))


def _reference_linears(keep=KEEP):
    """Host-only construction (no GPU, no tilequant_b200): oracle packs of the four
    config-2 linears plus seeded N(0, 1) BF16 inputs of 8192 rows each."""
    import numpy as np

    from oracle import oracle as O
    from tests.golden import inputs as I

    out = []
    for i, (name, members, k) in enumerate(REF_LINEARS):
        n_tc = (k + 63) // 64
        ws, keep_ids, r0 = [], [], 0
        for m, seed in members:
            ws.append(I.bits(I.weight(m, k, seed)))
            keep_ids.append(I.keep_ids(m // 64, n_tc, keep, seed + 1).numpy().astype(np.int64) + r0 * n_tc)
            r0 += m // 64
        fp16 = np.concatenate(keep_ids)
        w = np.concatenate(ws, axis=0)
        pk = O.pack(w, r0, n_tc, O.int8_ids_from_keep(fp16, r0, n_tc), fp16)
        x = I.bits(I.activations(TOKENS[0] * TOKENS[1], k, 4242 + i))
        out.append((name, pk, x, w.shape[0], k))
    return out


def _cpu_sample(linears, rows: int, window: int = 0):
    """The CPU restatement of the reference (oracle/, C + OpenMP on all host threads) on
    one window of `rows` consecutive activation rows of each config-2 linear: quantize
    that window (its own scales, as a call of that many rows) + mixed GEMM.  Returns
    (seconds, ops)."""
    import numpy as np

    from oracle import oracle as O

    t_total, ops = 0.0, 0
    for _, pk, x, m, k in linears:
        r0 = (window * rows) % max(1, x.shape[0] - rows + 1)
        xb = np.ascontiguousarray(x[r0:r0 + rows])
        t0 = time.perf_counter()
        q, sx = O.quantize_act(xb)
        O.gemm(q, sx, pk, xb, m, k, split_k=1)
        t_total += time.perf_counter() - t0
        ops += 2 * xb.shape[0] * m * k
    return t_total, ops


def _cpu_baseline_line(linears, rows: int, seconds: float):
    """Windows of `rows` rows through the four linears, repeated for about `seconds`."""
    from oracle import oracle as O

    threads = O.set_threads(os.cpu_count() or 1)  # all host threads, whatever the launcher set
    spent, ops, w = 0.0, 0, 0
    while spent < seconds or w < 1:
        s, o = _cpu_sample(linears, rows, w)
        spent += s
        ops += o
        w += 1
    return {"value": ops / spent / 1e12, "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{w} windows of {rows} consecutive rows (of 8192) through the 4 config-2 linears, each window "
                      "quantized and multiplied as one call by oracle/tq_oracle.c (the reference's arithmetic, "
                      "OpenMP on all host threads); weights and tile maps as the GPU run, seeded N(0,1) inputs"}


def _prefill_setup(device):
    from tests.golden import inputs as I

    block = Block(seed=7, device=device)
    rows = TOKENS[0] * TOKENS[1]
    hidden = I.activations(rows, LLAMA3B["hidden"], 42).to(device)
    acts = {}
    with torch.inference_mode():
        block.forward(hidden, capture=acts)
    torch.cuda.synchronize()
    return block, hidden, acts, rows


def _mixed_linear_shard(out_f, in_f, seed, device, rows=None, cols=None, keep=KEEP):
    """This rank's slice of the config-2 linear `_mixed_linear(out_f, in_f, seed)` makes:
    output features `rows` = [r0, r1) and input features `cols` = [c0, c1) (64-aligned)
    of the same seeded weight, packed with the full tile map restricted to the slice (so
    its tiles and scales are the single-GPU pack's)."""
    import tilequant_b200 as tq
    from tests.golden import inputs as I
    from tilequant_b200.parallel import restrict_keep_ids

    w = I.weight(out_f, in_f, seed)
    n_tr, n_tc = (out_f + 63) // 64, (in_f + 63) // 64
    keep_full = I.keep_ids(n_tr, n_tc, keep, seed + 1)
    r0, r1 = rows if rows is not None else (0, out_f)
    c0, c1 = cols if cols is not None else (0, in_f)
    keep_ids, s_tr, s_tc = restrict_keep_ids(keep_full, n_tc, rows=(r0 // 64, (r1 + 63) // 64),
                                             cols=(c0 // 64, (c1 + 63) // 64))
    ws_ = w[r0:r1, c0:c1].contiguous().to(device)
    pack = tq.pack_weight_from_tile_ids(ws_, n_tr=s_tr, n_tc=s_tc, int8_tile_ids=I.complement_ids(keep_ids, s_tr * s_tc),
                                        fp16_tile_ids=keep_ids, cfg=_cfg())
    return tq.MixedLinear(pack, None, _cfg())


class BlockShard:
    """Rank `rank`'s tensor-parallel shard of Block(seed=7)'s four linears over `world`
    ranks: Q/K/V (this rank's heads) and gate/up (its intermediate row tiles)
    column-parallel, O and down row-parallel over the same head / intermediate ranges."""

    def __init__(self, rank, world, device, seed=7, dims=LLAMA3B):
        import tilequant_b200 as tq
        from tilequant_b200.parallel import head_shard, split_range

        h, i, nh, nkv, hd = dims["hidden"], dims["inter"], dims["heads"], dims["kv_heads"], dims["head_dim"]
        hs = head_shard(nh, nkv, rank, world)
        (q0, q1), (k0, k1) = hs.q_heads, hs.kv_heads
        t0, t1 = split_range(i // 64, world, rank)
        self.q_cols = (q0 * hd, q1 * hd)   # this rank's attention-output columns (O's input)
        self.i_cols = (t0 * 64, t1 * 64)   # this rank's intermediate features (down's input)
        sd = seed * 100
        lin = lambda o, k, s, rows=None, cols=None: _mixed_linear_shard(o, k, sd + s, device, rows, cols)  # noqa: E731
        self.qkv = tq.MixedLinearGroup([lin(nh * hd, h, 1, rows=self.q_cols), lin(nkv * hd, h, 3, rows=(k0 * hd, k1 * hd)),
                                        lin(nkv * hd, h, 5, rows=(k0 * hd, k1 * hd))]).linear
        self.o = lin(h, nh * hd, 7, cols=self.q_cols)
        self.gate_up = tq.MixedLinearGroup([lin(i, h, 9, rows=self.i_cols), lin(i, h, 11, rows=self.i_cols)]).linear
        self.down = lin(h, i, 13, cols=self.i_cols)


def run_prefill_tp(args, ws, rank, device):
    """Config 2 strong-scaled over the ranks by tensor parallelism: the same block and
    total work at every N; a step = this rank's four MixedLinear forwards (quantize +
    mixed GEMM) plus the NCCL all-reduce of the O and down partial outputs."""
    import torch.distributed as dist

    from tilequant_b200 import _native as N

    full, hidden, acts, rows = _prefill_setup(device)
    ops = full.linear_ops(rows)
    shard = BlockShard(rank, ws, device)
    x_qkv, x_gu = acts["x_qkv"], acts["x_gu"]
    x_o = acts["x_o"][:, shard.q_cols[0]:shard.q_cols[1]].contiguous()
    x_down = acts["x_down"][:, shard.i_cols[0]:shard.i_cols[1]].contiguous()
    del full, acts
    torch.cuda.empty_cache()
    flush = torch.empty(int(256e6) // 4, device=device, dtype=torch.float32)

    def step(x_in=None):
        shard.qkv(x_qkv if x_in is None else x_in)
        y_o = shard.o(x_o)
        dist.all_reduce(y_o)
        shard.gate_up(x_gu)
        y_d = shard.down(x_down)
        dist.all_reduce(y_d)
        return y_d

    with torch.inference_mode():
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        _barrier(ws)
        launches0 = N.kernel_launches()
        evs = [(torch.cuda.Event(True), torch.cuda.Event(True)) for _ in range(args.steps)]
        with ClockSampler(device.index) as clocks:
            for e0, e1 in evs:
                flush.zero_()
                e0.record()
                step()
                e1.record()
            torch.cuda.synchronize()
        launches = N.kernel_launches() - launches0
        _barrier(ws)
        # the two all-reduces alone, same sizes (50 MB of BF16 each), for the split of the step
        buf = torch.zeros((rows, LLAMA3B["hidden"]), device=device, dtype=torch.bfloat16)
        for _ in range(3):
            dist.all_reduce(buf)
        torch.cuda.synchronize()
        _barrier(ws)
        a0, a1 = torch.cuda.Event(True), torch.cuda.Event(True)
        a0.record()
        for _ in range(10):
            dist.all_reduce(buf)
            dist.all_reduce(buf)
        a1.record()
        torch.cuda.synchronize()
        # e2e: the step with the hidden states copied in from pinned host memory and the
        # block's summed down output copied back, every step
        host_in = hidden.cpu().pin_memory()
        host_out = torch.empty((rows, LLAMA3B["hidden"]), dtype=torch.bfloat16).pin_memory()
        _barrier(ws)
        s0, s1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e2e_steps = max(3, args.steps // 10)
        s0.record()
        for _ in range(e2e_steps):
            y = step(host_in.to(device, non_blocking=True))
            host_out.copy_(y, non_blocking=True)
        s1.record()
        torch.cuda.synchronize()
        _barrier(ws)
    ms = _max_over_ranks(sum(e0.elapsed_time(e1) for e0, e1 in evs) / args.steps, ws)
    ar_ms = _max_over_ranks(a0.elapsed_time(a1) / 10, ws)
    e2e_ms = _max_over_ranks(s0.elapsed_time(s1) / e2e_steps, ws)
    return {
        "metric": METRIC_PREFILL, "value": round(ops / (ms * 1e-3) / 1e12, 2), "unit": "TOPS", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8 (exact i32 tile products) + bf16, f32 accumulate",
        "data": "synthetic (seeded random init)",
        "config": dict(PREFILL_CONFIG, parallelism=f"tp{ws}: Q/K/V and gate/up column-parallel (heads / tiles), "
                                                  "O and down row-parallel + NCCL all-reduce of BF16 partials"),
        "tp": {"allreduce_ms_per_step": round(ar_ms, 4), "allreduce_bytes": 2 * rows * LLAMA3B["hidden"] * 2,
               "gemm_ms_per_step": round(ms - ar_ms, 4),
               "limiter": "the two 50 MB all-reduces" if ar_ms > 0.5 * ms else "this rank's GEMMs"},
        "e2e": {"value": round(ops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TOPS",
                "h2d_bytes_per_step": hidden.numel() * 2, "d2h_bytes_per_step": hidden.numel() * 2,
                "what": "the tensor-parallel step with the hidden states copied in from pinned host memory on every "
                        "rank and the summed block output copied back"},
        "gpu_launches": launches, "clocks": clocks.summary(),
    }


# ----------------------------------------------------------------- workloads

def run_prefill(args, ws, rank, device):
    import tilequant_b200 as tq
    from tilequant_b200 import _native as N

    block, hidden, acts, rows = _prefill_setup(device)
    flush = torch.empty(int(256e6) // 4, device=device, dtype=torch.float32)  # > 2x the 126 MB L2
    ops = block.linear_ops(rows)

    def step():
        block.qkv(acts["x_qkv"])
        block.o(acts["x_o"])
        block.gate_up(acts["x_gu"])
        block.down(acts["x_down"])

    with torch.inference_mode():
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        _barrier(ws)
        torch.cuda.synchronize()
        launches0 = N.kernel_launches()
        evs = [(torch.cuda.Event(True), torch.cuda.Event(True)) for _ in range(args.steps)]
        with ClockSampler(device.index) as clocks:
            for e0, e1 in evs:
                flush.zero_()
                e0.record()
                step()
                e1.record()
            torch.cuda.synchronize()
        launches = N.kernel_launches() - launches0
        _barrier(ws)
        torch.cuda.synchronize()
    ms = _max_over_ranks(sum(e0.elapsed_time(e1) for e0, e1 in evs) / args.steps, ws)
    value = ws * ops / (ms * 1e-3) / 1e12

    # ---- dominant kernel alone: the stacked gate/up GEMM, CUDA events around it
    gu = block.gate_up
    with torch.inference_mode():
        q, sx = tq.quantize_activation_tile_absmax(acts["x_gu"])
        kw = dict(x_fp=acts["x_gu"], x_int8=q, sx=sx, out_dtype=torch.bfloat16, **gu._weights())
        y_gu = torch.empty((rows, gu.M_orig), device=device, dtype=torch.bfloat16)
        for _ in range(3):
            tq.gemm_mixed_rows_splitk(out=y_gu, **kw)
        kev = [(torch.cuda.Event(True), torch.cuda.Event(True)) for _ in range(max(5, args.steps // 4))]
        for e0, e1 in kev:
            flush.zero_()
            e0.record()
            tq.gemm_mixed_rows_splitk(out=y_gu, **kw)
            e1.record()
        torch.cuda.synchronize()
        # the same product as a dense BF16 cuBLAS GEMM of the unquantized weight, for context
        w_dense = torch.randn((gu.M_orig, gu.K_orig), device=device, dtype=torch.bfloat16)
        for _ in range(3):
            torch.matmul(acts["x_gu"], w_dense.t())
        dev_ = [(torch.cuda.Event(True), torch.cuda.Event(True)) for _ in range(5)]
        for e0, e1 in dev_:
            flush.zero_()
            e0.record()
            torch.matmul(acts["x_gu"], w_dense.t())
            e1.record()
        torch.cuda.synchronize()
        del w_dense
    k_ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in kev)
    bf16_ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in dev_)
    k_ops = 2 * rows * gu.M_orig * gu.K_orig
    peak, peak_src = _int8_peak(device)
    achieved = k_ops / (k_ms * 1e-3) / 1e12
    # outside the timed regions: the timed launch's output, checked on sampled rows
    checked = _verify_sample(acts["x_gu"], y_gu, gu, seed=rank)

    # ---- e2e: whole block through the module API, host buffers in and out
    host_in = hidden.cpu().pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    with torch.inference_mode():
        for _ in range(2):
            block.forward(hidden)
        torch.cuda.synchronize()
        e2e_steps = max(3, args.steps // 10)
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for _ in range(e2e_steps):
            out = block.forward(host_in.to(device, non_blocking=True))
            host_out.copy_(out, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1) / e2e_steps, ws)

    # ---- the whole block (attention, norms included), device resident, for context
    with torch.inference_mode():
        bev = [(torch.cuda.Event(True), torch.cuda.Event(True)) for _ in range(5)]
        for e0, e1 in bev:
            flush.zero_()
            e0.record()
            block.forward(hidden)
            e1.record()
        torch.cuda.synchronize()
    block_ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in bev)

    line = {
        "metric": METRIC_PREFILL, "value": round(value, 2), "unit": "TOPS", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8 (exact i32 tile products) + bf16, f32 accumulate",
        "data": "synthetic (seeded random init)",
        "config": dict(PREFILL_CONFIG, parallelism="tp1: the whole block on one GPU (the N = 1 point of the "
                                                   "tensor-parallel series run under torchrun)"),
        "roofline": {"kernel": "mixed GEMM, stacked gate/up (8192 x 16384 x 3072)", "bound": "tensor",
                     "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS",
                     "frac": round(achieved / peak, 3), "peak_source": peak_src, "ops_per_launch": k_ops,
                     "launch_ms": round(k_ms, 4), "traffic": _profile_traffic(GEMM_PROFILE),
                     "traffic_source": f"static: ncu capture summarised in profiles/{GEMM_PROFILE}",
                     "bf16_dense_ms": round(bf16_ms, 4),
                     "bf16_dense_what": "torch.matmul (cuBLAS) of the same activations by a dense BF16 weight "
                                        "of the same shape",
                     "frac_of_bf16_measured": round(achieved / _peaks().get("bf16_tflops", 1639.7), 3),
                     "checked_rows": checked,
                     "check": "output of the timed launch on sampled rows (every 128-row block) against the "
                              "CPU restatement (oracle/), within 1 BF16 ulp"},
        "e2e": {"value": round(ws * ops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TOPS",
                "h2d_bytes_per_step": hidden.numel() * 2, "d2h_bytes_per_step": hidden.numel() * 2,
                "what": "whole decoder block through MixedLinear modules, pinned host in/out"},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "block_ms": round(block_ms, 4),
    }
    if rank == 0 and ws == 1:
        line["cpu_baseline"] = _cpu_baseline_line(_reference_linears(), args.cpu_rows, args.cpu_seconds)
    return line


def decode_cpu_baseline(x, w, fp16, int8, n_tr, n_tc, bytes_per_call, seconds=3.0):
    """Config 1 on the host cores: the C restatement of the reference (oracle/, OpenMP,
    all host threads) quantizing the 16 tokens and running the full 3072 x 3072 mixed
    GEMM, repeated for about ``seconds``; GB/s over the same bytes per call as the GPU
    line."""
    import numpy as np  # noqa: F401  (the oracle's arrays)
    from oracle import oracle as O
    from tests.golden import inputs as I

    xb = I.bits(x)
    pk = O.pack(I.bits(w), n_tr, n_tc, int8.numpy(), fp16.numpy())
    m, k = w.shape
    threads = O.set_threads(os.cpu_count() or 1)  # all host threads, whatever the launcher set
    q, sx = O.quantize_act(xb)  # warm-up (loads the library, touches the arrays)
    O.gemm(q, sx, pk, xb, m, k, split_k=1)
    calls, spent = 0, 0.0
    while spent < seconds or calls < 3:
        t0 = time.perf_counter()
        q, sx = O.quantize_act(xb)
        O.gemm(q, sx, pk, xb, m, k, split_k=1)
        spent += time.perf_counter() - t0
        calls += 1
    return {"value": round(bytes_per_call * calls / spent / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port", "sample": f"{calls} whole config-1 calls (quantize 16 x {k} + mixed GEMM {m} x {k}) through "
                                      "oracle/tq_oracle.c (OpenMP)"}


def run_decode(args, ws, rank, device):
    """Config 1: one q_proj-shaped MixedLinear (3072 x 3072, 1 % BF16), 16 tokens."""
    import tilequant_b200 as tq
    from tests.golden import inputs as I
    from tilequant_b200 import _native as N

    x, w, fp16, int8, n_tr, n_tc = I.config1(0)
    nrot = 40  # distinct weight copies: 40 x 9.75 MB > 2x L2
    lins = []
    for _ in range(nrot):
        p = tq.pack_weight_from_tile_ids(w.to(device), n_tr=n_tr, n_tc=n_tc, int8_tile_ids=int8, fp16_tile_ids=fp16,
                                         cfg=_cfg())
        lins.append(tq.MixedLinear(p, None, _cfg()))
    xd = x.to(device)
    l0 = lins[0]
    bytes_per = (l0.int8_tiles.numel() + l0.fp16_tiles.numel() * 2 + l0.int8_scales.numel() * 4 +
                 (l0.int8_tile_ids.numel() + l0.fp16_tile_ids.numel()) * 4 + 2 * (n_tr + 1) * 4 + xd.numel() * 2 +
                 16 * 3072 * 2)
    with torch.inference_mode():
        for lin in lins:
            lin(xd)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        c0 = N.kernel_launches()
        with torch.cuda.graph(g):
            for lin in lins:
                lin(xd)
        per_replay = N.kernel_launches() - c0
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        _barrier(ws)
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        with ClockSampler(device.index) as clocks:
            e0.record()
            for _ in range(args.steps):
                g.replay()
            e1.record()
            torch.cuda.synchronize()
        _barrier(ws)
    us = _max_over_ranks(e0.elapsed_time(e1) * 1e3 / (args.steps * nrot), ws)
    gbs = ws * bytes_per / (us * 1e-6) / 1e9
    hbm = _peaks().get("hbm_gbs", 6543.1)

    # ---- e2e: the same call through the module with the 16 tokens copied in from pinned
    # host memory and the output copied back, every call (weights rotate as above)
    host_x = x.pin_memory()
    host_y = torch.empty((16, 3072), dtype=torch.bfloat16).pin_memory()
    with torch.inference_mode():
        for lin in lins[:3]:
            host_y.copy_(lin(host_x.to(device, non_blocking=True)), non_blocking=True)
        torch.cuda.synchronize()
        _barrier(ws)
        s0, s1 = torch.cuda.Event(True), torch.cuda.Event(True)
        s0.record()
        for _ in range(max(1, args.steps // 10)):
            for lin in lins:
                host_y.copy_(lin(host_x.to(device, non_blocking=True)), non_blocking=True)
        s1.record()
        torch.cuda.synchronize()
    e2e_us = _max_over_ranks(s0.elapsed_time(s1) * 1e3 / (max(1, args.steps // 10) * nrot), ws)
    cpu = decode_cpu_baseline(x, w, fp16, int8, n_tr, n_tc, bytes_per) if (ws == 1 and rank == 0) else None
    return {
        "metric": "mixed tile GEMM GB/s: config 1 (q_proj 3072x3072, 16 tokens, 1 % BF16), quantize+GEMM",
        "value": round(gbs, 1), "unit": "GB/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(us * nrot / 1e3, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 + bf16", "data": "synthetic (seeded random init)",
        "config": {"workload": "config1: one MixedLinear decode", "rows": 16, "bytes_per_call": bytes_per,
                   "calls_per_step": nrot, "l2": "40 distinct weight copies per step (> 2x L2)",
                   "graph": "one CUDA graph of 40 calls per step"},
        "roofline": {"bound": "hbm", "achieved": round(gbs / ws, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(gbs / ws / hbm, 3), "traffic": _profile_traffic(DECODE_PROFILE),
                     "us_per_call": round(us, 3),
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs"},
        "gpu_launches": per_replay * args.steps,
        "clocks": clocks.summary(),
        "e2e": {"value": round(ws * bytes_per / (e2e_us * 1e-6) / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": nrot * 16 * 3072 * 2, "d2h_bytes_per_step": nrot * 16 * 3072 * 2,
                "what": "MixedLinear calls with pinned host tokens in and outputs out, eagerly launched"},
        **({"cpu_baseline": cpu} if cpu is not None else {}),
    }


def run_gemm(args, ws, rank, device):
    """One mixed tile GEMM launch per step (activations already quantized), the shape
    given by --shape ROWSxMxK (default: the stacked gate/up GEMM of config 2)."""
    import tilequant_b200 as tq
    from tests.golden import inputs as I
    from tilequant_b200 import _native as N

    rows, m, k = (int(v) for v in args.shape.lower().split("x"))
    w = I.weight(m, k, 3).to(device)
    n_tr, n_tc = (m + 63) // 64, (k + 63) // 64
    fp16 = I.keep_ids(n_tr, n_tc, args.keep, 4)
    pack = tq.pack_weight_from_tile_ids(w, n_tr=n_tr, n_tc=n_tc, int8_tile_ids=I.complement_ids(fp16, n_tr * n_tc),
                                        fp16_tile_ids=fp16, cfg=_cfg())
    x = I.activations(rows, k, 5).to(device)
    q, sx = tq.quantize_activation_tile_absmax(x)
    kw = dict(x_fp=x, x_int8=q, sx=sx, int8_tiles=pack.int8_tiles, int8_scales=pack.int8_scales,
              int8_tile_ids=pack.int8_tile_ids, int8_row_ptr=pack.int8_row_ptr, fp16_tiles=pack.fp16_tiles,
              fp16_tile_ids=pack.fp16_tile_ids, fp16_row_ptr=pack.fp16_row_ptr, M=m, K=k, n_tr=n_tr, n_tc=n_tc,
              out_dtype=torch.bfloat16)
    flush = torch.empty(int(256e6) // 4, device=device, dtype=torch.float32)
    out = torch.empty((rows, m), device=device, dtype=torch.bfloat16)
    with torch.inference_mode():
        for _ in range(args.warmup):
            tq.gemm_mixed_rows_splitk(out=out, **kw)
        torch.cuda.synchronize()
        _barrier(ws)
        launches0 = N.kernel_launches()
        evs = [(torch.cuda.Event(True), torch.cuda.Event(True)) for _ in range(args.steps)]
        with ClockSampler(device.index) as clocks:
            for e0, e1 in evs:
                flush.zero_()
                e0.record()
                tq.gemm_mixed_rows_splitk(out=out, **kw)
                e1.record()
            torch.cuda.synchronize()
        launches = N.kernel_launches() - launches0
        _barrier(ws)
    ms = _max_over_ranks(statistics.median(e0.elapsed_time(e1) for e0, e1 in evs), ws)
    ops = 2 * rows * m * k
    peak, peak_src = _int8_peak(device)
    achieved = ops / (ms * 1e-3) / 1e12
    return {
        "metric": f"mixed tile GEMM TOPS ({rows}x{m}x{k}, {args.keep:.0%} BF16 tiles)", "value": round(ws * achieved, 1),
        "unit": "TOPS", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 + bf16, f32 accumulate",
        "data": "synthetic (seeded random init)",
        "config": {"workload": "one mixed GEMM launch", "rows": rows, "M": m, "K": k, "keep_bf16": args.keep,
                   "l2": "flushed (256 MB write) between timed steps"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS",
                     "frac": round(achieved / peak, 3), "peak_source": peak_src, "traffic": None},
        "gpu_launches": launches, "clocks": clocks.summary(),
    }


GEN_MODELS = {
    # config 3: Llama-3.2-3B, 1 % BF16 tiles, batch 4, prompt 2048, 256 new tokens
    "llama3b": dict(arch="llama", hidden=3072, inter=8192, layers=28, heads=24, kv_heads=8, head_dim=128,
                    vocab=128256, tie=True, rope_theta=500000.0, keep=0.01, batch=4, prompt=2048, new=256),
    # config 4: Qwen2.5-7B, 10 % BF16 tiles, batch 16, prompt 1024, 256 new tokens
    "qwen7b": dict(arch="qwen2", hidden=3584, inter=18944, layers=28, heads=28, kv_heads=4, head_dim=128,
                   vocab=152064, tie=False, rope_theta=1000000.0, keep=0.10, batch=16, prompt=1024, new=256),
    # config 5: Qwen2.5-14B, 20 % BF16 tiles chosen by IAA from 64 x 2048 random ids, batch 64, prompt
    # 1024, 256 new tokens
    "qwen14b": dict(arch="qwen2", hidden=5120, inter=13824, layers=48, heads=40, kv_heads=8, head_dim=128,
                    vocab=152064, tie=False, rope_theta=1000000.0, keep=0.20, batch=64, prompt=1024, new=256,
                    calib="iaa", calib_seqs=64, calib_len=2048),
}


def build_generation_model(spec, device, seed=0, tp=None, exchange=None):
    """Random-init decoder of the given architecture on `device` (bf16), projections
    replaced by MixedLinear with uniformly random tile maps; with tp = (rank, world,
    group), this rank's tensor-parallel shard of it (the same full model and maps on
    every rank), its decode-sized row-parallel sums in the GEMM when `exchange` (a
    connected PeerExchange) is given."""
    from tilequant_b200.apply import apply_random_tile_maps
    from tilequant_b200.parallel import projection_shapes, seeded_random_keep, tensor_parallel_

    common = dict(hidden_size=spec["hidden"], intermediate_size=spec["inter"], num_hidden_layers=spec["layers"],
                  num_attention_heads=spec["heads"], num_key_value_heads=spec["kv_heads"],
                  vocab_size=spec["vocab"], tie_word_embeddings=spec["tie"], rope_theta=spec["rope_theta"],
                  max_position_embeddings=max(4096, spec["prompt"] + spec["new"]), attn_implementation="sdpa")
    if spec["arch"] == "llama":
        from transformers import LlamaConfig as Cfg, LlamaForCausalLM as Model

        common["head_dim"] = spec["head_dim"]
    else:
        from transformers import Qwen2Config as Cfg, Qwen2ForCausalLM as Model
    torch.manual_seed(seed)
    with torch.device(device):
        model = Model(Cfg(**common)).to(torch.bfloat16).eval()
    if spec.get("calib") == "iaa":
        # IAA tile importance on the GPU over seeded random token ids, then the top tiles
        # per projection stay 16-bit and the INT8 scales use the IAA search
        from tilequant_b200.apply import apply_tile_maps, default_cfg
        from tilequant_b200.calibrate import collect_iaa_tile_scores_with_channel_stats, keep_ids_from_scores
        from tilequant_b200.rules import TARGET_SUFFIXES

        gen = torch.Generator().manual_seed(seed + 7)
        per = 4
        batches = [{"input_ids": torch.randint(0, spec["vocab"], (per, spec["calib_len"]), generator=gen)}
                   for _ in range(spec["calib_seqs"] // per)]
        scores, stats = collect_iaa_tile_scores_with_channel_stats(
            model, batches, lambda n: n.endswith(TARGET_SUFFIXES), {"calib": {}})
        kept = keep_ids_from_scores(scores, spec["keep"])
        cfg = default_cfg(quant_style="iaa")
        if tp is None:
            apply_tile_maps(model, kept, cfg, model_type=spec["arch"], iaa_channel_stats=stats)
        else:
            tensor_parallel_(model, tp[0], tp[1], lambda n, n_tr, n_tc: kept[n], cfg, group=tp[2],
                             model_type=spec["arch"], iaa_channel_stats=stats, exchange=exchange)
    elif tp is None:
        apply_random_tile_maps(model, spec["keep"], seed=seed + 1, model_type=spec["arch"])
    else:
        keep = seeded_random_keep(spec["keep"], seed + 1, list(projection_shapes(model)))
        tensor_parallel_(model, tp[0], tp[1], keep, group=tp[2], model_type=spec["arch"], exchange=exchange)
    torch.cuda.empty_cache()
    return model


def run_generate(args, ws, rank, device):
    """Configs 3-5: greedy generation with the CUDA-graph decoder; decode tokens/s,
    TTFT and TPOT (median over the timed requests)."""
    from tilequant_b200.graph_decode import CudaGraphGreedyDecoder

    spec = dict(GEN_MODELS[args.model])
    tp = args.tp and ws > 1
    exchange = None
    if tp and args.allreduce == "peer":
        from tilequant_b200.peer import PeerExchange

        exchange = PeerExchange(device, ws, rank).connect()
    model = build_generation_model(spec, device, tp=(rank, ws, None) if tp else None, exchange=exchange)
    B, P, T = spec["batch"], spec["prompt"], spec["new"]
    from tilequant_b200 import _native as N

    dec = CudaGraphGreedyDecoder.prepare(model, prompt_tokens=P, max_new_tokens=T, batch_size=B, device=device)
    # graph replays launch the captured kernels; an uncaptured (eager) prefill is counted live
    per_request = dec.captured_launches["prefill"] + (T - 1) * dec.captured_launches["decode"]
    layers = spec["layers"]
    gen = torch.Generator().manual_seed(1234)
    prompts = [torch.randint(0, spec["vocab"], (B, P), generator=gen).pin_memory()
               for _ in range(args.warmup + args.steps)]
    host_out = torch.empty((B, T), dtype=torch.long).pin_memory()
    ttft, dec_ms, tot_ms = [], [], []
    eager_launches = 0
    with ClockSampler(device.index) as clocks:
        for i, prompt in enumerate(prompts):
            _barrier(ws)
            torch.cuda.synchronize()
            e0, e1, e2 = (torch.cuda.Event(True) for _ in range(3))
            n0 = N.kernel_launches()
            e0.record()
            dec.prefill(prompt)
            e1.record()
            if i >= args.warmup:
                eager_launches += N.kernel_launches() - n0
            ids = dec.decode(T - 1)
            e2.record()
            host_out.copy_(ids, non_blocking=True)
            torch.cuda.synchronize()
            if i >= args.warmup:
                ttft.append(e0.elapsed_time(e1))
                dec_ms.append(e1.elapsed_time(e2))
                tot_ms.append(e0.elapsed_time(e2))
    dec.close()
    peer_status = None
    if exchange is not None:  # every rank takes the same collective steps, whatever its status
        peer_status = int(_max_over_ranks(float(exchange.status()), ws))
        _barrier(ws)
        exchange.close()
    t_med = statistics.median(tot_ms)
    d_med = _max_over_ranks(statistics.median(dec_ms), ws)
    t_med = _max_over_ranks(t_med, ws)
    jobs = 1 if tp else ws  # tensor parallel: one job over all ranks; else one replica per rank
    value = jobs * B * (T - 1) / (d_med * 1e-3)
    return {
        "metric": f"decode tokens/s: {args.model} greedy generation (batch {B}, prompt {P}, {T} new tokens), "
                  "CUDA-graph decode", "value": round(value, 1), "unit": "tokens/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_med, 3), "higher_is_better": True,
        "scaling": "strong" if tp else "weak", "vs_baseline": None,
        "dtype": "int8 + bf16 projections, bf16 elsewhere",
        "data": "synthetic (random-init weights and token ids; tile maps " +
                ("by IAA on the GPU over 64 x 2048 random ids)" if spec.get("calib") == "iaa" else "uniform random)"),
        "config": {"workload": f"config {'3' if args.model == 'llama3b' else ('4' if args.model == 'qwen7b' else '5')}:"
                               f" {args.model}", "layers": layers, "keep_bf16": spec["keep"], "batch": B,
                   "prompt": P, "new_tokens": T,
                   "parallelism": (f"tp{ws} (" + ("O/down sums inside the decode GEMM over NVLink where the "
                                                  "decode grid fits (<= 64 rows), "
                                                  "NCCL all-reduce otherwise)" if exchange is not None else
                                                  "NCCL all-reduce after O and down)")) if tp else f"replicas x{ws}",
                   "l2": "weights (GBs) and KV cache exceed L2 every step"},
        "ttft_ms_p50": round(statistics.median(ttft), 3), "tpot_ms_p50": round(d_med / (T - 1), 4),
        "e2e": {"value": round(jobs * B * T / (t_med * 1e-3), 1), "unit": "tokens/s (prefill + decode)",
                "h2d_bytes_per_step": B * P * 8, "d2h_bytes_per_step": B * T * 8},
        "gpu_launches": per_request * args.steps + eager_launches,
        "gpu_launches_per_graph": dec.captured_launches, "prefill_captured": dec.prefill_captured,
        **({} if peer_status is None else {"peer_sum_status": peer_status}),
        "clocks": clocks.summary(),
    }


def run_reference(args, ws, rank):
    """The reference arm: the reference's arithmetic on the host cores (the C
    restatement in oracle/, all host threads), on config 2.  The reference's own GEMM
    is a Triton GPU kernel and its Python sources do not travel to the GPU box, so the
    restatement stands in for it.  Nothing here loads this project's GPU library or
    touches a GPU: the packs are built by the restatement from the same seeded weights
    and tile maps as the GPU run.  Each step is one window of --cpu-rows consecutive
    rows of each linear's 8192-row input (the windows walk through the batch),
    quantized and multiplied as one call."""
    if rank != 0:
        return None
    from oracle import oracle as O

    # all host threads: torchrun hands every rank OMP_NUM_THREADS=1, and rank 0 runs alone
    threads = O.set_threads(os.cpu_count() or 1)
    linears = _reference_linears()
    for w in range(args.warmup):
        _cpu_sample(linears, args.cpu_rows, w)
    secs, ops = 0.0, 0
    for i in range(args.steps):
        s, o = _cpu_sample(linears, args.cpu_rows, args.warmup + i)
        secs += s
        ops += o
    value = ops / secs / 1e12
    sample = (f"per step one window of {args.cpu_rows} consecutive rows (of 8192) through the 4 config-2 linears, "
              "quantized and multiplied as one call by oracle/tq_oracle.c (OpenMP, all host threads); weights and "
              "tile maps as the GPU run (same seeds), seeded N(0,1) inputs")
    return {
        "impl": "reference", "metric": METRIC_PREFILL, "value": value, "unit": "TOPS", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8 + bf16 (CPU)",
        "data": "synthetic (seeded random init)",
        "config": dict(PREFILL_CONFIG, parallelism="one host, all cores"),
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def _extras(args, device):
    """The default (prefill) line also carries the decode-side numbers: config 1's
    decode GEMM (GB/s against HBM) and config 3's greedy generation (tokens/s, TTFT,
    TPOT), each run with its own short step count."""
    out = {}
    sub = argparse.Namespace(**vars(args))
    sub.steps, sub.warmup = 20, 3
    d = run_decode(sub, 1, 0, device)
    out["decode"] = {"what": d["metric"], "value": d["value"], "unit": d["unit"], "us_per_call": d["roofline"]["us_per_call"],
                     "frac_of_hbm": d["roofline"]["frac"], "hbm_peak_gbs": d["roofline"]["peak"],
                     "e2e_gbs": d["e2e"]["value"], "cpu_baseline": d.get("cpu_baseline"), "clocks": d["clocks"]}
    torch.cuda.empty_cache()
    sub.steps, sub.warmup, sub.model, sub.tp = 3, 2, "llama3b", False
    gl = run_generate(sub, 1, 0, device)
    out["generate"] = {"what": gl["metric"], "tokens_per_s": gl["value"], "ttft_ms_p50": gl["ttft_ms_p50"],
                       "tpot_ms_p50": gl["tpot_ms_p50"], "e2e_tokens_per_s": gl["e2e"]["value"],
                       "requests_timed": 3, "clocks": gl["clocks"]}
    torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["prefill", "decode", "gemm", "generate"], default="prefill")
    ap.add_argument("--model", choices=sorted(GEN_MODELS), default="llama3b", help="model of --workload generate")
    ap.add_argument("--tp", action="store_true", help="--workload generate: tensor parallel over the ranks")
    ap.add_argument("--allreduce", choices=["peer", "nccl"], default="peer",
                    help="--tp: row-parallel sums of decode calls inside the GEMM (peer) or by NCCL")
    ap.add_argument("--shape", default="8192x16384x3072", help="ROWSxMxK of --workload gemm")
    ap.add_argument("--keep", type=float, default=KEEP, help="BF16 tile fraction of --workload gemm")
    ap.add_argument("--cpu-rows", type=int, default=256, help="rows per linear in one CPU window")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline leg: seconds of windows")
    ap.add_argument("--no-extras", action="store_true",
                    help="prefill: skip the decode (config 1) and generation (config 3) sub-objects")
    args = ap.parse_args()
    ws, rank, local = _dist()
    if args.impl == "reference":
        line = run_reference(args, ws, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if ws > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    run = {"decode": run_decode, "gemm": run_gemm, "prefill": run_prefill, "generate": run_generate}[args.workload]
    if args.workload == "prefill" and ws > 1:
        run = run_prefill_tp
    line = run(args, ws, rank, device)
    if args.workload == "prefill" and ws == 1 and not args.no_extras:
        line.update(_extras(args, device))
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
