"""Greedy-generation latency, throughput and energy for one (prompt, output, batch)
shape, with the protocol of the reference's examples/benchmark_generation.py:34-155:
a fixed token prompt of length P repeated B times, two warm-up and five timed
requests, median TTFT (request through first token), TPOT (following tokens) and
output tokens/s, NVML energy per 1K generated tokens (the counter is read, never
changed), and the maximum peak allocated memory.  ``--method tilequant`` loads the
checkpoint with its tile maps (``loader.py``) and decodes with the CUDA-graph decoder;
``--method bf16`` runs the dense model eagerly, as the reference does.

    python -m tilequant_b200.benchmark_generation --model_dir /path/to/Llama-3.2-3B-Instruct \\
        --decision_root Decision --quant_style gi --keep_tag keep01 --prompt 2048 --output 256 --batch 4
"""

from __future__ import annotations

import argparse
import json
import statistics
import time
from pathlib import Path
from typing import List, Optional, Sequence

import torch

WARMUPS, REPEATS = 2, 5
PROMPT_TEXT = "Tile-level mixed-precision quantization benchmark. "


def prompt_tokens(model_dir, length: int) -> List[int]:
    """The benchmark prompt: PROMPT_TEXT's tokens repeated to ``length`` after BOS.  A
    checkpoint without a tokenizer gets the ids 1, 2, ..., 100 repeated instead."""
    try:
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(str(model_dir))
        pattern = tok(PROMPT_TEXT, add_special_tokens=False).input_ids
        bos = [tok.bos_token_id] if tok.bos_token_id is not None else []
    except (OSError, ValueError, TypeError):
        pattern, bos = list(range(1, 101)), []
    return bos + (pattern * (length // len(pattern) + 1))[: length - len(bos)]


def load_model(args, device: torch.device) -> torch.nn.Module:
    if args.method == "bf16":
        from transformers import AutoModelForCausalLM

        model = AutoModelForCausalLM.from_pretrained(args.model_dir, dtype=torch.bfloat16, attn_implementation="sdpa")
        model = model.to(device)
    else:
        from .decisions import infer_model_type
        from .loader import ApplyConfig, TileConfig, load_mixed_precision_model_from_masks

        decision = Path(args.decision_root) / Path(args.model_dir).name / args.quant_style
        model_type = infer_model_type(Path(args.model_dir))
        apply_cfg = ApplyConfig(model_type=model_type, dtype_out="bf16", tile=TileConfig(64, 64), module_filters=[],
                                quant_style=args.quant_style,
                                iaa_channel_stats_path=(str(decision / "iaa_channel_mean_abs.npz")
                                                        if args.quant_style == "iaa" else None))
        model, _ = load_mixed_precision_model_from_masks(Path(args.model_dir), decision / "tile_masks" / args.keep_tag,
                                                         apply_cfg, torch.bfloat16, device, attn_implementation="sdpa")
    model.eval()
    model.config.use_cache = True
    return model


def _energy_mj(handle) -> Optional[int]:
    if handle is None:
        return None
    import pynvml

    return int(pynvml.nvmlDeviceGetTotalEnergyConsumption(handle))


@torch.inference_mode()
def eager_request(model, tokens, batch, output_tokens, handle, device):
    torch.cuda.synchronize(device)
    torch.cuda.reset_peak_memory_stats(device)
    e0 = _energy_mj(handle)
    start = time.perf_counter()
    inputs = torch.tensor([tokens] * batch, device=device)
    out = model(input_ids=inputs, use_cache=True, logits_to_keep=1)
    current, cache = out.logits[:, -1:].argmax(-1), out.past_key_values
    torch.cuda.synchronize(device)
    first = time.perf_counter()
    for _ in range(output_tokens - 1):
        out = model(input_ids=current, past_key_values=cache, use_cache=True, logits_to_keep=1)
        current, cache = out.logits[:, -1:].argmax(-1), out.past_key_values
    torch.cuda.synchronize(device)
    return start, first, time.perf_counter(), e0, _energy_mj(handle)


@torch.inference_mode()
def graph_request(decoder, tokens, batch, output_tokens, handle, device):
    torch.cuda.synchronize(device)
    torch.cuda.reset_peak_memory_stats(device)
    e0 = _energy_mj(handle)
    start = time.perf_counter()
    decoder.prefill([tokens] * batch)
    torch.cuda.synchronize(device)
    first = time.perf_counter()
    decoder.decode(output_tokens - 1)
    torch.cuda.synchronize(device)
    return start, first, time.perf_counter(), e0, _energy_mj(handle)


def summarize(rows: Sequence[dict]) -> dict:
    """Medians of the timed requests (energy only when every request has it) and the
    maximum peak allocation."""
    out = {k: statistics.median(r[k] for r in rows) for k in ("ttft_ms", "tpot_ms", "output_tok_s")}
    if all(r["energy_j_per_1k_tokens"] is not None for r in rows):
        out["energy_j_per_1k_tokens"] = statistics.median(r["energy_j_per_1k_tokens"] for r in rows)
    out["peak_allocated_gib"] = max(r["peak_allocated_gib"] for r in rows)
    return out


def run(args) -> dict:
    device = torch.device("cuda", torch.cuda.current_device())
    try:
        import pynvml

        pynvml.nvmlInit()
        handle = pynvml.nvmlDeviceGetHandleByIndex(device.index)
    except Exception:  # no NVML or no energy counter: energy is left out
        handle = None
    tokens = prompt_tokens(args.model_dir, args.prompt)
    model = load_model(args, device)
    decoder = None
    if args.method == "tilequant":
        from .graph_decode import CudaGraphGreedyDecoder

        decoder = CudaGraphGreedyDecoder.prepare(model, prompt_tokens=args.prompt, max_new_tokens=args.output,
                                                 batch_size=args.batch, device=device)
        request = lambda: graph_request(decoder, tokens, args.batch, args.output, handle, device)  # noqa: E731
    else:
        request = lambda: eager_request(model, tokens, args.batch, args.output, handle, device)  # noqa: E731
    try:
        for _ in range(WARMUPS):
            request()
        rows = []
        for _ in range(REPEATS):
            start, first, end, e0, e1 = request()
            rows.append({
                "ttft_ms": (first - start) * 1000,
                "tpot_ms": (end - first) * 1000 / max(args.output - 1, 1),
                "output_tok_s": args.batch * args.output / (end - start),
                "energy_j_per_1k_tokens": (e1 - e0) / (args.batch * args.output) if e0 is not None else None,
                "peak_allocated_gib": torch.cuda.max_memory_allocated(device) / 2**30,
            })
    finally:
        if decoder is not None:
            decoder.close()
    return {**vars(args), **summarize(rows)}


def main(argv: Optional[Sequence[str]] = None) -> dict:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--model_dir", required=True)
    parser.add_argument("--decision_root", default="Decision", help="directory holding <model>/<style>/tile_masks")
    parser.add_argument("--method", choices=["tilequant", "bf16"], default="tilequant")
    parser.add_argument("--quant_style", choices=["gi", "iaa"], default="gi")
    parser.add_argument("--keep_tag", default="keep01")
    parser.add_argument("--prompt", type=int, default=2048)
    parser.add_argument("--output", type=int, default=256)
    parser.add_argument("--batch", type=int, default=1)
    result = run(parser.parse_args(argv))
    print(json.dumps(result, indent=1))
    return result


if __name__ == "__main__":
    main()
