"""Host logic of the generation benchmark tool (no GPU)."""

from tilequant_b200.benchmark_generation import REPEATS, WARMUPS, prompt_tokens, summarize


def test_protocol_constants():
    assert (WARMUPS, REPEATS) == (2, 5)  # examples/benchmark_generation.py:34


def test_prompt_without_tokenizer(tmp_path):
    toks = prompt_tokens(tmp_path, 250)
    assert len(toks) == 250 and toks[:3] == [1, 2, 3] and toks[100] == 1


def test_summarize_medians_and_energy():
    rows = [{"ttft_ms": t, "tpot_ms": 2 * t, "output_tok_s": 10 * t, "energy_j_per_1k_tokens": e,
             "peak_allocated_gib": p} for t, e, p in [(3, 1.0, 2.0), (1, 2.0, 5.0), (2, 3.0, 1.0)]]
    s = summarize(rows)
    assert (s["ttft_ms"], s["tpot_ms"], s["output_tok_s"], s["energy_j_per_1k_tokens"], s["peak_allocated_gib"]) == \
        (2, 4, 20, 2.0, 5.0)
    rows[0]["energy_j_per_1k_tokens"] = None
    assert "energy_j_per_1k_tokens" not in summarize(rows)
