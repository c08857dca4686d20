"""The generation benchmark tool end to end on a tiny saved checkpoint with a decision
directory: both methods run the reference's protocol and report its fields."""

from __future__ import annotations

import numpy as np
import pytest

from tests.loader_fixtures import save_checkpoint, tiny_model
from tilequant_b200.benchmark_generation import main
from tilequant_b200.decisions import save_masks
from tilequant_b200.rules import iter_target_linears

pytestmark = pytest.mark.gpu


def test_benchmark_generation_both_methods(cuda_device, tmp_path):
    dense = tiny_model("llama", tie=True)
    ckpt = save_checkpoint(dense, tmp_path / "tiny-llama", sharded=False)
    rng = np.random.default_rng(1)
    scores = {}
    for _, _, name, lin in iter_target_linears(dense, {}, model_type="llama"):
        m, k = lin.weight.shape
        scores[name.replace(".", "_")] = rng.random(((m + 63) // 64, (k + 63) // 64)).astype(np.float32)
    save_masks(tmp_path / "Decision" / "tiny-llama" / "gi", scores, [0.01], "tiny", "synthetic", "-", "gi")
    common = ["--model_dir", str(ckpt), "--decision_root", str(tmp_path / "Decision"), "--prompt", "32",
              "--output", "8", "--batch", "2"]
    for method in ("tilequant", "bf16"):
        res = main(common + ["--method", method])
        assert res["method"] == method
        assert res["ttft_ms"] > 0 and res["tpot_ms"] > 0 and res["output_tok_s"] > 0
        assert res["peak_allocated_gib"] > 0
