"""Top-k tile selection of the calibration decisions, against the reference's own
outputs (tests/golden/calib.npz), on the CPU."""

from pathlib import Path

import numpy as np
import pytest
import torch

from tilequant_b200.calibrate import keep_ids_from_scores, topk_mask

CALIB = np.load(Path(__file__).resolve().parent / "golden" / "calib.npz")


@pytest.mark.parametrize("i", range(4))
def test_topk_mask_matches_reference(i):
    m = topk_mask(CALIB[f"topk{i}__imp"], float(CALIB[f"topk{i}__frac"][0]))
    np.testing.assert_array_equal(m, CALIB[f"topk{i}__mask"])


def test_topk_keeps_at_least_one_and_all():
    imp = np.arange(12, dtype=np.float32).reshape(3, 4)
    assert topk_mask(imp, 0.0).sum() == 1 and topk_mask(imp, 0.0).reshape(-1)[-1] == 1
    assert topk_mask(imp, 1.0).sum() == 12


def test_keep_ids_from_scores():
    s = {"a": torch.tensor([[0.1, 5.0], [3.0, 0.2]])}
    ids = keep_ids_from_scores(s, 0.5)["a"]
    assert ids.dtype == torch.int32 and ids.tolist() == [1, 2]
