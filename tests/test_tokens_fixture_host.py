"""The greedy-token fixture's models rebuild bit-identically from their seeds on the CPU
(the GPU test builds them the same way before moving them to the device), and the rows
the fixture requires to match lead by the stated margin at every step."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from tests.golden import tiny_models as T

FIX = np.load(Path(__file__).resolve().parent / "golden" / "tokens.npz")


@pytest.mark.parametrize("name", sorted(T.MODELS))
def test_tiny_model_rebuilds_from_seed(name):
    model = T.build(T.MODELS[name])
    assert T.state_sha(model) == str(FIX[f"{name}__state_sha"])


@pytest.mark.parametrize("name", sorted(T.MODELS))
def test_required_rows_have_margin(name):
    rows = FIX[f"{name}__rows"]
    margins = FIX[f"{name}__margins"]
    assert rows.size >= 4
    assert (margins[rows] >= T.MIN_MARGIN_ULPS).all()
    assert FIX[f"{name}__tokens"].shape == (T.BATCH, T.NEW_TOKENS)
