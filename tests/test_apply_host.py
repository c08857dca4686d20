"""Host logic of the tile-map application (no GPU)."""

import torch

from tilequant_b200.apply import complement_ids, default_cfg, random_keep_ids


def test_random_keep_ids_counts_and_order():
    g = torch.Generator().manual_seed(0)
    ids = random_keep_ids(48, 48, 0.01, g)
    assert ids.dtype == torch.int32 and ids.numel() == 24  # ceil(0.01 * 2304)
    assert torch.all(ids[1:] > ids[:-1]) and int(ids.min()) >= 0 and int(ids.max()) < 2304
    assert random_keep_ids(3, 3, 1.0, g).tolist() == list(range(9))
    assert random_keep_ids(3, 3, 0.0, g).numel() == 0


def test_complement_ids():
    keep = torch.tensor([5, 0, 7], dtype=torch.int32)
    assert complement_ids(keep, 9).tolist() == [1, 2, 3, 4, 6, 8]
    assert complement_ids(torch.zeros(0, dtype=torch.int32), 3).tolist() == [0, 1, 2]


def test_default_cfg():
    cfg = default_cfg(quant_style="iaa")
    assert (cfg.tile_m, cfg.tile_n, cfg.quant_style, cfg.dtype_out) == (64, 64, "iaa", "bf16")
