"""bench.py's end-to-end loop derives the deep-supervision targets on the device as
the labels at all-multiple positions; at the heads' power-of-two sizes that equals
the nearest interpolation the timed step's targets are built with (CPU only)."""

from __future__ import annotations

import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402


def test_strided_labels_equal_nearest_downsampling():
    gen = torch.Generator().manual_seed(0)
    for spatial in (32, 64):
        target = torch.randint(0, 3, (1, spatial, spatial, spatial), generator=gen)
        want = bench.downsampled_targets(target)
        for size, t in want.items():
            f = spatial // size[0]
            got = target.to(torch.uint8).long()[:, ::f, ::f, ::f]
            assert got.shape == t.shape and torch.equal(got, t), (spatial, size)
