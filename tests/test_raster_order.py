"""Host side of the raster-order layout (``raster_order`` / ``RasterOrder``),
on the oracle's plans (no GPU): every physical 64-token image block of a plan is
an aligned 8x8 square, the block origins describe it, ``rows()`` is a
permutation of the raster rows that keeps each block's token set, and a plan
whose blocks are not squares is refused."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from hilberta_b200.paired_kernel import RasterOrder, raster_order
from oracle import plan_oracle as po


@pytest.mark.parametrize("grid,tiles,k,shared", [(32, 4, 1, False), (64, 16, 3, False), (64, 4, 1, True), (128, 16, 3, False)])
def test_raster_order_of_oracle_plans(grid, tiles, k, shared):
    ref = po.bridge_k_plan(tiles, k, shared, grid_size=grid)
    order = np.asarray(ref["image_order"] if isinstance(ref, dict) else ref.image_order)
    plan = SimpleNamespace(text_tokens=512, image_order=torch.as_tensor(order))
    ro = raster_order(plan, "cpu")
    assert ro.grid == grid and ro.text_tokens == 512 and ro.block_origin.dtype == torch.int32
    rows = ro.rows().numpy()
    assert sorted(rows.tolist()) == list(range(512 + grid * grid))
    assert np.array_equal(rows[:512], np.arange(512))
    # same token set per block as the plan's physical order (only the order inside a square differs)
    phys = 512 + order.reshape(-1, 64)
    assert np.array_equal(np.sort(rows[512:].reshape(-1, 64), axis=1), np.sort(phys, axis=1))


def test_raster_order_rejects_non_square_blocks():
    g = 32
    order = torch.arange(g * g)  # plain raster: a 64-token block is two image rows, not a square
    with pytest.raises(ValueError, match="not aligned 8x8 squares"):
        raster_order(SimpleNamespace(text_tokens=512, image_order=order), "cpu")
    with pytest.raises(ValueError, match="square image"):
        raster_order(SimpleNamespace(text_tokens=500, image_order=order), "cpu")


def test_raster_order_rows_of_a_hand_built_layout():
    ro = RasterOrder(64, 8, torch.tensor([0], dtype=torch.int32))  # one 8x8 image after 64 text tokens
    assert torch.equal(ro.rows(), torch.arange(128, dtype=torch.int32))
