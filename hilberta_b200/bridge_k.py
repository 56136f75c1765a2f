"""Top-K reciprocal block bridges (API of ``hilberta/bridge_k.py``), built on the device."""

from __future__ import annotations

from .plan import AttentionPlan, PhasePlan, _build


def bridge_k_plan(tiles=4, k=1, shared=False, *, grid_size=64, device=None):
    """``hilberta/bridge_k.py:10-51``: the base plan (no bridge) plus, per phase,
    each block's top-K bridge blocks by cut-edge score with the phase-rolled
    tie-break, the block adjacency closed under transpose (reciprocal), rows
    re-emitted ascending.  ``bridge_original_blocks`` is int64 [nb, K], -1 padded.
    """
    if isinstance(k, bool) or k not in (1, 2, 3, 4):
        raise ValueError("This bounded comparison supports integer K=1..4")
    if isinstance(tiles, bool) or int(tiles) != tiles or tiles <= 0:
        raise ValueError("tile_count must be a positive integer")
    if isinstance(grid_size, bool) or int(grid_size) != grid_size or grid_size <= 0:
        raise ValueError("grid_size must be a positive integer")
    if grid_size < 8 or int(grid_size) & (int(grid_size) - 1):
        raise ValueError("grid_size must be a power of two >= 8")
    r = _build(int(tiles), int(grid_size), 512, shared, int(k), 1, 64, device)
    phases = tuple(PhasePlan(off, ids, cnt, br) for off, ids, cnt, br in r["phases"])
    return AttentionPlan(
        int(grid_size),
        int(tiles),
        512,
        r["shared_tokens"],
        64,
        r["image_order"],
        r["inverse_image_order"],
        r["original_order"],
        r["physical_original_blocks"],
        phases,
        True,
    )
