"""CPU restatement (numpy) of HilbertA's static plan / metadata builders.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (``hilberta_b200``)
imports this module: it exists so ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg can check the CUDA metadata builder bit for bit.

Parity pin: every function here is checked against golden vectors produced by
running the reference implementation itself (``tests/golden/make_golden.py``
imports ``hilberta.geometry/plan/bridge_k/paired_metadata`` from the reference
checkout and stores full arrays for small plans and sha256 digests for the
BASELINE-sized ones), and against the reference's own known-answer constants
(``tests/test_plan.py:54-59``, ``tests/test_paired_metadata.py:46-55``).

All citations are ``path:line`` inside the reference project (wenboluu/hilberta).
Integer-only; results are exact.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


# --------------------------------------------------------------------------
# geometry.py
# --------------------------------------------------------------------------
def hilbert_order(grid_size: int) -> np.ndarray:
    """Raster id of the Hilbert walk's d-th cell, vertically flipped.

    Restates ``hilberta/geometry.py:6-25``: per level s = 1, 2, 4, ...:
    rx = (t >> 1) & 1, ry = (t ^ rx) & 1; when ry == 0 the quadrant is
    reflected (if rx) then transposed; x += s*rx, y += s*ry; t >>= 2.
    The cell's raster id is (g - 1 - y) * g + x.  Vectorised over d.
    """
    g = int(grid_size)
    if g < 2 or g & (g - 1):
        raise ValueError("Hilbert grid side must be a power of two >= 2")
    t = np.arange(g * g, dtype=np.int64)
    x = np.zeros_like(t)
    y = np.zeros_like(t)
    s = 1
    while s < g:
        rx = (t >> 1) & 1
        ry = (t ^ rx) & 1
        flip = (ry == 0) & (rx == 1)
        x = np.where(flip, s - 1 - x, x)
        y = np.where(flip, s - 1 - y, y)
        swap = ry == 0
        x, y = np.where(swap, y, x), np.where(swap, x, y)
        x = x + s * rx
        y = y + s * ry
        t = t >> 2
        s *= 2
    return (g - 1 - y) * g + x


def neighbor_pairs(grid_size: int, connectivity: int = 4) -> np.ndarray:
    """Ascending undirected raster neighbour pairs (``geometry.py:28-43``).

    Order: for y, for x, for (dy, dx) in [(0,1), (1,0)] (+ diagonals for 8).
    """
    if int(grid_size) != grid_size or grid_size < 1 or connectivity not in (4, 8):
        raise ValueError("positive integer grid_size and connectivity 4 or 8 required")
    g = int(grid_size)
    dirs = [(0, 1), (1, 0)] + ([(1, 1), (1, -1)] if connectivity == 8 else [])
    yy, xx = np.meshgrid(np.arange(g), np.arange(g), indexing="ij")
    cols = []
    for dy, dx in dirs:
        ny, nx = yy + dy, xx + dx
        ok = (ny >= 0) & (ny < g) & (nx >= 0) & (nx < g)
        a = np.where(ok, yy * g + xx, -1)
        b = np.where(ok, ny * g + nx, -1)
        cols.append(np.stack([a, b], -1))
    # interleave directions in (y, x, dir) order, then drop invalid
    allp = np.stack(cols, 2).reshape(-1, 2)
    return allp[allp[:, 0] >= 0].astype(np.int64)


# --------------------------------------------------------------------------
# plan.py
# --------------------------------------------------------------------------
@dataclass
class PhasePlanNP:
    offset: int
    kv_indices: np.ndarray  # int32 [rows, W], zero padded
    kv_counts: np.ndarray  # int32 [rows]
    bridge_original_blocks: np.ndarray  # int64 [nb] (build_plan) or [nb, K] (bridge_k)


@dataclass
class AttentionPlanNP:
    grid_size: int
    tile_count: int
    text_tokens: int
    shared_tokens: int
    block_size: int
    image_order: np.ndarray
    inverse_image_order: np.ndarray
    original_order: np.ndarray
    physical_original_blocks: np.ndarray
    phases: list = field(default_factory=list)
    bridge: bool = False

    @property
    def image_tokens(self):
        return self.grid_size**2

    @property
    def global_tokens(self):
        return self.text_tokens + self.shared_tokens

    @property
    def total_tokens(self):
        return self.text_tokens + self.image_tokens

    def dense_mask(self, phase: int) -> np.ndarray:
        """Token-level bool mask, ``plan.py:70-84``."""
        p = self.phases[phase % 4]
        total = self.total_tokens // self.block_size
        glob = self.global_tokens // self.block_size
        blocks = np.zeros((total, total), dtype=bool)
        blocks[:glob] = True
        for q in range(len(p.kv_counts)):
            blocks[glob + q, p.kv_indices[q, : p.kv_counts[q]]] = True
        b = self.block_size
        return np.repeat(np.repeat(blocks, b, 0), b, 1)


def _composite(grid_size: int):
    """``plan.py:133-135``: middle half of the Hilbert walk + its point reflection."""
    n = grid_size**2
    h = hilbert_order(grid_size)
    mid = h[n // 4 : 3 * n // 4]
    original = np.concatenate([mid, n - 1 - mid])
    inverse = np.argsort(original, kind="stable")
    return original, inverse


def _pad_rows(rows):
    counts = np.array([len(r) for r in rows], dtype=np.int32)
    ids = np.zeros((len(rows), int(counts.max())), dtype=np.int32)
    for q, r in enumerate(rows):
        ids[q, : len(r)] = r
    return ids, counts


def _cut_scores(inverse, labels, pairs, block_size, nb):
    """Counter of cut 4-neighbour pixel pairs between original-order blocks, both
    directions (``plan.py:160-166``, ``bridge_k.py:22-28``) as a dense [nb, nb]."""
    cut = pairs[labels[pairs[:, 0]] != labels[pairs[:, 1]]]
    ob = inverse[cut] // block_size
    key = np.concatenate([ob[:, 0] * nb + ob[:, 1], ob[:, 1] * nb + ob[:, 0]])
    return np.bincount(key, minlength=nb * nb).reshape(nb, nb)


def _rank_keys(scores_row, off_blocks, nb, k):
    """Top-k keys by (-score, (key - offset/b) mod nb) (``bridge_k.py:36-43``,
    ``plan.py:167-172`` for k = 1)."""
    keys = np.nonzero(scores_row)[0]
    if len(keys) == 0:
        return keys
    tie = (keys - off_blocks) % nb
    order = np.lexsort((tie, -scores_row[keys]))
    return keys[order[:k]]


def build_plan(tile_count=4, grid_size=64, text_tokens=512, shared=True, bridge=True, block_size=64):
    """Restates ``hilberta/plan.py:114-197`` (``build_plan``)."""
    for name, value in [
        ("tile_count", tile_count),
        ("grid_size", grid_size),
        ("text_tokens", text_tokens),
        ("block_size", block_size),
    ]:
        if isinstance(value, bool) or int(value) != value or value <= 0:
            raise ValueError(f"{name} must be a positive integer")
    tile_count, grid_size, text_tokens, block_size = map(
        int, (tile_count, grid_size, text_tokens, block_size)
    )
    n = grid_size**2
    if grid_size < 8 or grid_size & (grid_size - 1):
        raise ValueError("grid_size must be a power of two >= 8")
    if n % tile_count or (n // tile_count) % (4 * block_size) or text_tokens % block_size:
        raise ValueError("Tile quarter offsets and text prefix must be block aligned")
    original, inverse = _composite(grid_size)
    blocks = original.reshape(-1, block_size)
    nb = blocks.shape[0]
    shared_ids = np.zeros(n, dtype=bool)
    if shared:
        s0, s1 = 3 * grid_size // 8, 5 * grid_size // 8
        shared_ids.reshape(grid_size, grid_size)[s0:s1, s0:s1] = True
    share_counts = shared_ids[blocks].sum(1)
    if ((share_counts != 0) & (share_counts != block_size)).any():
        raise ValueError("Shared square must be a union of complete original blocks")
    share_blocks = np.nonzero(share_counts == block_size)[0]
    ordinary = np.nonzero(share_counts == 0)[0]
    packed = np.concatenate([share_blocks, ordinary]).astype(np.int64)
    order = blocks[packed].reshape(-1)
    original_to_physical = np.argsort(packed, kind="stable") + text_tokens // block_size
    global_blocks = text_tokens // block_size + len(share_blocks)
    pairs = neighbor_pairs(grid_size, 4)
    width = n // tile_count
    phases = []
    for offset in (0, width // 4, width // 2, 3 * width // 4):
        labels = ((inverse - offset) % n) // width
        block_labels = labels[blocks[:, 0]]
        if not np.array_equal(labels[blocks], np.broadcast_to(block_labels[:, None], blocks.shape)):
            raise AssertionError("A physical block crosses a tile boundary")
        chosen = np.full(nb, -1, dtype=np.int64)
        if bridge:
            scores = _cut_scores(inverse, labels, pairs, block_size, nb)
            for q in range(nb):
                top = _rank_keys(scores[q], offset // block_size, nb, 1)
                if len(top):
                    chosen[q] = top[0]
        rows = []
        glob_keys = np.arange(global_blocks)
        for q in ordinary:
            same = ordinary[block_labels[ordinary] == block_labels[q]]
            keys = np.union1d(glob_keys, original_to_physical[same])
            if chosen[q] >= 0:
                keys = np.union1d(keys, [original_to_physical[chosen[q]]])
            rows.append(keys)
        ids, counts = _pad_rows(rows)
        phases.append(PhasePlanNP(offset, ids, counts, chosen))
    return AttentionPlanNP(
        grid_size,
        tile_count,
        text_tokens,
        len(share_blocks) * block_size,
        block_size,
        order.astype(np.int64),
        np.argsort(order, kind="stable").astype(np.int64),
        original.astype(np.int64),
        packed,
        phases,
        bool(bridge),
    )


# --------------------------------------------------------------------------
# bridge_k.py
# --------------------------------------------------------------------------
def bridge_k_plan(tiles=4, k=1, shared=False, *, grid_size=64):
    """Restates ``hilberta/bridge_k.py:10-51``: top-K bridges + reciprocal closure."""
    if isinstance(k, bool) or k not in (1, 2, 3, 4):
        raise ValueError("This bounded comparison supports integer K=1..4")
    plan = build_plan(tiles, grid_size=grid_size, shared=shared, bridge=False)
    n = plan.image_tokens
    b = plan.block_size
    nb = n // b
    g = plan.global_tokens // b
    inverse = np.argsort(plan.original_order, kind="stable")
    physical = np.argsort(plan.physical_original_blocks, kind="stable") + plan.text_tokens // b
    pairs = neighbor_pairs(plan.grid_size, 4)
    total = plan.total_tokens // b
    phases = []
    for p in plan.phases:
        labels = ((inverse - p.offset) % n) // (n // tiles)
        scores = _cut_scores(inverse, labels, pairs, b, nb)
        chosen = np.full((nb, k), -1, dtype=np.int64)
        adj = np.zeros((total, total), dtype=bool)
        adj[:g, :] = True
        for row in range(len(p.kv_counts)):
            adj[g + row, p.kv_indices[row, : p.kv_counts[row]]] = True
        for q in range(nb):
            top = _rank_keys(scores[q], p.offset // b, nb, k)
            chosen[q, : len(top)] = top
            adj[physical[q], physical[top]] = True
        adj = adj | adj.T
        rows = [np.nonzero(adj[q])[0] for q in range(g, total)]
        ids, counts = _pad_rows(rows)
        phases.append(PhasePlanNP(p.offset, ids, counts, chosen))
    plan.phases = phases
    plan.bridge = True
    return plan


# --------------------------------------------------------------------------
# sparse_kernel.py (validator) + paired_metadata.py
# --------------------------------------------------------------------------
def validate_metadata(kv_indices, kv_counts, *, tokens, global_tokens=768, block_size=64):
    """Restates the checks of ``hilberta/sparse_kernel.py:100-152`` (numpy arrays)."""
    if block_size != 64:
        raise ValueError("This kernel currently requires 64-token physical blocks")
    if not (0 <= global_tokens < tokens) or tokens % block_size or global_tokens % block_size:
        raise ValueError("tokens/global prefix must be block-aligned with at least one ordinary block")
    rows = (tokens - global_tokens) // block_size
    if kv_indices.ndim != 2 or kv_indices.shape[0] != rows or kv_indices.shape[1] < 1:
        raise ValueError("kv_indices must be [ordinary_query_blocks, max_KV_blocks]")
    nblocks, gblocks = tokens // block_size, global_tokens // block_size
    for row, count in enumerate(kv_counts.tolist()):
        if not 1 <= count <= kv_indices.shape[1]:
            raise ValueError(f"Invalid K/V count in ordinary query block {row}")
        ids = kv_indices[row, :count]
        if ids.min() < 0 or ids.max() >= nblocks or len(set(ids.tolist())) != count:
            raise ValueError(f"Out-of-range or duplicate K/V blocks in row {row}")
        if not set(range(gblocks)).issubset(ids.tolist()):
            raise ValueError(f"Row {row} misses global-prefix keys")


def pair_metadata(kv_indices, kv_counts, *, tokens, global_tokens=768, key_block_size=64):
    """Restates ``hilberta/paired_metadata.py:26-51``.

    Returns (ids int32 [rows/2, W], flags int32 [rows/2, W], counts int32 [rows/2]).
    Flag bit (half + 2*key_half) marks that query half ``half`` sees key half
    ``key_half`` of the listed ``key_block_size`` key block.
    """
    kv_indices = np.asarray(kv_indices)
    kv_counts = np.asarray(kv_counts)
    validate_metadata(kv_indices, kv_counts, tokens=tokens, global_tokens=global_tokens)
    if key_block_size not in (64, 128) or tokens % 128 or global_tokens % 128:
        raise ValueError("Paired queries require N/global aligned to 128; KV must be 64/128")
    ratio = key_block_size // 64
    rows = []
    for q in range(0, len(kv_counts), 2):
        union = {}
        for half in range(2):
            for block in kv_indices[q + half, : int(kv_counts[q + half])].tolist():
                bid, kh = divmod(block, ratio)
                union[bid] = union.get(bid, 0) | (1 << (half + 2 * kh))
        rows.append(sorted(union.items()))
    counts = np.array([len(r) for r in rows], dtype=np.int32)
    ids = np.zeros((len(rows), int(counts.max())), dtype=np.int32)
    flags = np.zeros_like(ids)
    for q, r in enumerate(rows):
        for j, (bid, f) in enumerate(r):
            ids[q, j], flags[q, j] = bid, f
    return ids, flags, counts


def unpair_metadata(ids, flags, counts, key_block_size=64):
    """Restates ``hilberta/paired_metadata.py:54-70``."""
    ratio = key_block_size // 64
    rows = []
    for row, count in enumerate(np.asarray(counts).tolist()):
        for half in range(2):
            out = []
            for bid, f in zip(ids[row, :count].tolist(), flags[row, :count].tolist()):
                for kh in range(ratio):
                    if f & (1 << (half + 2 * kh)):
                        out.append(bid * ratio + kh)
            rows.append(sorted(out))
    return rows


def active_blocks(kv_counts, tokens, global_tokens, block_size=64):
    """Active 64x64 (query-block, key-block) pairs of one phase: global rows see
    every block, ordinary rows their listed blocks (FLOP numerator)."""
    return (global_tokens // block_size) * (tokens // block_size) + int(np.asarray(kv_counts).sum())
