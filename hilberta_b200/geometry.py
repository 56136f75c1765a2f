"""Hilbert ordering and grid neighbours (API of ``hilberta/geometry.py``).

``hilbert_order`` runs on the device (``hb_hilbert_order``); ``neighbor_pairs``
is host-side index bookkeeping with the reference's ordering.
"""

from __future__ import annotations

import torch

from . import _lib


def hilbert_order(grid_size=64, *, device=None):
    """Raster id of the Hilbert walk's d-th cell, vertically flipped, int64 [g^2] on CPU.

    Same values as ``hilberta/geometry.py:6-25``; computed by the CUDA builder.
    """
    if isinstance(grid_size, bool) or int(grid_size) != grid_size or grid_size < 2 or int(grid_size) & (int(grid_size) - 1):
        raise ValueError("Hilbert grid side must be a power of two >= 2")
    g = int(grid_size)
    dev = _lib.require_cuda(device)
    out = torch.empty(g * g, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().hb_hilbert_order(g, _lib.ptr(out), _lib.stream_ptr(dev)), "hb_hilbert_order")
    return out.cpu()


def neighbor_pairs(grid_size, connectivity=4):
    """Unique undirected non-periodic 2-D neighbours, ascending pairs, int64 [P, 2]
    in the order of ``hilberta/geometry.py:28-43`` (y, x, direction)."""
    if int(grid_size) != grid_size or grid_size < 1 or connectivity not in (4, 8):
        raise ValueError("positive integer grid_size and connectivity 4 or 8 required")
    g = int(grid_size)
    dirs = [(0, 1), (1, 0)] + ([(1, 1), (1, -1)] if connectivity == 8 else [])
    yy, xx = torch.meshgrid(torch.arange(g), torch.arange(g), indexing="ij")
    cols = []
    for dy, dx in dirs:
        ny, nx = yy + dy, xx + dx
        ok = (ny >= 0) & (ny < g) & (nx >= 0) & (nx < g)
        a = torch.where(ok, yy * g + xx, torch.full_like(yy, -1))
        b = torch.where(ok, ny * g + nx, torch.full_like(yy, -1))
        cols.append(torch.stack([a, b], -1))
    pairs = torch.stack(cols, 2).reshape(-1, 2)
    return pairs[pairs[:, 0] >= 0].to(torch.long).reshape(-1, 2)
