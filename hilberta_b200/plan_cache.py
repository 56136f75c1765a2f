"""On-disk plans: ``save_plan`` / ``load_plan`` and a directory cache.

A plan is a handful of integer arrays (image order and its inverse, the
composite order, the physical block map, and per phase the sorted KV rows,
their counts and the chosen bridge blocks).  They are stored in one numpy
``.npz`` archive (no pickled objects) together with the plan's ``manifest()``
(``hilberta/plan.py:86-111``) as JSON.  A SHA-256 over every
array's dtype, shape and bytes is stored beside them.  ``load_plan`` checks
that digest, rebuilds the ``AttentionPlan``, recomputes its manifest and
compares it with the stored one, and checks that the inverse order inverts the
order, so a truncated or edited file is refused instead of producing a wrong
mask.

``PlanCache(directory).get(tiles, k, shared, grid_size)`` returns the cached
bridge-K plan or builds it (``bridge_k_plan``, on the GPU) and stores it
atomically (write to a temporary name, then rename).
"""

from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

import numpy as np
import torch

from .plan import AttentionPlan, PhasePlan

FORMAT = "hilberta_b200.plan/1"
_SCALARS = ("grid_size", "tile_count", "text_tokens", "shared_tokens", "block_size")


def _np(t):
    return t.detach().cpu().numpy()


def _digest(arrays):
    h = hashlib.sha256()
    for name in sorted(arrays):
        a = np.ascontiguousarray(arrays[name])
        h.update(f"{name}:{a.dtype.str}:{a.shape};".encode())
        h.update(a.tobytes())
    return h.hexdigest()


def save_plan(plan, path):
    """Write ``plan`` to ``path`` (``.npz``); returns the path written."""
    path = Path(path)
    arrays = {
        "image_order": _np(plan.image_order).astype(np.int64),
        "inverse_image_order": _np(plan.inverse_image_order).astype(np.int64),
        "original_order": _np(plan.original_order).astype(np.int64),
        "physical_original_blocks": _np(plan.physical_original_blocks).astype(np.int64),
    }
    for i, p in enumerate(plan.phases):
        arrays[f"phase{i}_kv_indices"] = _np(p.kv_indices).astype(np.int32)
        arrays[f"phase{i}_kv_counts"] = _np(p.kv_counts).astype(np.int32)
        arrays[f"phase{i}_bridge_original_blocks"] = _np(p.bridge_original_blocks).astype(np.int64)
    header = {
        "format": FORMAT,
        "phases": len(plan.phases),
        "offsets": [int(p.offset) for p in plan.phases],
        "bridge": bool(plan.bridge),
        "full": bool(plan.full),
        **{k: int(getattr(plan, k)) for k in _SCALARS},
        "manifest": plan.manifest(),
        "arrays_sha256": _digest(arrays),
    }
    arrays["header"] = np.array(json.dumps(header, sort_keys=True))
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + f".tmp{os.getpid()}")
    with open(tmp, "wb") as f:
        np.savez(f, **arrays)
    os.replace(tmp, path)
    return path


def load_plan(path):
    """Read a plan written by ``save_plan``; raises ``ValueError`` when the file
    is not one or does not match its own manifest."""
    with np.load(Path(path), allow_pickle=False) as z:
        try:
            header = json.loads(str(z["header"]))
        except (KeyError, ValueError) as e:
            raise ValueError(f"{path}: not a saved plan ({e})") from None
        if header.get("format") != FORMAT:
            raise ValueError(f"{path}: unknown plan format {header.get('format')!r}")
        arrays = {k: np.array(z[k]) for k in z.files if k != "header"}
        if _digest(arrays) != header.get("arrays_sha256"):
            raise ValueError(f"{path}: array checksum does not match (file edited or truncated)")
        try:
            t = {k: torch.from_numpy(np.array(z[k])) for k in
                 ("image_order", "inverse_image_order", "original_order", "physical_original_blocks")}
            phases = tuple(
                PhasePlan(
                    offset=int(off),
                    kv_indices=torch.from_numpy(np.array(z[f"phase{i}_kv_indices"])),
                    kv_counts=torch.from_numpy(np.array(z[f"phase{i}_kv_counts"])),
                    bridge_original_blocks=torch.from_numpy(np.array(z[f"phase{i}_bridge_original_blocks"])),
                )
                for i, off in enumerate(header["offsets"])
            )
        except KeyError as e:
            raise ValueError(f"{path}: missing array {e}") from None
    plan = AttentionPlan(
        **{k: int(header[k]) for k in _SCALARS},
        **t,
        phases=phases,
        bridge=bool(header["bridge"]),
        full=bool(header["full"]),
    )
    n = plan.image_tokens
    order, inv = plan.image_order, plan.inverse_image_order
    if order.shape != (n,) or inv.shape != (n,) or not torch.equal(inv[order], torch.arange(n)):
        raise ValueError(f"{path}: inverse_image_order is not the inverse of image_order")
    if json.loads(json.dumps(plan.manifest(), sort_keys=True)) != header["manifest"]:
        raise ValueError(f"{path}: plan arrays do not match the stored manifest")
    return plan


class PlanCache:
    """Directory of saved bridge-K plans keyed by (tiles, k, shared, grid_size)."""

    def __init__(self, directory):
        self.directory = Path(directory)

    def path(self, tiles, k, shared, grid_size):
        return self.directory / f"bridge_t{int(tiles)}_k{int(k)}_{'shared' if shared else 'noshared'}_g{int(grid_size)}.npz"

    def get(self, tiles, k, shared=False, grid_size=64, *, build=None):
        """The cached plan, or ``build(tiles, k, shared, grid_size=...)``
        (default ``bridge_k_plan``) saved for next time."""
        p = self.path(tiles, k, shared, grid_size)
        if p.exists():
            return load_plan(p)
        if build is None:
            from .bridge_k import bridge_k_plan as build
        plan = build(tiles, k, shared, grid_size=grid_size)
        save_plan(plan, p)
        return plan


__all__ = ["save_plan", "load_plan", "PlanCache", "FORMAT"]
