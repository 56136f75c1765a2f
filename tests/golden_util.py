"""Helpers shared by the oracle and builder parity tests: load the golden
vectors written by ``tests/golden/make_golden.py`` and compare plans against them."""

from __future__ import annotations

import hashlib
import json
from functools import lru_cache
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


@lru_cache(None)
def records():
    return json.loads((GOLDEN / "plans.json").read_text())


@lru_cache(None)
def arrays():
    with np.load(GOLDEN / "plans_small.npz") as z:
        return {k: z[k] for k in z.files}


def digest(arr, dtype):
    a = np.ascontiguousarray(np.asarray(arr).astype(dtype))
    return hashlib.sha256(a.tobytes()).hexdigest()


def check_plan(name, plan, pair_fn=None):
    """Compare a plan-like object (numpy or torch fields) with the golden record.

    ``pair_fn(phase_index, phase, key_block_size) -> (ids, flags, counts)`` builds
    paired metadata for the phases when the record holds paired digests.
    Returns a list of mismatch descriptions (empty == bit-exact).
    """
    rec = records()[name]
    arr = arrays()
    bad = []

    def np_(x):
        return x.cpu().numpy() if hasattr(x, "cpu") else np.asarray(x)

    for f in ("grid_size", "tile_count", "text_tokens", "shared_tokens", "block_size"):
        if int(getattr(plan, f)) != rec[f]:
            bad.append(f"{f}: {getattr(plan, f)} != {rec[f]}")
    for f in ("image_order", "inverse_image_order", "original_order", "physical_original_blocks"):
        a = np_(getattr(plan, f))
        if digest(a, np.int64) != rec[f]:
            bad.append(f"{f} digest")
            key = f"{name}.{f}"
            if key in arr and a.shape == arr[key].shape:
                bad.append(f"  first diff at {int(np.argmax(a != arr[key]))}")
    for i, (p, ph) in enumerate(zip(plan.phases, rec["phases"])):
        if int(p.offset) != ph["offset"]:
            bad.append(f"p{i} offset")
        ids, cnt = np_(p.kv_indices), np_(p.kv_counts)
        if list(ids.shape) != ph["kv_shape"]:
            bad.append(f"p{i} kv shape {ids.shape} != {ph['kv_shape']}")
        if digest(ids, np.int32) != ph["kv_indices"]:
            bad.append(f"p{i} kv_indices digest")
        if digest(cnt, np.int32) != ph["kv_counts"]:
            bad.append(f"p{i} kv_counts digest")
        bob = np_(p.bridge_original_blocks)
        if list(bob.shape) != ph["bridge_shape"] or digest(bob, np.int64) != ph["bridge_original_blocks"]:
            bad.append(f"p{i} bridge_original_blocks")
        if pair_fn is not None:
            for kvb, pr in ph["paired"].items():
                pids, pflags, pcnt = (np_(x) for x in pair_fn(i, p, int(kvb)))
                if list(pids.shape) != pr["shape"]:
                    bad.append(f"p{i} kv{kvb} paired shape {pids.shape} != {pr['shape']}")
                for nm, x in (("kv_indices", pids), ("kv_flags", pflags), ("kv_counts", pcnt)):
                    if digest(x, np.int32) != pr[nm]:
                        bad.append(f"p{i} kv{kvb} paired {nm} digest")
    return bad
