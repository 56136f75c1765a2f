"""On-disk plans (hilberta_b200/plan_cache.py): round trip of a bridge-K plan
built by the CPU oracle, refusal of edited or foreign files, and the directory
cache building once and loading afterwards.  No GPU."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from hilberta_b200.plan import AttentionPlan, PhasePlan
from hilberta_b200.plan_cache import PlanCache, load_plan, save_plan
from oracle import plan_oracle as po


def _plan(tiles=4, k=1, shared=False, grid_size=32):
    p = po.bridge_k_plan(tiles, k, shared, grid_size=grid_size)
    t = lambda a, dt=torch.int64: torch.from_numpy(np.asarray(a)).to(dt)
    return AttentionPlan(
        grid_size=p.grid_size, tile_count=p.tile_count, text_tokens=p.text_tokens, shared_tokens=p.shared_tokens,
        block_size=p.block_size, image_order=t(p.image_order), inverse_image_order=t(p.inverse_image_order),
        original_order=t(p.original_order), physical_original_blocks=t(p.physical_original_blocks),
        phases=tuple(PhasePlan(int(ph.offset), t(ph.kv_indices, torch.int32), t(ph.kv_counts, torch.int32),
                               t(ph.bridge_original_blocks)) for ph in p.phases),
        bridge=bool(p.bridge))


def _equal(a, b):
    assert a.manifest() == b.manifest()
    for f in ("image_order", "inverse_image_order", "original_order", "physical_original_blocks"):
        assert torch.equal(getattr(a, f), getattr(b, f)), f
    for pa, pb in zip(a.phases, b.phases):
        assert pa.offset == pb.offset
        assert torch.equal(pa.kv_indices, pb.kv_indices) and pa.kv_indices.dtype == torch.int32
        assert torch.equal(pa.kv_counts, pb.kv_counts)
        assert torch.equal(pa.bridge_original_blocks, pb.bridge_original_blocks)


@pytest.mark.parametrize("tiles,k,grid", [(4, 1, 32), (16, 3, 64)])
def test_round_trip(tmp_path, tiles, k, grid):
    plan = _plan(tiles, k, grid_size=grid)
    path = save_plan(plan, tmp_path / "p.npz")
    _equal(plan, load_plan(path))
    assert not list(tmp_path.glob("*.tmp*"))  # written atomically


def _rewrite(path, **changes):
    with np.load(path, allow_pickle=False) as z:
        arrays = {k: np.array(z[k]) for k in z.files}
    arrays.update(changes)
    for k in [k for k, v in changes.items() if v is None]:
        del arrays[k]
    with open(path, "wb") as f:
        np.savez(f, **arrays)


def test_edited_files_are_refused(tmp_path):
    plan = _plan()
    path = save_plan(plan, tmp_path / "p.npz")
    ids = plan.phases[2].kv_indices.numpy().copy()
    ids[3, 0] = ids[3, 1]  # one KV entry changed
    _rewrite(path, phase2_kv_indices=ids)
    with pytest.raises(ValueError, match="checksum"):
        load_plan(path)

    path = save_plan(plan, tmp_path / "q.npz")
    order = plan.image_order.numpy().copy()
    order[[0, 1]] = order[[1, 0]]  # a different order with the stored inverse
    _rewrite(path, image_order=order)
    with pytest.raises(ValueError, match="checksum"):
        load_plan(path)

    path = save_plan(plan, tmp_path / "r.npz")
    _rewrite(path, phase1_kv_counts=None)
    with pytest.raises(ValueError, match="checksum"):
        load_plan(path)

    path = save_plan(plan, tmp_path / "s.npz")
    with np.load(path, allow_pickle=False) as z:
        header = json.loads(str(z["header"]))
    header["format"] = "something/9"
    _rewrite(path, header=np.array(json.dumps(header)))
    with pytest.raises(ValueError, match="format"):
        load_plan(path)


def test_directory_cache_builds_once(tmp_path):
    calls = []

    def build(tiles, k, shared, grid_size):
        calls.append((tiles, k, shared, grid_size))
        return _plan(tiles, k, shared, grid_size)

    cache = PlanCache(tmp_path / "plans")
    a = cache.get(4, 1, False, 32, build=build)
    b = cache.get(4, 1, False, 32, build=build)
    assert calls == [(4, 1, False, 32)]
    _equal(a, b)
    assert cache.path(4, 1, False, 32).name == "bridge_t4_k1_noshared_g32.npz"
    cache.get(4, 2, False, 32, build=build)
    assert len(calls) == 2


def test_consistent_checksum_but_wrong_plan_is_refused(tmp_path):
    """A file whose checksum was recomputed over wrong arrays (a faulty writer)
    still fails the structural checks."""
    from hilberta_b200.plan_cache import _digest

    def rewrite_with_digest(path, **changes):
        with np.load(path, allow_pickle=False) as z:
            arrays = {k: np.array(z[k]) for k in z.files}
        header = json.loads(str(arrays.pop("header")))
        arrays.update(changes)
        header["arrays_sha256"] = _digest(arrays)
        arrays["header"] = np.array(json.dumps(header))
        with open(path, "wb") as f:
            np.savez(f, **arrays)

    plan = _plan()
    path = save_plan(plan, tmp_path / "a.npz")
    order = plan.image_order.numpy().copy()
    order[[0, 1]] = order[[1, 0]]
    rewrite_with_digest(path, image_order=order)
    with pytest.raises(ValueError, match="inverse"):
        load_plan(path)

    path = save_plan(plan, tmp_path / "b.npz")
    counts = plan.phases[0].kv_counts.numpy().copy()
    counts[0] -= 1  # a row shortened: the manifest's entry count changes
    rewrite_with_digest(path, phase0_kv_counts=counts)
    with pytest.raises(ValueError, match="manifest"):
        load_plan(path)
