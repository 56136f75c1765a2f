"""PlanBank on the device: per-row checks with the reference adapter's
messages, device caches, paired metadata and dense masks equal to the direct
builders (hilberta/flux_adapter.py:26-146)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bank_caches_and_matches_builders():
    import hilberta_b200 as hb
    from hilberta_b200.plan_bank import PlanBank

    plan = hb.bridge_k_plan(16, 3, False, grid_size=64)
    info = {"backend": "paired"}
    bank = PlanBank(plan, info)
    dev = bank.on_device("cuda:0")
    assert bank.on_device("cuda:0") is dev and info["metadata_device_copies"] == 1
    assert torch.equal(dev["order"].cpu(), torch.as_tensor(plan.image_order))
    for ph, p in enumerate(plan.phases):
        want = hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=plan.total_tokens, global_tokens=plan.global_tokens)
        got = dev["paired_phases"][ph]
        assert got.kv_indices.is_cuda
        assert torch.equal(got.kv_indices.cpu(), want.kv_indices.cpu())
        assert torch.equal(got.kv_flags.cpu(), want.kv_flags.cpu())
        assert torch.equal(got.kv_counts.cpu(), want.kv_counts.cpu())
    assert dev["raster"].grid == 64 and dev["raster"].block_origin.is_cuda
    mask = bank.dense_mask(2, "cuda:0")
    assert torch.equal(mask.cpu(), torch.as_tensor(plan.dense_mask(2)).cpu())
    assert info["reference_masks_prepared"] == 1
    bank.clear()
    assert bank.device_cache == {} and bank.mask_cache == {}


@pytest.mark.parametrize("fault,message", [
    ("duplicate", "Active KV block IDs must be valid and unique"),
    ("range", "Active KV block IDs must be valid and unique"),
    ("prefix", "retain every text/shared global key block"),
])
def test_row_checks(fault, message):
    import hilberta_b200 as hb
    from hilberta_b200.plan_bank import PlanBank

    import dataclasses

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    ids = plan.phases[1].kv_indices.clone()
    count = int(plan.phases[1].kv_counts[4])
    nkb = plan.total_tokens // 64
    if fault == "duplicate":
        ids[4, count - 1] = ids[4, count - 2]
    elif fault == "range":
        ids[4, count - 1] = nkb
    else:  # replace global block 0 by an ordinary block the row does not list
        free = next(b for b in range(nkb - 1, 0, -1) if b not in set(ids[4, :count].tolist()))
        ids[4, 0] = free
    phases = list(plan.phases)
    phases[1] = dataclasses.replace(phases[1], kv_indices=ids)
    bad = dataclasses.replace(plan, phases=type(plan.phases)(phases))
    with pytest.raises(ValueError, match=message):
        PlanBank(bad)


def test_plan_cache_round_trip_feeds_the_kernel(tmp_path):
    """A plan built on the GPU, cached on disk and loaded back gives the same
    manifest, rows and attention output (bit for bit) as the fresh plan."""
    import hilberta_b200 as hb
    from hilberta_b200.plan_cache import PlanCache

    cache = PlanCache(tmp_path)
    fresh = cache.get(4, 1, False, 32)
    loaded = cache.get(4, 1, False, 32)
    assert fresh.manifest() == loaded.manifest()
    for a, b in zip(fresh.phases, loaded.phases):
        assert torch.equal(a.kv_indices, b.kv_indices) and torch.equal(a.kv_counts, b.kv_counts)
    g = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(1, 2, fresh.total_tokens, 128, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    outs = []
    for plan in (fresh, loaded):
        meta = hb.PlanBank(plan).on_device(torch.device("cuda"))["paired_phases"][1]
        outs.append(hb.paired_attention(q, k, v, meta))
    assert torch.equal(outs[0], outs[1])
