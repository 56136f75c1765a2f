"""PlanBank host checks (the reference adapter's _PlanBank,
hilberta/flux_adapter.py:26-146): the checks that run before any device work,
with the reference's messages, on a plan built by the oracle."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from hilberta_b200.plan_bank import PlanBank
from oracle import plan_oracle as po


def _plan(grid=32):
    ref = po.bridge_k_plan(4, 1, False, grid_size=grid)
    get = (lambda k: ref[k]) if isinstance(ref, dict) else (lambda k: getattr(ref, k))
    order = torch.as_tensor(np.asarray(get("image_order")), dtype=torch.int64)
    phases = [SimpleNamespace(kv_indices=torch.as_tensor(np.asarray(p["kv_indices"] if isinstance(p, dict) else p.kv_indices), dtype=torch.int32),
                              kv_counts=torch.as_tensor(np.asarray(p["kv_counts"] if isinstance(p, dict) else p.kv_counts), dtype=torch.int32))
              for p in get("phases")]
    n = grid * grid
    return SimpleNamespace(image_tokens=n, text_tokens=512, shared_tokens=0, global_tokens=512, total_tokens=512 + n,
                           block_size=64, image_order=order, inverse_image_order=torch.argsort(order), phases=phases)


@pytest.mark.parametrize("field,value,message", [
    ("text_tokens", 0, "nonempty image/text tokens"),
    ("shared_tokens", -1, "valid shared-image count"),
    ("global_tokens", 576, "global/total token counts are inconsistent"),
    ("total_tokens", 999, "global/total token counts are inconsistent"),
    ("block_size", 48, "block-aligned"),
])
def test_token_count_checks(field, value, message):
    plan = _plan()
    setattr(plan, field, value)
    with pytest.raises(ValueError, match=message):
        PlanBank(plan)


def test_permutation_checks():
    plan = _plan()
    plan.image_order = plan.image_order.clone()
    plan.image_order[3] = plan.image_order[4]
    with pytest.raises(ValueError, match="every image-token identity exactly once"):
        PlanBank(plan)
    plan = _plan()
    plan.inverse_image_order = plan.inverse_image_order.roll(1)
    with pytest.raises(ValueError, match="not the inverse of image_order"):
        PlanBank(plan)


def test_phase_table_checks():
    plan = _plan()
    plan.phases = plan.phases[:3]
    with pytest.raises(ValueError, match="Exactly four phase"):
        PlanBank(plan)
    plan = _plan()
    plan.phases[1].kv_counts = plan.phases[1].kv_counts[:-1]
    with pytest.raises(ValueError, match="one row per ordinary physical query block"):
        PlanBank(plan)
    plan = _plan()
    plan.phases[2].kv_counts = plan.phases[2].kv_counts.clone()
    plan.phases[2].kv_counts[5] = plan.phases[2].kv_indices.shape[1] + 1
    with pytest.raises(ValueError, match="counts are outside their metadata width"):
        PlanBank(plan)


def test_valid_plan_needs_the_device_for_row_checks():
    if torch.cuda.is_available():
        pytest.skip("covered by the GPU tests")
    with pytest.raises(RuntimeError, match="requires a CUDA device"):
        PlanBank(_plan())
