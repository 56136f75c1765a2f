"""A FLUX.1-architecture step (hilberta_b200/flux_model.py, small widths) with
HilbertA attention in every joint-attention call:

* against the same weights with dense attention under the plan's phase masks
  (the reference adapter's correctness path, hilberta/flux_adapter.py:299-307);
* with a full-attention plan (hilberta/plan.py:200-212) against plain dense
  attention in raster order: every op but attention is per-token, so the entry
  permutation, the permuted rotary positions and the exit permutation must cancel.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(model, grid, text_tokens, seed=3):
    g = torch.Generator(device="cpu").manual_seed(seed)
    latents = torch.randn(2, grid * grid, 64, generator=g).to(torch.bfloat16).cuda()
    text = torch.randn(2, text_tokens, 64, generator=g).to(torch.bfloat16).cuda()
    pooled = torch.randn(2, 32, generator=g).to(torch.bfloat16).cuda()
    return latents, text, pooled, torch.tensor([0.3, 0.9], device="cuda"), torch.tensor([3.5, 3.5], device="cuda")


def _model(bank, grid, attention):
    from hilberta_b200.flux_model import FluxLikeTransformer

    torch.manual_seed(0)
    return FluxLikeTransformer(grid, bank, attention=attention, num_double=2, num_single=3, dim=256, heads=2,
                               text_dim=64, pooled_dim=32, device="cuda")


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


def test_step_matches_masked_dense():
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    bank = hb.PlanBank(plan)
    model = _model(bank, 32, "hilberta")
    x = _inputs(model, 32, plan.text_tokens)
    with torch.inference_mode():
        sparse = model(*x)
        model.set_attention("masked")
        masked = model(*x)
        model.set_attention("dense")
        dense = model(*x)
    assert sparse.shape == (2, 32 * 32, 64)
    assert torch.isfinite(sparse).all()
    # 5 layers of bf16 activations: relative L2 within 2 %, far below the
    # sparse-vs-dense distance
    assert _rel(sparse, masked) < 2e-2
    assert _rel(dense, masked) > 5 * _rel(sparse, masked)


def test_full_plan_step_is_permutation_equivalent_to_dense():
    import hilberta_b200 as hb
    from hilberta_b200.plan import full_attention_plan

    plan = full_attention_plan(hb.bridge_k_plan(4, 1, False, grid_size=32))
    bank = hb.PlanBank(plan)
    sparse_model = _model(bank, 32, "hilberta")
    dense_model = _model(None, 32, "dense")  # same seed: same weights; raster order
    for a, b in zip(sparse_model.parameters(), dense_model.parameters()):
        assert torch.equal(a, b)
    x = _inputs(sparse_model, 32, plan.text_tokens)
    with torch.inference_mode():
        out_sparse = sparse_model(*x)
        out_dense = dense_model(*x)
    assert _rel(out_sparse, out_dense) < 2e-2


def test_step_requires_inference_mode():
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    model = _model(hb.PlanBank(plan), 32, "hilberta")
    with pytest.raises(RuntimeError, match="inference-only"):
        model(*_inputs(model, 32, plan.text_tokens))
