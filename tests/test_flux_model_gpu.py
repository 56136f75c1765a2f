"""The reference adapter's entry, ``persistent_flux_attention`` (hilberta/
flux_adapter.py:343-430), on a FLUX.1-architecture model with small widths
(hilberta_b200/flux_model.py):

* backend "paired" (the sm_100a kernel) against "sdpa_reference" (torch SDPA
  under the plan's dense mask, the reference's correctness path) on the same
  weights and inputs;
* with a full-attention plan (hilberta/plan.py:200-212) against the model with
  dense attention outside the context: every op but attention is per-token, so
  the entry gather, the permuted rotary positions and the exit gather cancel;
* "sparse" equal to "paired"; the "sampling" layout scope; the info counters;
  processors restored on exit; the call checks, including a forward that
  raises.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _model():
    from hilberta_b200.flux_model import FluxTransformer

    torch.manual_seed(0)
    return FluxTransformer(num_double=2, num_single=3, dim=256, heads=2, text_dim=64, pooled_dim=32, device="cuda")


def _inputs(plan, batch=2):
    from hilberta_b200.flux_model import step_inputs

    x = step_inputs(plan.grid_size, plan.text_tokens, "cuda", batch=batch, seed=3, text_dim=64, pooled_dim=32)
    x["timestep"] = torch.tensor([0.3, 0.9][:batch], device="cuda")
    return x


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


def _run(model, plan, x, **kw):
    from hilberta_b200 import persistent_flux_attention

    with torch.inference_mode(), persistent_flux_attention(model, plan, **kw) as info:
        out = model(**x).sample
    return out, info


def test_paired_matches_sdpa_reference():
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    model, x = _model(), _inputs(plan)
    paired, info = _run(model, plan, x, backend="paired")
    ref, _ = _run(model, plan, x, backend="sdpa_reference")
    with torch.inference_mode():
        dense = model(**x).sample
    assert paired.shape == (2, 32 * 32, 64) and torch.isfinite(paired).all()
    # 5 layers of bf16 activations: relative L2 within 2 %, far below the
    # sparse-vs-dense distance
    assert _rel(paired, ref) < 2e-2
    assert _rel(dense, ref) > 5 * _rel(paired, ref)
    assert info["kernel"].startswith("sm_100a")
    assert hb.device_status() == 0


def test_full_plan_is_permutation_equivalent_to_dense():
    import hilberta_b200 as hb
    from hilberta_b200.plan import full_attention_plan

    plan = full_attention_plan(hb.bridge_k_plan(4, 1, False, grid_size=32))
    model, x = _model(), _inputs(plan)
    sparse, _ = _run(model, plan, x, backend="paired")
    with torch.inference_mode():
        dense = model(**x).sample  # raster order, dense SDPA
    assert _rel(sparse, dense) < 2e-2


def test_sparse_backend_sampling_scope_counters_and_restore():
    import hilberta_b200 as hb
    from hilberta_b200.flux_adapter import _ACTIVE

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    model, x = _model(), _inputs(plan)
    before = [m.processor for m in model.attention_modules()]
    with torch.inference_mode(), hb.persistent_flux_attention(model, plan, backend="paired") as info:
        a = model(**x).sample
        b = model(**x).sample
    assert torch.equal(a, b)
    assert info["transformer_calls"] == 2 and info["image_reorder_calls"] == 2 and info["image_inverse_calls"] == 2
    assert info["layer_calls"] == [2] * 5 and info["layer_phases"] == [0, 1, 2, 3, 0]
    assert info["joint_layers"] == 2 and info["single_layers"] == 3
    assert [m.processor for m in model.attention_modules()] == before
    assert not hasattr(model, _ACTIVE)
    sparse, _ = _run(model, plan, x, backend="sparse")
    assert torch.equal(sparse, a)
    # sampling scope: the caller keeps latents and ids in the plan's order
    order = plan.image_order.cuda()
    xs = dict(x, hidden_states=x["hidden_states"].index_select(1, order), img_ids=x["img_ids"].index_select(0, order))
    packed, info = _run(model, plan, xs, backend="paired", layout_scope="sampling")
    assert info["image_reorder_calls"] == 0 and info["image_inverse_calls"] == 0
    assert torch.equal(packed, a.index_select(1, order))


def test_call_checks_and_failed_forward():
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    model, x = _model(), _inputs(plan)
    with hb.persistent_flux_attention(model, plan, backend="paired"):
        with pytest.raises(RuntimeError, match="inference-only"):
            model(**x)
        with torch.inference_mode():
            with pytest.raises(ValueError, match="image-token count"):
                model(**dict(x, hidden_states=x["hidden_states"][:, :-64]))
            with pytest.raises(ValueError, match="LoRA scale"):
                model(**x, joint_attention_kwargs={"ip_adapter": 1})
            attn = model.transformer_blocks[0].attn
            with pytest.raises(RuntimeError, match="whole Transformer"):
                attn.processor(attn, torch.zeros(2, 1024, 256, device="cuda"))
            with pytest.raises(Exception):  # fails inside the forward, after the entry hook
                model(**dict(x, pooled_projections=x["pooled_projections"][:, :16]))
            out = model(**x).sample  # the failed call left no call in progress
    assert torch.isfinite(out).all()
