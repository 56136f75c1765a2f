"""sample_flux_persistent (hilberta/sampling_layout.py:21-165) around a tiny
pipeline with FluxPipeline's hooks and a per-token Euler loop: with the
latents packed once for the whole trajectory, the result equals (bit for bit)
the same pipeline run inside persistent_flux_attention with the transformer-
scope gathers at every call; the latent-only return is restored to raster
order; callbacks see packed latents; counters and the pipeline's own methods
are as before afterwards."""

from __future__ import annotations

import pytest
import torch

from tests._tiny_pipe import TinyPipe

pytestmark = pytest.mark.gpu


def _setup():
    import hilberta_b200 as hb
    from hilberta_b200.flux_model import FluxTransformer

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    torch.manual_seed(0)
    model = FluxTransformer(num_double=2, num_single=2, dim=256, heads=2, text_dim=64, pooled_dim=32, device="cuda")
    return hb, plan, TinyPipe(model, 32, plan.text_tokens)


def test_sampling_scope_equals_transformer_scope():
    hb, plan, pipe = _setup()
    with torch.inference_mode(), hb.persistent_flux_attention(pipe.transformer, plan, backend="paired") as tinfo:
        want = pipe(steps=3, seed=4).images
    assert tinfo["image_reorder_calls"] == 3
    seen = []
    with torch.inference_mode():
        got, info = hb.sample_flux_persistent(pipe, plan, steps=3, seed=4,
                                              packed_callback_on_step_end=lambda p, i, t, d: seen.append(d["latents"]))
    assert torch.equal(got.images, want)
    assert info["sampling_image_reorder_calls"] == 1 and info["sampling_inverse_calls"] == 1
    assert info["transformer_calls"] == 3 and info["image_reorder_calls"] == 0
    assert info["layout_scope"] == "sampling" and len(seen) == 3
    # callbacks saw packed latents: the raster latents gathered by the plan's order
    raster_last = want.reshape(1, -1, 64)
    assert torch.equal(seen[-1], raster_last.index_select(1, plan.image_order.cuda()))
    assert "prepare_latents" not in pipe.__dict__ and "_unpack_latents" not in pipe.__dict__


def test_latent_output_is_restored():
    hb, plan, pipe = _setup()
    with torch.inference_mode():
        images, _ = hb.sample_flux_persistent(pipe, plan, steps=2, seed=5)
        latents, info = hb.sample_flux_persistent(pipe, plan, steps=2, seed=5, output_type="latent")
    assert info["sampling_inverse_calls"] == 1
    assert torch.equal(latents.images.reshape(images.images.shape), images.images)
