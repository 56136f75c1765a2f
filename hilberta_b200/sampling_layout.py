"""One entry and one exit permutation for a whole FLUX sampling trajectory.

``sample_flux_persistent(pipe, plan, ...)`` is the reference's sampling wrapper
(hilberta/sampling_layout.py:21-165) for any pipeline with diffusers'
``FluxPipeline`` hooks: ``prepare_latents`` (returns packed latents and their
image position ids), ``_unpack_latents`` (called once, right before decoding),
``transformer`` and ``scheduler``.  The wrapper replaces those two methods for the
duration of one call:

* the first ``prepare_latents`` draws the initial noise in raster order (the
  seed keeps its meaning) and gathers latents and ids into the plan's order;
* the transformer then runs inside ``persistent_flux_attention(...,
  layout_scope="sampling")``: latents stay packed through every denoising step,
  with no per-step permutation;
* ``_unpack_latents`` gathers them back to raster order once before decoding,
  and a latent-only return is restored explicitly.

Nothing here imports diffusers; the reference's type checks on the pipeline and
scheduler become checks of the hooks the wrapper needs and of the scheduler's
``stochastic_sampling`` flag (a stochastic sampler's noise would not follow the
token permutation).
"""

from __future__ import annotations

import torch

from .flux_adapter import persistent_flux_attention

_ACTIVE = "_flux_sampling_layout_active"
_MISSING = object()


@torch.no_grad()
def sample_flux_persistent(pipe, plan, *, backend="paired", sdpa_backend="efficient", kernel_options=None,
                           packed_callback_on_step_end=None, **pipeline_kwargs):
    """Run ``pipe(**pipeline_kwargs)`` in the plan's packed layout; returns
    ``(result, info)`` with the result in public raster order."""
    for name in ("prepare_latents", "_unpack_latents", "transformer", "scheduler"):
        if not hasattr(pipe, name):
            raise TypeError(f"pipeline lacks {name}: only FluxPipeline-style pipelines are supported")
    config = getattr(pipe.scheduler, "config", {}) or {}
    if config.get("stochastic_sampling", False):
        raise ValueError("Stochastic scheduler noise requires token-identity-aware RNG")
    if getattr(pipe, _ACTIVE, False):
        raise RuntimeError("Nested sampling layout is unsupported")
    if pipeline_kwargs.get("callback_on_step_end") is not None:
        raise ValueError("Use packed_callback_on_step_end: its latents are in packed image order")
    for name in ("ip_adapter_image", "ip_adapter_image_embeds", "negative_ip_adapter_image",
                 "negative_ip_adapter_image_embeds"):
        if pipeline_kwargs.get(name) is not None:
            raise ValueError("IP-adapter needs a separate layout-aware implementation")
    if kernel_options is None and backend == "paired":
        kernel_options = dict(global_strategy="triton", num_warps=8, num_stages=2)
    if packed_callback_on_step_end is not None:
        pipeline_kwargs["callback_on_step_end"] = packed_callback_on_step_end
    order = plan.image_order.detach().cpu().clone()
    inverse = plan.inverse_image_order.detach().cpu().clone()
    n = int(plan.image_tokens)
    per_device = {}

    def indices(device):
        key = str(device)
        if key not in per_device:
            per_device[key] = (order.to(device), inverse.to(device))
        return per_device[key]

    boundary = dict(sampling_image_reorder_calls=0, sampling_id_reorder_calls=0, sampling_inverse_calls=0,
                    sampling_layout_read_write_bytes=0, callback_layout="packed", public_output_layout="raster")
    originals = {name: pipe.__dict__.get(name, _MISSING) for name in ("prepare_latents", "_unpack_latents")}
    prepare, unpack = pipe.prepare_latents, pipe._unpack_latents

    def packed_prepare(*args, **kwargs):
        if boundary["sampling_image_reorder_calls"]:
            raise RuntimeError("Expected exactly one native prepare_latents call")
        latent, ids = prepare(*args, **kwargs)
        if latent.ndim != 3 or latent.shape[1] != n:
            raise ValueError("Prepared image-token count does not match the plan")
        if ids.ndim not in (2, 3) or ids.shape[-2:] != (n, 3):
            raise ValueError("Prepared image position IDs do not match the plan")
        latent = latent.index_select(1, indices(latent.device)[0])
        ids = ids.index_select(ids.ndim - 2, indices(ids.device)[0])
        boundary["sampling_image_reorder_calls"] += 1
        boundary["sampling_id_reorder_calls"] += 1
        boundary["sampling_layout_read_write_bytes"] += 2 * (
            latent.numel() * latent.element_size() + ids.numel() * ids.element_size())
        return latent, ids

    def restore(latent):
        if boundary["sampling_image_reorder_calls"] != 1 or boundary["sampling_inverse_calls"]:
            raise RuntimeError("Expected exactly one sampling entry and exit permutation")
        if latent.ndim != 3 or latent.shape[1] != n:
            raise ValueError("Final latent image-token count does not match the plan")
        out = latent.index_select(1, indices(latent.device)[1])
        boundary["sampling_inverse_calls"] += 1
        boundary["sampling_layout_read_write_bytes"] += 2 * latent.numel() * latent.element_size()
        return out

    def raster_unpack(latents, *args, **kwargs):
        return unpack(restore(latents), *args, **kwargs)

    setattr(pipe, _ACTIVE, True)
    try:
        with persistent_flux_attention(pipe.transformer, plan, backend=backend, sdpa_backend=sdpa_backend,
                                       kernel_options=kernel_options, layout_scope="sampling") as info:
            pipe.prepare_latents = packed_prepare
            pipe._unpack_latents = raster_unpack
            result = pipe(**pipeline_kwargs)
            if pipeline_kwargs.get("output_type") == "latent":
                if hasattr(result, "images"):
                    result = type(result)(images=restore(result.images))
                elif isinstance(result, tuple) and len(result) == 1:
                    result = (restore(result[0]),)
                else:
                    raise TypeError("Unexpected native Flux latent return type")
            if boundary["sampling_inverse_calls"] != 1:
                raise RuntimeError("Native pipeline did not pass the sampling exit boundary")
            info.update(boundary)
            return result, info
    finally:
        for name, old in originals.items():
            if old is _MISSING:
                pipe.__dict__.pop(name, None)
            else:
                setattr(pipe, name, old)
        delattr(pipe, _ACTIVE)


__all__ = ["sample_flux_persistent"]
