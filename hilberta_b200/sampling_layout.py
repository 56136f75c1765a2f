"""One entry and one exit permutation for a whole FLUX sampling trajectory.

``sample_flux_persistent(pipe, plan, ...)`` has the signature, refusals
(exception types and messages) and boundary counters of the reference's
sampling wrapper (hilberta/sampling_layout.py:21-148), for any pipeline with
the hooks of diffusers' ``FluxPipeline`` that matter here: ``prepare_latents``
(returns packed latents and their image position ids), ``_unpack_latents``
(called once, right before decoding), ``transformer`` and ``scheduler``.  No
diffusers import: the reference's exact-type checks on the pipeline and its
scheduler become checks of those hooks and of the scheduler's
``stochastic_sampling`` flag (a stochastic sampler's noise would not follow the
token permutation).

How it is built:

* ``_Trajectory`` is the layout boundary of one call, a three-state machine
  (raster -> packed -> restored) that owns the plan's permutation per device
  and the counters.  Its transitions are the only places tensors move: the
  first ``prepare_latents`` result is gathered into the plan's order (noise is
  still drawn in raster order, so a seed keeps its meaning), and the latents
  handed to ``_unpack_latents`` (or a latent-only return) are gathered back.
* ``_instance_override`` swaps one bound method on the pipeline instance for
  the duration of the call and puts back exactly what was there.
* the transformer runs inside ``persistent_flux_attention(...,
  layout_scope="sampling")``: every denoising step reads the packed tokens in
  place, with no per-step permutation.
"""

from __future__ import annotations

import contextlib

import torch

from .flux_adapter import persistent_flux_attention

# Marker on the pipeline while a call is in flight (the reference's attribute name).
_ACTIVE = "_flux_sampling_layout_active"
_HOOKS = ("prepare_latents", "_unpack_latents", "transformer", "scheduler")
_IP_ADAPTER_ARGUMENTS = ("ip_adapter_image", "ip_adapter_image_embeds", "negative_ip_adapter_image",
                         "negative_ip_adapter_image_embeds")
_PAIRED_OPTIONS = dict(global_strategy="triton", num_warps=8, num_stages=2)


def _refuse_unsupported(pipe, pipeline_kwargs):
    """Raise on a pipeline or call the wrapper cannot serve, before any work."""
    for hook in _HOOKS:
        if not hasattr(pipe, hook):
            raise TypeError(f"pipeline lacks {hook}: only FluxPipeline-style pipelines are supported")
    scheduler_config = getattr(pipe.scheduler, "config", None) or {}
    if scheduler_config.get("stochastic_sampling", False):
        raise ValueError("Stochastic scheduler noise requires token-identity-aware RNG")
    if getattr(pipe, _ACTIVE, False):
        raise RuntimeError("Nested sampling layout is unsupported")
    if pipeline_kwargs.get("callback_on_step_end") is not None:
        raise ValueError("Use packed_callback_on_step_end: its latents are in packed image order")
    if any(pipeline_kwargs.get(name) is not None for name in _IP_ADAPTER_ARGUMENTS):
        raise ValueError("IP-adapter needs a separate layout-aware implementation")


class _Trajectory:
    """Layout state of one sampling call: ``raster`` until the entry
    permutation, ``packed`` while denoising, ``restored`` after the exit."""

    def __init__(self, plan):
        self.image_tokens = int(plan.image_tokens)
        self._host = {"pack": plan.image_order.detach().cpu().clone(),
                      "restore": plan.inverse_image_order.detach().cpu().clone()}
        self._on_device = {}
        self.state = "raster"
        self.counters = dict(sampling_image_reorder_calls=0, sampling_id_reorder_calls=0, sampling_inverse_calls=0,
                             sampling_layout_read_write_bytes=0, callback_layout="packed",
                             public_output_layout="raster")

    def _move(self, x, dim, direction):
        key = (direction, str(x.device))
        index = self._on_device.get(key)
        if index is None:
            index = self._on_device[key] = self._host[direction].to(x.device)
        self.counters["sampling_layout_read_write_bytes"] += 2 * x.numel() * x.element_size()  # read + write
        return x.index_select(dim, index)

    def admit_entry(self):
        """Called before the pipeline's own prepare_latents runs."""
        if self.state != "raster":
            raise RuntimeError("Expected exactly one native prepare_latents call")

    def enter(self, latents, ids):
        if latents.ndim != 3 or latents.shape[1] != self.image_tokens:
            raise ValueError("Prepared image-token count does not match the plan")
        if ids.ndim not in (2, 3) or ids.shape[-2:] != (self.image_tokens, 3):
            raise ValueError("Prepared image position IDs do not match the plan")
        packed = (self._move(latents, 1, "pack"), self._move(ids, ids.ndim - 2, "pack"))
        self.counters["sampling_image_reorder_calls"] += 1
        self.counters["sampling_id_reorder_calls"] += 1
        self.state = "packed"
        return packed

    def leave(self, latents):
        if self.state != "packed":
            raise RuntimeError("Expected exactly one sampling entry and exit permutation")
        if latents.ndim != 3 or latents.shape[1] != self.image_tokens:
            raise ValueError("Final latent image-token count does not match the plan")
        raster = self._move(latents, 1, "restore")
        self.counters["sampling_inverse_calls"] += 1
        self.state = "restored"
        return raster

    def close(self):
        if self.state != "restored":
            raise RuntimeError("Native pipeline did not pass the sampling exit boundary")


@contextlib.contextmanager
def _instance_override(obj, name, value):
    """Set ``obj.name`` for the duration of the block, then put back exactly
    what the instance had: its own attribute, or none (so the class's method
    shows through again)."""
    own = vars(obj)
    had, old = name in own, own.get(name)
    setattr(obj, name, value)
    try:
        yield
    finally:
        if had:
            setattr(obj, name, old)
        else:
            own.pop(name, None)


def _latent_return(result, leave):
    """A latent-only pipeline return with its latents back in raster order."""
    if hasattr(result, "images"):
        return type(result)(images=leave(result.images))
    if isinstance(result, tuple) and len(result) == 1:
        return (leave(result[0]),)
    raise TypeError("Unexpected native Flux latent return type")


@torch.no_grad()
def sample_flux_persistent(pipe, plan, *, backend="paired", sdpa_backend="efficient", kernel_options=None,
                           packed_callback_on_step_end=None, **pipeline_kwargs):
    """Run ``pipe(**pipeline_kwargs)`` with the image tokens in the plan's packed
    order for the whole trajectory; returns ``(result, info)``, the result in
    public raster order.  ``packed_callback_on_step_end`` is passed to the
    pipeline as its ``callback_on_step_end`` and sees packed latents; a plain
    ``callback_on_step_end`` is refused.  Inference only, single-threaded,
    reversible: the pipeline's methods are as before afterwards."""
    _refuse_unsupported(pipe, pipeline_kwargs)
    if kernel_options is None and backend == "paired":
        kernel_options = dict(_PAIRED_OPTIONS)
    call = dict(pipeline_kwargs)
    if packed_callback_on_step_end is not None:
        call["callback_on_step_end"] = packed_callback_on_step_end
    trajectory = _Trajectory(plan)
    native_prepare, native_unpack = pipe.prepare_latents, pipe._unpack_latents

    def prepare_packed(*args, **kwargs):
        trajectory.admit_entry()
        return trajectory.enter(*native_prepare(*args, **kwargs))

    def unpack_raster(latents, *args, **kwargs):
        return native_unpack(trajectory.leave(latents), *args, **kwargs)

    with contextlib.ExitStack() as stack:
        setattr(pipe, _ACTIVE, True)
        stack.callback(delattr, pipe, _ACTIVE)
        info = stack.enter_context(persistent_flux_attention(
            pipe.transformer, plan, backend=backend, sdpa_backend=sdpa_backend, kernel_options=kernel_options,
            layout_scope="sampling"))
        stack.enter_context(_instance_override(pipe, "prepare_latents", prepare_packed))
        stack.enter_context(_instance_override(pipe, "_unpack_latents", unpack_raster))
        result = pipe(**call)
        if call.get("output_type") == "latent":
            result = _latent_return(result, trajectory.leave)
        trajectory.close()
        info.update(trajectory.counters)
        return result, info


__all__ = ["sample_flux_persistent"]
