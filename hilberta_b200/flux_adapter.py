"""Transformer-scope adapter: run a FLUX transformer in a plan's persistent
token layout with HilbertA attention in every joint-attention call.

``persistent_flux_attention(model, plan, backend=...)`` is the reference
adapter's entry (hilberta/flux_adapter.py:343-430): the same arguments, checks,
messages and ``info`` counters, for any model with the module names and forward
signature of diffusers' ``FluxTransformer2DModel`` (``transformer_blocks``,
``single_transformer_blocks``, ``attn.set_processor``, ``forward(hidden_states,
encoder_hidden_states, ..., img_ids, txt_ids, ...)``).  Nothing here imports
diffusers: the reference's type checks on the installed processors become checks
of their attributes (no parallel config, native attention backend).

Inside the context:

* a forward pre-hook checks the call (inference only, token counts, no
  ControlNet residuals, only a LoRA ``scale`` in ``joint_attention_kwargs``) and,
  with ``layout_scope="transformer"``, gathers ``hidden_states`` and ``img_ids``
  into the plan's physical order once; a post-hook (which also runs when the
  forward raises) gathers the prediction back to raster order
  (flux_adapter.py:149-256);
* every attention module runs layer ``i``'s processor on phase ``i % 4``
  (flux_adapter.py:259-340): ``"paired"`` = ``HilbertAProcessor`` (fused Q/K/V
  preparation + the sm_100a paired kernel on the phase's paired rows);
  ``"sparse"`` = the same preparation and ``sparse_attention`` on the phase's
  unpaired rows (which pairs them once and runs the same kernel);
  ``"sdpa_reference"`` = the correctness path, torch ops restating diffusers'
  RMSNorm and rotary embedding and SDPA under the plan's dense mask.
"""

from __future__ import annotations

import contextlib
import inspect

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

from .plan_bank import PlanBank
from .processor import HilbertAProcessor
from .sparse_kernel import sparse_attention

_ACTIVE = "_flux_kernel_persistent_layout"
_SDP_BACKENDS = {"math": SDPBackend.MATH, "efficient": SDPBackend.EFFICIENT_ATTENTION}


class _Runtime:
    """Call state of one context: the plan bank, the model's forward signature,
    whether a transformer call is in progress."""

    def __init__(self, model, bank, info):
        self.bank, self.info = bank, info
        self.signature = inspect.signature(model.forward)
        self.in_forward = False
        self.expected_output_batch = None

    def before(self, model, args, kwargs):
        if self.in_forward:
            raise RuntimeError("Reentrant Transformer forwards are unsupported in persistent-layout context")
        if torch.is_grad_enabled():
            raise RuntimeError("Persistent sparse Flux is inference-only; use torch.no_grad or inference_mode")
        bound = self.signature.bind(*args, **kwargs)
        values = bound.arguments
        hidden, text = values.get("hidden_states"), values.get("encoder_hidden_states")
        ids, text_ids = values.get("img_ids"), values.get("txt_ids")
        bank = self.bank
        if not isinstance(hidden, torch.Tensor) or hidden.ndim != 3 or hidden.shape[1] != bank.image_tokens:
            raise ValueError("hidden_states image-token count does not match the plan")
        if not isinstance(text, torch.Tensor) or text.ndim != 3 or text.shape[:2] != (hidden.shape[0], bank.text_tokens):
            raise ValueError("encoder_hidden_states batch/text-token count does not match the plan")
        if not isinstance(ids, torch.Tensor) or ids.ndim not in (2, 3) or ids.shape[-2:] != (bank.image_tokens, 3):
            raise ValueError("img_ids must match image token identities with final shape [image_tokens,3]")
        if (not isinstance(text_ids, torch.Tensor) or text_ids.ndim not in (2, 3)
                or text_ids.shape[-2:] != (bank.text_tokens, 3)):
            raise ValueError("txt_ids must match the native text prefix")
        if values.get("controlnet_block_samples") is not None or values.get("controlnet_single_block_samples") is not None:
            raise ValueError("ControlNet residuals require a separate layout-aware implementation")
        extra = values.get("joint_attention_kwargs")
        if extra is not None and (not isinstance(extra, dict) or set(extra) - {"scale"}):
            raise ValueError(
                "Only native scalar LoRA scale is supported in joint_attention_kwargs; no IP-adapter/extra masks")
        if self.info["layout_scope"] == "transformer":
            values["hidden_states"] = hidden.index_select(1, bank.on_device(hidden.device)["order"])
            values["img_ids"] = ids.index_select(ids.ndim - 2, bank.on_device(ids.device)["order"])
            self.info["image_reorder_calls"] += 1
            self.info["image_id_reorder_calls"] += 1
            self.info["image_layout_gather_read_write_bytes"] += 2 * hidden.numel() * hidden.element_size()
        self.expected_output_batch = hidden.shape[0]
        self.in_forward = True
        self.info["transformer_calls"] += 1
        return bound.args, bound.kwargs

    def after(self, model, args, output):
        # registered with always_call: a forward that raised still clears the
        # call state here (and has no prediction to restore)
        active, self.in_forward = self.in_forward, False
        if output is None or not active:
            return output
        if hasattr(output, "sample"):
            value = output.sample
        elif isinstance(output, tuple) and len(output) == 1:
            value = output[0]
        else:
            raise TypeError("Expected native Flux Transformer2DModelOutput or one-element tuple")
        if value.ndim != 3 or value.shape[:2] != (self.expected_output_batch, self.bank.image_tokens):
            raise ValueError("Transformer output shape does not match image layout")
        if self.info["layout_scope"] == "sampling":
            return output
        restored = value.index_select(1, self.bank.on_device(value.device)["inverse"])
        self.info["image_inverse_calls"] += 1
        self.info["image_layout_gather_read_write_bytes"] += 2 * value.numel() * value.element_size()
        return type(output)(sample=restored) if hasattr(output, "sample") else (restored,)


def _rms_norm(x, norm):
    """diffusers 0.36 RMSNorm: fp32 mean of squares, x * rsqrt(v + eps) in the
    input dtype, times the weight (when it has one)."""
    v = x.to(torch.float32).pow(2).mean(-1, keepdim=True)
    y = x * torch.rsqrt(v + norm.eps)
    w = getattr(norm, "weight", None)
    if w is None:
        return y.to(x.dtype)
    if w.dtype in (torch.float16, torch.bfloat16):
        y = y.to(w.dtype)
    return y * w


def _rotary(x, cos, sin):
    """diffusers' apply_rotary_emb (real cos/sin, pairs (2i, 2i+1)) on [B, S, H, D]."""
    re, im = x.reshape(*x.shape[:-1], -1, 2).unbind(-1)
    rot = torch.stack([-im, re], dim=-1).flatten(3)
    return (x.float() * cos[None, :, None] + rot.float() * sin[None, :, None]).to(x.dtype)


class _SparseRowsProcessor(HilbertAProcessor):
    """``HilbertAProcessor`` whose attention is ``sparse_attention`` on the
    phase's unpaired rows, as the reference's "sparse" backend calls it
    (flux_adapter.py:313-326)."""

    def _attend(self, q, k, v):
        ids, counts = self.bank.on_device(q.device)["phases"][self.phase]
        return sparse_attention(q, k, v, ids, counts, global_tokens=self.bank.global_tokens,
                                block_size=self.bank.block_size, **self.kernel_options)


class PersistentFluxProcessor:
    """Layer ``layer``'s processor inside ``persistent_flux_attention``."""

    def __init__(self, runtime, layer, backend, kernel_options):
        self.runtime, self.layer, self.phase = runtime, int(layer), int(layer) % 4
        self.backend, self.kernel_options = backend, dict(kernel_options)
        native = {"paired": HilbertAProcessor, "sparse": _SparseRowsProcessor}.get(backend)
        self.native = native(runtime.bank, layer, kernel_options) if native is not None else None

    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None, image_rotary_emb=None):
        if not self.runtime.in_forward:
            raise RuntimeError("Call the whole Transformer so the persistent image layout is established")
        if attention_mask is not None:
            raise ValueError("External attention masks cannot be combined implicitly with the registered plan")
        if self.native is not None:
            out = self.native(attn, hidden_states, encoder_hidden_states, None, image_rotary_emb)
        else:
            out = self._reference(attn, hidden_states, encoder_hidden_states, image_rotary_emb)
        self.runtime.info["layer_calls"][self.layer] += 1
        return out

    def _reference(self, attn, hidden_states, encoder_hidden_states, image_rotary_emb):
        """Dense-mask SDPA after the processor's own steps (flux_adapter.py:
        276-307, sdpa_reference backend)."""
        bank = self.runtime.bank
        h = attn.heads
        split = lambda t: t.unflatten(-1, (h, -1))
        q = _rms_norm(split(attn.to_q(hidden_states)), attn.norm_q)
        k = _rms_norm(split(attn.to_k(hidden_states)), attn.norm_k)
        v = split(attn.to_v(hidden_states))
        if encoder_hidden_states is not None and attn.added_kv_proj_dim is not None:
            q = torch.cat([_rms_norm(split(attn.add_q_proj(encoder_hidden_states)), attn.norm_added_q), q], dim=1)
            k = torch.cat([_rms_norm(split(attn.add_k_proj(encoder_hidden_states)), attn.norm_added_k), k], dim=1)
            v = torch.cat([split(attn.add_v_proj(encoder_hidden_states)), v], dim=1)
        if image_rotary_emb is not None:
            q, k = _rotary(q, *image_rotary_emb), _rotary(k, *image_rotary_emb)
        if q.shape[1] != bank.total_tokens:
            raise ValueError("Native attention sequence length does not match the plan")
        out = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                             attn_mask=bank.dense_mask(self.phase, q.device))
        out = out.transpose(1, 2).flatten(2, 3).to(q.dtype)
        if encoder_hidden_states is None:
            return out
        text, image = out.split_with_sizes(
            [encoder_hidden_states.shape[1], out.shape[1] - encoder_hidden_states.shape[1]], dim=1)
        return attn.to_out[1](attn.to_out[0](image)), attn.to_add_out(text)


@contextlib.contextmanager
def persistent_flux_attention(model, plan, backend="sdpa_reference", sdpa_backend="math", kernel_options=None, *,
                              layout_scope="transformer"):
    """Reversibly run a FLUX transformer in the plan's persistent layout
    (flux_adapter.py:343-430): processors installed on entry and restored on
    exit, plan metadata moved once per device, yields the ``info`` dict."""
    if layout_scope not in ("transformer", "sampling"):
        raise ValueError("layout_scope must be transformer or sampling")
    if backend not in ("sdpa_reference", "sparse", "paired") or sdpa_backend not in _SDP_BACKENDS:
        raise ValueError("backend must be sdpa_reference/sparse/paired; sdpa_backend must be math/efficient")
    if getattr(model, _ACTIVE, False) or getattr(model, "_hilbert_flux_mask_context_active", False):
        raise RuntimeError("Nested/conflicting Flux layout or image-mask contexts are unsupported")
    if model.training or getattr(model, "gradient_checkpointing", False):
        raise ValueError("Native Flux model must be in eval mode without gradient checkpointing")
    if getattr(model, "_cache_config", None) is not None:
        raise ValueError("Transformer cache state needs a separate layout-aware implementation")
    joint, single = list(model.transformer_blocks), list(model.single_transformer_blocks)
    if not joint or not single:
        raise ValueError("Both native Flux joint and single blocks are required")
    blocks = joint + single
    originals = [block.attn.processor for block in blocks]
    for i, (block, processor) in enumerate(zip(blocks, originals)):
        if (isinstance(processor, PersistentFluxProcessor)
                or getattr(processor, "_attention_backend", None) not in (None, "native")
                or getattr(processor, "_parallel_config", None) is not None):
            raise ValueError("Only native, non-parallel Diffusers FluxAttnProcessor is supported")
        if (block.attn.added_kv_proj_dim is not None) != (i < len(joint)):
            raise ValueError("Native joint/single projection types disagree with block layout")
    info = {
        "backend": backend,
        "sdpa_backend": sdpa_backend,
        "kernel_options": dict(kernel_options or {}),
        "layout_scope": layout_scope,
        "transformer_calls": 0,
        "image_reorder_calls": 0,
        "image_inverse_calls": 0,
        "image_id_reorder_calls": 0,
        "per_layer_image_permutations": 0,
        "layer_calls": [0] * len(blocks),
        "layer_phases": [i % 4 for i in range(len(blocks))],
        "joint_layers": len(joint),
        "single_layers": len(single),
        "metadata_device_copies": 0,
        "reference_masks_prepared": 0,
        "image_layout_gather_read_write_bytes": 0,
        "layout": "native text prefix; shared image prefix; remaining image tokens; "
        + ("one Transformer-entry/exit gather" if layout_scope == "transformer" else "packed throughout sampling"),
        "shared_tokens_keep_image_projections": True,
        "native_dynamic_text_preserved": True,
        "precision": "unchanged; native QK RMSNorm and RoPE",
        "weights_modified": False,
        "kernel": "sm_100a paired (hb_paired_fwd)" if backend != "sdpa_reference" else "torch SDPA, dense plan mask",
    }
    bank = PlanBank(plan, info)
    info["image_order_sha256"] = bank.order_hash
    runtime = _Runtime(model, bank, info)
    handles = []
    setattr(model, _ACTIVE, True)
    try:
        for i, block in enumerate(blocks):
            block.attn.set_processor(PersistentFluxProcessor(runtime, i, backend, kernel_options or {}))
        # outside hooks registered earlier still see raster inputs; the restore
        # runs first so outside post-hooks see raster predictions
        handles.append(model.register_forward_pre_hook(runtime.before, with_kwargs=True))
        handles.append(model.register_forward_hook(runtime.after, prepend=True, always_call=True))
        with sdpa_kernel([_SDP_BACKENDS[sdpa_backend]]):
            yield info
    finally:
        for handle in handles:
            handle.remove()
        for block, processor in zip(blocks, originals):
            block.attn.set_processor(processor)
        bank.clear()
        delattr(model, _ACTIVE)


__all__ = ["persistent_flux_attention", "PersistentFluxProcessor"]
