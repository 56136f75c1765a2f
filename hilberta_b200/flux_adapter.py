"""Transformer-scope adapter: run a FLUX transformer in a plan's persistent
token layout with HilbertA attention in every joint-attention call.

``persistent_flux_attention(model, plan, backend=...)`` keeps the reference
adapter's contract (hilberta/flux_adapter.py:149-256 and 343-440): its
arguments, the exception types and messages of its refusals, and the keys and
meaning of the ``info`` dict it yields.  It serves any model with the module
names and forward signature of diffusers' ``FluxTransformer2DModel``
(``transformer_blocks``, ``single_transformer_blocks``, ``attn.set_processor``,
``forward(hidden_states, encoder_hidden_states, ..., img_ids, txt_ids, ...)``).
Nothing here imports diffusers: the reference's type checks on the installed
processors become checks of their attributes (no parallel config, the native
attention backend).

How it is built:

* refusals are data: ``_Refusal`` rows (a test, an exception type, the
  message), checked in order by ``_refuse`` on the arguments, the model, each
  attention block and each transformer call;
* ``_Boundary`` owns the model-level hooks.  Its entry hook binds the call to
  the forward signature, applies the call refusals and hands ``hidden_states`` /
  ``img_ids`` to the scope; its exit hook (registered first, and run even when
  the forward raises) hands the prediction back to the scope;
* the scope is a strategy object: ``_GatherAtBoundary`` (``layout_scope=
  "transformer"``: one gather into the plan's order on entry and one back on
  exit per call) or ``_AlreadyPacked`` (``"sampling"``: the tokens stay packed
  for the whole trajectory, see ``sampling_layout``);
* everything the context changes is undone by an ``ExitStack`` in reverse
  order of installation: hooks, processors, the plan's device copies, the
  model's marker.

Every attention module runs layer ``i``'s processor on tile phase ``i % 4``
(flux_adapter.py:259-340): ``"paired"`` = ``HilbertAProcessor`` (fused Q/K/V
preparation and the sm_100a paired kernel on the phase's paired rows);
``"sparse"`` = the same preparation and ``sparse_attention`` on the phase's
unpaired rows (paired once per table, same kernel); ``"sdpa_reference"`` = the
correctness path, torch ops restating diffusers' RMSNorm and rotary embedding
and SDPA under the plan's dense mask.
"""

from __future__ import annotations

import contextlib
import inspect
from dataclasses import dataclass
from typing import Any, Callable

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

from .plan_bank import PlanBank
from .processor import HilbertAProcessor
from .sparse_kernel import sparse_attention

# Markers set on a model by this context and by the reference's image-mask
# context (nesting either one inside the other is refused).
_ACTIVE = "_flux_kernel_persistent_layout"
_MASK_CONTEXT = "_hilbert_flux_mask_context_active"
_SDP_BACKENDS = {"math": SDPBackend.MATH, "efficient": SDPBackend.EFFICIENT_ATTENTION}
_BACKENDS = ("sdpa_reference", "sparse", "paired")


@dataclass(frozen=True)
class _Refusal:
    applies: Callable[[Any], bool]
    error: type
    message: str


def _refuse(refusals, subject):
    """Raise the first refusal whose test holds for `subject`."""
    for r in refusals:
        if r.applies(subject):
            raise r.error(r.message)


def _tensor_with(x, ndims, tail):
    """x is a tensor of one of `ndims` ranks whose trailing shape is `tail`."""
    return isinstance(x, torch.Tensor) and x.ndim in ndims and tuple(x.shape[-len(tail):]) == tuple(tail)


_ARGUMENT_REFUSALS = (
    _Refusal(lambda a: a["layout_scope"] not in ("transformer", "sampling"), ValueError,
             "layout_scope must be transformer or sampling"),
    _Refusal(lambda a: a["backend"] not in _BACKENDS or a["sdpa_backend"] not in _SDP_BACKENDS, ValueError,
             "backend must be sdpa_reference/sparse/paired; sdpa_backend must be math/efficient"),
)

_MODEL_REFUSALS = (
    _Refusal(lambda m: getattr(m, _ACTIVE, False) or getattr(m, _MASK_CONTEXT, False), RuntimeError,
             "Nested/conflicting Flux layout or image-mask contexts are unsupported"),
    _Refusal(lambda m: m.training or getattr(m, "gradient_checkpointing", False), ValueError,
             "Native Flux model must be in eval mode without gradient checkpointing"),
    _Refusal(lambda m: getattr(m, "_cache_config", None) is not None, ValueError,
             "Transformer cache state needs a separate layout-aware implementation"),
    _Refusal(lambda m: len(m.transformer_blocks) == 0 or len(m.single_transformer_blocks) == 0, ValueError,
             "Both native Flux joint and single blocks are required"),
)

# subject: (block, is_joint)
_BLOCK_REFUSALS = (
    _Refusal(lambda b: isinstance(b[0].attn.processor, PersistentFluxProcessor)
             or getattr(b[0].attn.processor, "_attention_backend", None) not in (None, "native")
             or getattr(b[0].attn.processor, "_parallel_config", None) is not None, ValueError,
             "Only native, non-parallel Diffusers FluxAttnProcessor is supported"),
    _Refusal(lambda b: (b[0].attn.added_kv_proj_dim is not None) != b[1], ValueError,
             "Native joint/single projection types disagree with block layout"),
)

# subject: (arguments of the bound forward call, plan bank)
_CALL_REFUSALS = (
    _Refusal(lambda c: not (isinstance(c[0].get("hidden_states"), torch.Tensor) and c[0]["hidden_states"].ndim == 3
                            and c[0]["hidden_states"].shape[1] == c[1].image_tokens), ValueError,
             "hidden_states image-token count does not match the plan"),
    _Refusal(lambda c: not (isinstance(c[0].get("encoder_hidden_states"), torch.Tensor)
                            and c[0]["encoder_hidden_states"].ndim == 3
                            and c[0]["encoder_hidden_states"].shape[:2] == (c[0]["hidden_states"].shape[0],
                                                                            c[1].text_tokens)), ValueError,
             "encoder_hidden_states batch/text-token count does not match the plan"),
    _Refusal(lambda c: not _tensor_with(c[0].get("img_ids"), (2, 3), (c[1].image_tokens, 3)), ValueError,
             "img_ids must match image token identities with final shape [image_tokens,3]"),
    _Refusal(lambda c: not _tensor_with(c[0].get("txt_ids"), (2, 3), (c[1].text_tokens, 3)), ValueError,
             "txt_ids must match the native text prefix"),
    _Refusal(lambda c: c[0].get("controlnet_block_samples") is not None
             or c[0].get("controlnet_single_block_samples") is not None, ValueError,
             "ControlNet residuals require a separate layout-aware implementation"),
    _Refusal(lambda c: c[0].get("joint_attention_kwargs") is not None
             and (not isinstance(c[0]["joint_attention_kwargs"], dict) or set(c[0]["joint_attention_kwargs"]) - {"scale"}),
             ValueError, "Only native scalar LoRA scale is supported in joint_attention_kwargs; no IP-adapter/extra masks"),
)


class _GatherAtBoundary:
    """layout_scope="transformer": raster tensors at the model's boundary; the
    image tokens (and their position ids) are gathered into the plan's order
    when a call enters and the prediction is gathered back when it leaves."""

    def __init__(self, bank, info):
        self.bank, self.info = bank, info

    def _gather(self, x, dim, which):
        self.info["image_layout_gather_read_write_bytes"] += 2 * x.numel() * x.element_size()
        return x.index_select(dim, self.bank.on_device(x.device)[which])

    def enter(self, arguments):
        hidden, ids = arguments["hidden_states"], arguments["img_ids"]
        ids_moved = ids.index_select(ids.ndim - 2, self.bank.on_device(ids.device)["order"])
        arguments["hidden_states"] = self._gather(hidden, 1, "order")
        arguments["img_ids"] = ids_moved
        self.info["image_reorder_calls"] += 1
        self.info["image_id_reorder_calls"] += 1

    def leave(self, prediction):
        self.info["image_inverse_calls"] += 1
        return self._gather(prediction, 1, "inverse")


class _AlreadyPacked:
    """layout_scope="sampling": the caller keeps the tokens in the plan's order
    for the whole trajectory; nothing moves at the model's boundary."""

    def enter(self, arguments):
        pass

    def leave(self, prediction):
        return prediction


def _split_prediction(output):
    """(prediction tensor, function rebuilding the output around a new one) of a
    transformer output: an object with ``sample`` or a one-element tuple."""
    if hasattr(output, "sample"):
        return output.sample, lambda t: type(output)(sample=t)
    if isinstance(output, tuple) and len(output) == 1:
        return output[0], lambda t: (t,)
    raise TypeError("Expected native Flux Transformer2DModelOutput or one-element tuple")


class _Boundary:
    """The model-level hooks of one context.  ``in_forward`` is true between a
    call's entry and exit hooks; the processors refuse to run outside it."""

    def __init__(self, model, bank, info, scope):
        self.bank, self.info, self.scope = bank, info, scope
        self._bind = inspect.signature(model.forward).bind
        self.in_forward = False
        self._batch = None

    def on_entry(self, module, args, kwargs):
        if self.in_forward:
            raise RuntimeError("Reentrant Transformer forwards are unsupported in persistent-layout context")
        if torch.is_grad_enabled():
            raise RuntimeError("Persistent sparse Flux is inference-only; use torch.no_grad or inference_mode")
        call = self._bind(*args, **kwargs)
        _refuse(_CALL_REFUSALS, (call.arguments, self.bank))
        self._batch = call.arguments["hidden_states"].shape[0]
        self.scope.enter(call.arguments)
        self.in_forward = True
        self.info["transformer_calls"] += 1
        return call.args, call.kwargs

    def on_exit(self, module, args, output):
        was_running, self.in_forward = self.in_forward, False  # also after a forward that raised
        if output is None or not was_running:
            return output
        prediction, rebuild = _split_prediction(output)
        if prediction.ndim != 3 or tuple(prediction.shape[:2]) != (self._batch, self.bank.image_tokens):
            raise ValueError("Transformer output shape does not match image layout")
        moved = self.scope.leave(prediction)
        return output if moved is prediction else rebuild(moved)


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


def _info(backend, sdpa_backend, kernel_options, layout_scope, joint, single):
    """The ``info`` dict the context yields: its settings, then counters the
    hooks, processors and plan bank advance."""
    layers = joint + single
    boundary = "one Transformer-entry/exit gather" if layout_scope == "transformer" else "packed throughout sampling"
    settings = dict(backend=backend, sdpa_backend=sdpa_backend, kernel_options=dict(kernel_options),
                    layout_scope=layout_scope)
    counters = dict.fromkeys(("transformer_calls", "image_reorder_calls", "image_inverse_calls",
                              "image_id_reorder_calls", "per_layer_image_permutations", "metadata_device_copies",
                              "reference_masks_prepared", "image_layout_gather_read_write_bytes"), 0)
    layout = dict(layer_calls=[0] * layers, layer_phases=[i % 4 for i in range(layers)], joint_layers=joint,
                  single_layers=single, layout="native text prefix; shared image prefix; remaining image tokens; "
                  + boundary)
    guarantees = dict(shared_tokens_keep_image_projections=True, native_dynamic_text_preserved=True,
                      precision="unchanged; native QK RMSNorm and RoPE", weights_modified=False,
                      kernel="torch SDPA, dense plan mask" if backend == "sdpa_reference"
                      else "sm_100a paired (hb_paired_fwd)")
    return {**settings, **counters, **layout, **guarantees}


@contextlib.contextmanager
def persistent_flux_attention(model, plan, backend="sdpa_reference", sdpa_backend="math", kernel_options=None, *,
                              layout_scope="transformer"):
    """Reversibly run a FLUX transformer in the plan's persistent layout:
    processors installed on entry and restored on exit, plan metadata checked
    once and copied once per device, the ``info`` dict yielded.  Single-
    threaded; reentrant forwards, ControlNet residuals and IP-adapter inputs are
    refused.  With ``layout_scope="sampling"`` the caller passes inputs already
    in the plan's order and gets packed predictions back
    (``sample_flux_persistent`` manages that)."""
    _refuse(_ARGUMENT_REFUSALS, dict(layout_scope=layout_scope, backend=backend, sdpa_backend=sdpa_backend))
    _refuse(_MODEL_REFUSALS, model)
    joint, single = list(model.transformer_blocks), list(model.single_transformer_blocks)
    blocks = joint + single
    for i, block in enumerate(blocks):
        _refuse(_BLOCK_REFUSALS, (block, i < len(joint)))
    options = dict(kernel_options or {})
    info = _info(backend, sdpa_backend, options, layout_scope, len(joint), len(single))
    bank = PlanBank(plan, info)
    info["image_order_sha256"] = bank.order_hash
    scope = _GatherAtBoundary(bank, info) if layout_scope == "transformer" else _AlreadyPacked()
    boundary = _Boundary(model, bank, info, scope)
    with contextlib.ExitStack() as undo:
        setattr(model, _ACTIVE, True)
        undo.callback(delattr, model, _ACTIVE)
        undo.callback(bank.clear)
        saved = [block.attn.processor for block in blocks]
        undo.callback(lambda: [b.attn.set_processor(p) for b, p in zip(blocks, saved)])
        for i, block in enumerate(blocks):
            block.attn.set_processor(PersistentFluxProcessor(boundary, i, backend, options))
        # hooks registered earlier by others still see raster inputs; the exit
        # hook goes first so their post-hooks see raster predictions
        undo.callback(model.register_forward_pre_hook(boundary.on_entry, with_kwargs=True).remove)
        undo.callback(model.register_forward_hook(boundary.on_exit, prepend=True, always_call=True).remove)
        undo.enter_context(sdpa_kernel([_SDP_BACKENDS[sdpa_backend]]))
        yield info


__all__ = ["persistent_flux_attention", "PersistentFluxProcessor"]
