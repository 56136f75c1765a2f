"""FLUX joint-attention processor on this package's kernels.

The call of the reference adapter's ``PersistentFluxProcessor``
(hilberta/flux_adapter.py:259-340), for any attention module with the
attributes of diffusers' ``FluxAttention`` (``heads``, ``to_q``/``to_k``/
``to_v``, ``norm_q``/``norm_k`` with ``weight`` and ``eps``; for double-stream
blocks ``added_kv_proj_dim``, ``add_q_proj``/``add_k_proj``/``add_v_proj``,
``norm_added_q``/``norm_added_k``, ``to_out`` and ``to_add_out``).  Nothing here
imports diffusers: the projections are the module's own layers, and the steps
between them run as

* ``prepare_qkv``: per-head RMSNorm, text tokens first, rotary embedding and the
  ``[B, S, H, D]`` packing in one pass per tensor (``hb_norm_rope_pack``);
* ``paired_attention`` on the plan's paired metadata of phase ``layer % 4``
  (``PlanBank.on_device``), reading the packed tensors in place;
* the output split and projections of the reference (``to_out[0]``,
  ``to_out[1]``, ``to_add_out``).

Tokens arrive in the order the plan's metadata indexes (the reference permutes
latents once per image or per transformer call, ``sampling_layout.py:88-116``,
``flux_adapter.py:208-217``); the layer-counting runtime around the processors
stays with the caller.
"""

from __future__ import annotations

import torch

from .paired_kernel import paired_attention
from .prep import norm_rope_pack


class HilbertAProcessor:
    """Processor for one transformer layer: ``__call__(attn, hidden_states,
    encoder_hidden_states=None, attention_mask=None, image_rotary_emb=None)`` as
    diffusers calls it."""

    def __init__(self, bank, layer, kernel_options=None):
        self.bank, self.layer, self.phase = bank, int(layer), int(layer) % 4
        self.kernel_options = dict(kernel_options or {})

    def attention(self, attn, hidden_states, encoder_hidden_states=None, image_rotary_emb=None):
        """The attention output ``[B, S, H*D]`` (text tokens first) before the
        output projections."""
        if torch.is_grad_enabled():
            raise RuntimeError("HilbertA attention is inference-only; use torch.no_grad or inference_mode")
        heads = attn.heads
        cos, sin = (None, None) if image_rotary_emb is None else image_rotary_emb
        if encoder_hidden_states is not None and getattr(attn, "added_kv_proj_dim", None) is not None:
            streams = [
                (attn.add_q_proj(encoder_hidden_states), attn.to_q(hidden_states), attn.norm_added_q, attn.norm_q),
                (attn.add_k_proj(encoder_hidden_states), attn.to_k(hidden_states), attn.norm_added_k, attn.norm_k),
                (attn.add_v_proj(encoder_hidden_states), attn.to_v(hidden_states), None, None),
            ]
        else:  # single-stream block: text and image tokens already concatenated
            streams = [
                (None, attn.to_q(hidden_states), attn.norm_q, attn.norm_q),
                (None, attn.to_k(hidden_states), attn.norm_k, attn.norm_k),
                (None, attn.to_v(hidden_states), None, None),
            ]
        packed = []
        for txt, img, n_txt, n_img in streams:
            rot = (cos, sin) if n_img is not None else (None, None)
            packed.append(
                norm_rope_pack(
                    txt,
                    img,
                    heads=heads,
                    weight_txt=None if n_txt is None else n_txt.weight,
                    weight_img=None if n_img is None else n_img.weight,
                    eps=1e-6 if n_img is None else float(n_img.eps),
                    cos=rot[0],
                    sin=rot[1],
                )
            )
        q, k, v = (x.transpose(1, 2) for x in packed)  # [B, H, S, D] views of [B, S, H, D]
        if q.shape[2] != self.bank.total_tokens:
            raise ValueError("Native attention sequence length does not match the plan")
        return self._attend(q, k, v).transpose(1, 2).flatten(2, 3)

    def _attend(self, q, k, v):
        """The attention of the layer's phase on the prepared [B, H, S, D] views."""
        metadata = self.bank.on_device(q.device)["paired_phases"][self.phase]
        return paired_attention(q, k, v, metadata, **self.kernel_options)

    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None, image_rotary_emb=None):
        if attention_mask is not None:
            raise ValueError("External attention masks cannot be combined implicitly with the registered plan")
        out = self.attention(attn, hidden_states, encoder_hidden_states, image_rotary_emb).to(hidden_states.dtype)
        if encoder_hidden_states is None:
            return out
        text, image = out.split_with_sizes(
            [encoder_hidden_states.shape[1], out.shape[1] - encoder_hidden_states.shape[1]], dim=1
        )
        image = attn.to_out[1](attn.to_out[0](image))
        text = attn.to_add_out(text)
        return image, text
