"""A FLUX.1-architecture transformer with random weights, for timing one
denoising step with HilbertA attention in every joint-attention call.

The architecture follows FLUX.1's published design (the model the reference
adapts, hilberta/flux_adapter.py): 19 double-stream blocks (separate weights
for text and image tokens, one joint attention), 38 single-stream blocks
(attention and MLP in parallel on the joined sequence), hidden 3072, 24 heads of
128, per-head RMSNorm on Q/K, 3-axis rotary embedding (16/56/56 dimensions over
(index, row, column) positions), adaLN-Zero modulation from the timestep
embedding, tanh-GELU MLPs with ratio 4.  Weights are random (no checkpoint is
available); the step's cost and data flow are the model's.

``FluxTransformer`` carries the module names and the forward signature of
diffusers' ``FluxTransformer2DModel`` (``transformer_blocks``,
``single_transformer_blocks``, ``attn.set_processor``; ``forward(hidden_states,
encoder_hidden_states, pooled_projections, timestep, img_ids, txt_ids, guidance,
...)``, rotary tables from the position ids), so the reference's adapter entry,
``flux_adapter.persistent_flux_attention``, applies to it unchanged.  Outside
that context every joint attention is dense (``DenseProcessor``: the fused Q/K/V
preparation and torch SDPA); inside it, ``HilbertAProcessor`` on the layer's
phase with the image tokens permuted into the plan's order once per call.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .block_ops import NativeBlockOps
from .prep import norm_rope_pack


class RMSNormWeight(torch.nn.Module):
    """The per-head RMSNorm parameters the processors read (``weight``, ``eps``)."""

    def __init__(self, d, dtype, device):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(d, dtype=dtype, device=device), requires_grad=False)
        self.eps = 1e-6


def _linear(i, o, dtype, device, std=0.02):
    lin = torch.nn.Linear(i, o, dtype=dtype, device=device)
    with torch.no_grad():
        lin.weight.normal_(0.0, std)
        lin.bias.zero_()
    return lin.requires_grad_(False)


class JointAttention(torch.nn.Module):
    """Attribute layout of a FLUX attention module; ``processor`` does the work."""

    def __init__(self, dim, heads, head_dim, double, dtype, device):
        super().__init__()
        inner = heads * head_dim
        self.heads = heads
        self.to_q, self.to_k, self.to_v = (_linear(dim, inner, dtype, device) for _ in range(3))
        self.norm_q, self.norm_k = RMSNormWeight(head_dim, dtype, device), RMSNormWeight(head_dim, dtype, device)
        self.added_kv_proj_dim = dim if double else None
        if double:
            self.add_q_proj, self.add_k_proj, self.add_v_proj = (_linear(dim, inner, dtype, device) for _ in range(3))
            self.norm_added_q = RMSNormWeight(head_dim, dtype, device)
            self.norm_added_k = RMSNormWeight(head_dim, dtype, device)
            self.to_out = torch.nn.ModuleList([_linear(inner, dim, dtype, device), torch.nn.Dropout(0.0)])
            self.to_add_out = _linear(inner, dim, dtype, device)
        self.processor = None

    def set_processor(self, processor):
        self.processor = processor

    def forward(self, hidden_states, encoder_hidden_states=None, image_rotary_emb=None):
        return self.processor(self, hidden_states, encoder_hidden_states, image_rotary_emb=image_rotary_emb)


class DenseProcessor:
    """The same steps as ``HilbertAProcessor`` with dense attention over all
    tokens, or over the plan's dense mask of the layer's phase when ``bank`` is
    given (the correctness reference of the sparse step)."""

    def __init__(self, bank=None, layer=0):
        self.bank, self.phase = bank, int(layer) % 4

    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None, image_rotary_emb=None):
        if attention_mask is not None:
            raise ValueError("External attention masks are not supported")
        cos, sin = image_rotary_emb
        h = attn.heads
        if encoder_hidden_states is not None:
            q = norm_rope_pack(attn.add_q_proj(encoder_hidden_states), attn.to_q(hidden_states), heads=h,
                               weight_txt=attn.norm_added_q.weight, weight_img=attn.norm_q.weight, cos=cos, sin=sin)
            k = norm_rope_pack(attn.add_k_proj(encoder_hidden_states), attn.to_k(hidden_states), heads=h,
                               weight_txt=attn.norm_added_k.weight, weight_img=attn.norm_k.weight, cos=cos, sin=sin)
            v = norm_rope_pack(attn.add_v_proj(encoder_hidden_states), attn.to_v(hidden_states), heads=h)
        else:
            q = norm_rope_pack(None, attn.to_q(hidden_states), heads=h, weight_txt=attn.norm_q.weight,
                               weight_img=attn.norm_q.weight, cos=cos, sin=sin)
            k = norm_rope_pack(None, attn.to_k(hidden_states), heads=h, weight_txt=attn.norm_k.weight,
                               weight_img=attn.norm_k.weight, cos=cos, sin=sin)
            v = norm_rope_pack(None, attn.to_v(hidden_states), heads=h)
        mask = None if self.bank is None else self.bank.dense_mask(self.phase, q.device)
        out = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), attn_mask=mask)
        out = out.transpose(1, 2).flatten(2, 3).to(hidden_states.dtype)
        if encoder_hidden_states is None:
            return out
        text, image = out.split_with_sizes([encoder_hidden_states.shape[1], out.shape[1] - encoder_hidden_states.shape[1]], 1)
        return attn.to_out[1](attn.to_out[0](image)), attn.to_add_out(text)


def _same(x):
    return x


def _modulate(x, shift, scale):
    """adaLN of the output layer (once per step, eager)."""
    return F.layer_norm(x, x.shape[-1:], eps=1e-6) * (1 + scale[:, None]) + shift[:, None]


class JoinedLinear(torch.nn.Module):
    """FLUX's single-stream ``proj_out`` over [attention | MLP hidden]: one
    weight ``[dim, inner + hidden]``, applied as ``ops.joined_linear`` so the
    concatenated input is never materialised."""

    def __init__(self, inner, hidden, dim, dtype, device):
        super().__init__()
        full = _linear(inner + hidden, dim, dtype, device)
        self.weight, self.bias, self.split = full.weight, full.bias, inner

    def forward(self, a, m, ops):
        return ops.joined_linear(a, m, self.weight[:, : self.split], self.weight[:, self.split :], self.bias)


class DoubleStreamBlock(torch.nn.Module):
    def __init__(self, dim, heads, head_dim, dtype, device):
        super().__init__()
        self.mod_img = _linear(dim, 6 * dim, dtype, device)
        self.mod_txt = _linear(dim, 6 * dim, dtype, device)
        self.attn = JointAttention(dim, heads, head_dim, True, dtype, device)
        self.ff_img = torch.nn.ModuleList([_linear(dim, 4 * dim, dtype, device), _linear(4 * dim, dim, dtype, device)])
        self.ff_txt = torch.nn.ModuleList([_linear(dim, 4 * dim, dtype, device), _linear(4 * dim, dim, dtype, device)])

    def forward(self, img, txt, temb, rot, ops, gather=_same):
        """``gather``: token all-gather of the image stream before its
        projections (sequence parallelism; identity otherwise)."""
        mi = self.mod_img(F.silu(temb)).chunk(6, dim=-1)
        mt = self.mod_txt(F.silu(temb)).chunk(6, dim=-1)
        a_img, a_txt = self.attn(gather(ops.modulate(img, mi[0], mi[1])), ops.modulate(txt, mt[0], mt[1]), rot)
        img, h_img = ops.gate_add_modulate(img, a_img, mi[2], mi[3], mi[4])
        txt, h_txt = ops.gate_add_modulate(txt, a_txt, mt[2], mt[3], mt[4])
        f_img = self.ff_img[1](ops.linear_gelu(gather(h_img), self.ff_img[0].weight, self.ff_img[0].bias))
        f_txt = self.ff_txt[1](ops.linear_gelu(h_txt, self.ff_txt[0].weight, self.ff_txt[0].bias))
        return ops.gate_add(img, f_img, mi[5]), ops.gate_add(txt, f_txt, mt[5])


class SingleStreamBlock(torch.nn.Module):
    def __init__(self, dim, heads, head_dim, dtype, device):
        super().__init__()
        self.mod = _linear(dim, 3 * dim, dtype, device)
        self.attn = JointAttention(dim, heads, head_dim, False, dtype, device)
        self.proj_mlp = _linear(dim, 4 * dim, dtype, device)
        self.proj_out = JoinedLinear(heads * head_dim, 4 * dim, dim, dtype, device)

    def forward(self, x, temb, rot, ops, gather=_same):
        shift, scale, gate = self.mod(F.silu(temb)).chunk(3, dim=-1)
        h = gather(ops.modulate(x, shift, scale))
        mlp = ops.linear_gelu(h, self.proj_mlp.weight, self.proj_mlp.bias)
        a = self.attn(h, None, rot)
        return ops.gate_add(x, self.proj_out(a, mlp, ops), gate)


def timestep_features(t, dim=256, max_period=10000.0):
    """Sinusoidal features [B, dim] of scalar times ``t`` [B] (scaled by 1000,
    cosines first, as FLUX's time embedding takes them)."""
    half = dim // 2
    freqs = torch.exp(-torch.log(torch.tensor(max_period, dtype=torch.float32, device=t.device))
                      * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    ang = (t.float() * 1000.0)[:, None] * freqs[None]
    return torch.cat([torch.cos(ang), torch.sin(ang)], dim=1)


class ConditioningEmbedder(torch.nn.Module):
    """temb = MLP(time features) + MLP(guidance features) + MLP(pooled text)."""

    def __init__(self, dim, pooled_dim, dtype, device):
        super().__init__()
        mlp = lambda i: torch.nn.ModuleList([_linear(i, dim, dtype, device), _linear(dim, dim, dtype, device)])
        self.time, self.guidance, self.text = mlp(256), mlp(256), mlp(pooled_dim)

    def forward(self, timestep, guidance, pooled):
        run = lambda m, x: m[1](F.silu(m[0](x)))
        dt = pooled.dtype
        temb = run(self.time, timestep_features(timestep).to(dt)) + run(self.text, pooled)
        if guidance is not None:
            temb = temb + run(self.guidance, timestep_features(guidance).to(dt))
        return temb


def rotary_3axis(ids, axes=(16, 56, 56), theta=10000.0):
    """cos/sin [N, sum(axes)] fp32 of 3-axis positions ``ids`` [N, 3]: per axis,
    frequencies theta^(-2i/d) on that coordinate, each repeated for its pair."""
    cos, sin = [], []
    for a, d in enumerate(axes):
        freqs = 1.0 / theta ** (torch.arange(0, d, 2, dtype=torch.float64, device=ids.device) / d)
        ang = ids[:, a].to(torch.float64)[:, None] * freqs[None]
        cos.append(torch.cos(ang).repeat_interleave(2, dim=1))
        sin.append(torch.sin(ang).repeat_interleave(2, dim=1))
    return torch.cat(cos, 1).float().contiguous(), torch.cat(sin, 1).float().contiguous()


class FluxOutput:
    """Prediction of one call (``.sample``), like diffusers'
    ``Transformer2DModelOutput``."""

    def __init__(self, sample):
        self.sample = sample


class FluxTransformer(torch.nn.Module):
    """FLUX.1 transformer with random weights (defaults: FLUX.1-dev's sizes,
    11.90 B parameters) and diffusers' ``FluxTransformer2DModel`` interface.

    ``forward(hidden_states [B, n, 64], encoder_hidden_states [B, T, text_dim],
    pooled_projections [B, pooled_dim], timestep [B], img_ids [n, 3],
    txt_ids [T, 3], guidance [B] or None, joint_attention_kwargs=None,
    controlnet_block_samples=None, controlnet_single_block_samples=None,
    return_dict=True)`` -> ``FluxOutput`` (or a 1-tuple).  Tokens are processed in
    the order given; the rotary tables follow the ids.  ``block_ops`` (default
    ``NativeBlockOps``: the library's adaLN kernels and cuBLASLt epilogues) runs
    the blocks' modulation, residual and MLP steps."""

    def __init__(self, num_double=19, num_single=38, dim=3072, heads=24, head_dim=128, in_channels=64, text_dim=4096,
                 pooled_dim=768, axes=(16, 56, 56), dtype=torch.bfloat16, device="cuda", block_ops=None):
        super().__init__()
        if sum(axes) != head_dim:
            raise ValueError("rotary axes must add up to head_dim")
        self.ops = NativeBlockOps() if block_ops is None else block_ops
        self.axes = tuple(int(a) for a in axes)
        self.x_embedder = _linear(in_channels, dim, dtype, device)
        self.context_embedder = _linear(text_dim, dim, dtype, device)
        self.time_text_embed = ConditioningEmbedder(dim, pooled_dim, dtype, device)
        self.transformer_blocks = torch.nn.ModuleList(
            DoubleStreamBlock(dim, heads, head_dim, dtype, device) for _ in range(num_double))
        self.single_transformer_blocks = torch.nn.ModuleList(
            SingleStreamBlock(dim, heads, head_dim, dtype, device) for _ in range(num_single))
        self.norm_out = _linear(dim, 2 * dim, dtype, device)
        self.proj_out = _linear(dim, in_channels, dtype, device)
        self.gradient_checkpointing = False
        self.sequence_parallel = None  # flux_tp.TokenShards when the blocks' streams are sharded by tokens
        self.eval()
        for m in self.attention_modules():
            m.set_processor(DenseProcessor())

    def attention_modules(self):
        return [b.attn for b in self.transformer_blocks] + [b.attn for b in self.single_transformer_blocks]

    def forward(self, hidden_states, encoder_hidden_states=None, pooled_projections=None, timestep=None, img_ids=None,
                txt_ids=None, guidance=None, joint_attention_kwargs=None, controlnet_block_samples=None,
                controlnet_single_block_samples=None, return_dict=True):
        if controlnet_block_samples is not None or controlnet_single_block_samples is not None:
            raise ValueError("ControlNet residuals are not supported")
        if txt_ids.ndim == 3:
            txt_ids = txt_ids[0]
        if img_ids.ndim == 3:
            img_ids = img_ids[0]
        if img_ids.shape[0] != hidden_states.shape[1] or txt_ids.shape[0] != encoder_hidden_states.shape[1]:
            raise ValueError("position ids do not match the token counts")
        rot = rotary_3axis(torch.cat([txt_ids, img_ids], 0), self.axes)
        temb = self.time_text_embed(timestep, guidance, pooled_projections)
        img = self.x_embedder(hidden_states)
        txt = self.context_embedder(encoder_hidden_states)
        seq = self.sequence_parallel
        gather = _same if seq is None else seq.gather
        if seq is not None:  # this rank's token range of the image stream
            img = seq.scatter(img)
        for b in self.transformer_blocks:
            img, txt = b(img, txt, temb, rot, self.ops, gather)
        x = torch.cat([txt, gather(img)], dim=1)
        if seq is not None:  # this rank's token range of the joined stream
            x = seq.scatter(x)
        for b in self.single_transformer_blocks:
            x = b(x, temb, rot, self.ops, gather)
        img = gather(x)[:, txt.shape[1]:]
        shift, scale = self.norm_out(F.silu(temb)).chunk(2, dim=-1)
        out = self.proj_out(_modulate(img, shift, scale))
        return FluxOutput(out) if return_dict else (out,)


def image_ids(grid, device=None):
    """Position ids [grid*grid, 3] of a raster image: (0, row, column)."""
    r = torch.arange(grid * grid, device=device)
    return torch.stack([torch.zeros_like(r), r // grid, r % grid], dim=1)


def parameter_count(model) -> int:
    return sum(p.numel() for p in model.parameters())


def attention_flops_per_step(bank, heads=24, head_dim=128, layers=57):
    """Active-block FLOPs of the step's attention calls (phase of layer i = i % 4)."""
    total = 0
    for layer in range(layers):
        p = bank.phases[layer % 4]
        active = (bank.global_tokens // 64) * (bank.total_tokens // 64) + int(p[1].sum())
        total += heads * 4 * 64 * 64 * head_dim * active
    return total


__all__ = ["FluxTransformer", "FluxOutput", "DenseProcessor", "JoinedLinear", "ConditioningEmbedder", "timestep_features",
           "image_ids", "step_inputs", "rotary_3axis", "parameter_count", "attention_flops_per_step"]


def step_inputs(grid, text_tokens, device, batch=1, seed=6, text_dim=4096, pooled_dim=768, dtype=torch.bfloat16):
    """Seeded synthetic inputs of one denoising call, as keyword arguments."""
    g = torch.Generator().manual_seed(seed)
    return dict(
        hidden_states=torch.randn(batch, grid * grid, 64, generator=g).to(dtype).to(device),
        encoder_hidden_states=torch.randn(batch, text_tokens, text_dim, generator=g).to(dtype).to(device),
        pooled_projections=torch.randn(batch, pooled_dim, generator=g).to(dtype).to(device),
        timestep=torch.full((batch,), 0.75, device=device),
        img_ids=image_ids(grid, device),
        txt_ids=torch.zeros(text_tokens, 3, dtype=torch.int64, device=device),
        guidance=torch.full((batch,), 3.5, device=device),
    )
