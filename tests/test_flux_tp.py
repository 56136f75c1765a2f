"""Tensor-parallel FLUX.1-architecture step (hilberta_b200/flux_tp.py) on CPU
ranks (gloo, world sizes 2 and 4): the sharded step equals the unsharded one.
Attention runs through a torch processor here (RMSNorm, rotary, dense SDPA) so
that no GPU is needed; the GPU processors see the same per-rank module
attributes (local ``heads``, column-sliced projections)."""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F


class TorchProcessor:
    """FluxAttention's processor steps in plain torch (fp32 reference)."""

    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None, image_rotary_emb=None):
        cos, sin = image_rotary_emb
        h = attn.heads

        def heads(x):
            return x.unflatten(-1, (h, -1))

        def norm(x, m):
            return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + m.eps) * m.weight

        def rope(x):  # x [B, S, H, D]; pairs (2i, 2i+1) rotate
            re, im = x.unflatten(-1, (-1, 2)).unbind(-1)
            rot = torch.stack([-im, re], dim=-1).flatten(-2)
            return x * cos[None, :, None] + rot * sin[None, :, None]

        if encoder_hidden_states is not None:
            q = torch.cat([norm(heads(attn.add_q_proj(encoder_hidden_states)), attn.norm_added_q),
                           norm(heads(attn.to_q(hidden_states)), attn.norm_q)], 1)
            k = torch.cat([norm(heads(attn.add_k_proj(encoder_hidden_states)), attn.norm_added_k),
                           norm(heads(attn.to_k(hidden_states)), attn.norm_k)], 1)
            v = torch.cat([heads(attn.add_v_proj(encoder_hidden_states)), heads(attn.to_v(hidden_states))], 1)
        else:
            q = norm(heads(attn.to_q(hidden_states)), attn.norm_q)
            k = norm(heads(attn.to_k(hidden_states)), attn.norm_k)
            v = heads(attn.to_v(hidden_states))
        q, k = rope(q), rope(k)
        out = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
        out = out.transpose(1, 2).flatten(2, 3)
        if encoder_hidden_states is None:
            return out
        t = encoder_hidden_states.shape[1]
        return attn.to_out[1](attn.to_out[0](out[:, t:])), attn.to_add_out(out[:, :t])


class EagerBlockOps:
    """The blocks' modulation, residual and MLP steps as plain torch ops (CPU)."""

    @staticmethod
    def modulate(x, shift, scale):
        return F.layer_norm(x, x.shape[-1:], eps=1e-6) * (1 + scale[:, None]) + shift[:, None]

    @staticmethod
    def gate_add(x, y, gate):
        return x + gate[:, None] * y

    @classmethod
    def gate_add_modulate(cls, x, y, gate, shift, scale):
        x = cls.gate_add(x, y, gate)
        return x, cls.modulate(x, shift, scale)

    @staticmethod
    def linear_gelu(x, weight, bias):
        return F.gelu(F.linear(x, weight, bias), approximate="tanh")

    @staticmethod
    def joined_linear(a, m, weight_a, weight_m, bias, out=None):
        y = F.linear(torch.cat([a, m], -1), torch.cat([weight_a, weight_m], 1), bias)
        if out is None:
            return y
        out.copy_(y.reshape(out.shape))
        return out


def _model_and_inputs():
    from hilberta_b200.flux_model import FluxTransformer, image_ids

    torch.manual_seed(0)
    model = FluxTransformer(num_double=2, num_single=2, dim=128, heads=4, head_dim=32, text_dim=48, pooled_dim=16,
                            axes=(8, 12, 12), dtype=torch.float32, device="cpu", block_ops=EagerBlockOps())
    for m in model.attention_modules():
        m.set_processor(TorchProcessor())
    g = torch.Generator().manual_seed(1)
    x = dict(hidden_states=torch.randn(2, 64, 64, generator=g), encoder_hidden_states=torch.randn(2, 16, 48, generator=g),
             pooled_projections=torch.randn(2, 16, generator=g), timestep=torch.tensor([0.2, 0.7]),
             img_ids=image_ids(8), txt_ids=torch.zeros(16, 3, dtype=torch.int64), guidance=torch.tensor([3.5, 2.0]))
    return model, x


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, chunks=1, sp=False):
    try:
        from hilberta_b200.flux_tp import shard_flux_model

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
        model, x = _model_and_inputs()
        with torch.no_grad():
            full = model(**x).sample
            n_full = sum(p.numel() for p in model.parameters())
            shard_flux_model(model, chunks=chunks, carveout=None, min_rows=1, sequence_parallel=sp)
            local = model(**x).sample
        n_local = sum(p.numel() for p in model.parameters())
        err = float((local - full).abs().max() / full.abs().max())
        ok = err < 1e-5 and model.transformer_blocks[0].attn.heads == 4 // world and n_local < n_full
        q.put((rank, "ok" if ok else f"mismatch {err}"))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, f"error: {type(e).__name__}: {e}"))
        traceback.print_exc()


@pytest.mark.parametrize("world,chunks,sp", [(2, 1, False), (4, 1, False), (2, 3, False), (2, 1, True), (4, 1, True)])
def test_tensor_parallel_step_matches_unsharded(world, chunks, sp):
    """chunks > 1: row-parallel GEMMs in row chunks with async all-reduces;
    sp: sequence parallelism (token-split streams, all-gather / reduce-scatter;
    batch 2, so the batch-major reorder of both collectives is exercised)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, chunks, sp)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {r: "ok" for r in range(world)}


def test_shard_rejects_uneven_heads():
    from hilberta_b200.flux_tp import _slice

    with pytest.raises(ValueError, match="does not split"):
        _slice(24, 0, 5)
    assert torch.equal(_slice(12, 1, 3), torch.arange(4, 8))
