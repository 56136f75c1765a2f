"""Tensor-parallel FLUX.1-architecture step over P ranks (one per GPU).

The model of ``flux_model.FluxLikeTransformer`` is split the Megatron way,
head-aligned so that every rank runs HilbertA attention on its own heads
(``heads / P`` of them) with the replicated plan metadata:

* column-parallel (output rows sliced, no communication): ``to_q``/``to_k``/
  ``to_v`` and ``add_q_proj``/``add_k_proj``/``add_v_proj`` by head, the MLP
  input projections (``ff_*[0]``, ``proj_mlp``) by hidden slice;
* row-parallel (input columns sliced, partial sums all-reduced, bias added by
  rank 0's GEMM):
  ``to_out[0]``, ``to_add_out``, ``ff_*[1]``, and the single-stream ``proj_out``,
  whose input is [attention heads | MLP hidden] so its columns are taken from
  both parts;
* replicated: embedders, adaLN modulation, norms, the output layer.

A double-stream block all-reduces 4 times (attention and MLP outputs of the
image and text streams), a single-stream block once.  The reference has no
multi-GPU step (it rejects diffusers' parallel attention,
hilberta/flux_adapter.py:385); this is the head-parallel split of its
attention (rank r owns heads [r*H/P, (r+1)*H/P)) carried through the block.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F


def _param(t):
    return torch.nn.Parameter(t.detach().contiguous(), requires_grad=False)


class RowParallelLinear(torch.nn.Module):
    """``y = all_reduce(x_shard @ W[:, cols]^T (+ b on rank 0))``: ``x`` holds
    this rank's input columns ``cols`` of the full layer; the bias enters once,
    through rank 0's GEMM."""

    def __init__(self, full: torch.nn.Linear, cols: torch.Tensor, group, rank):
        super().__init__()
        self.weight = _param(full.weight.index_select(1, cols.to(full.weight.device)))
        self.bias = _param(full.bias) if full.bias is not None and rank == 0 else None
        self.group = group

    def forward(self, x):
        y = F.linear(x, self.weight, self.bias)
        dist.all_reduce(y, group=self.group)
        return y


class RowParallelJoined(torch.nn.Module):
    """Row-parallel form of ``flux_model.JoinedLinear``: this rank's attention
    columns ``cols_a`` and MLP columns ``cols_m``, partial sums all-reduced."""

    def __init__(self, full, cols_a, cols_m, group, rank):
        super().__init__()
        w = full.weight
        self.weight_a = _param(w.index_select(1, cols_a.to(w.device)))
        self.weight_m = _param(w.index_select(1, (full.split + cols_m).to(w.device)))
        self.bias = _param(full.bias) if full.bias is not None and rank == 0 else None
        self.group = group

    def forward(self, a, m, ops):
        y = ops.joined_linear(a, m, self.weight_a, self.weight_m, self.bias)
        dist.all_reduce(y, group=self.group)
        return y


def _column(full: torch.nn.Linear, rows: torch.Tensor) -> torch.nn.Linear:
    """A Linear holding output rows ``rows`` of ``full``."""
    w = full.weight.detach()
    lin = torch.nn.Linear(w.shape[1], rows.numel(), bias=full.bias is not None, dtype=w.dtype, device=w.device)
    with torch.no_grad():
        lin.weight.copy_(w.index_select(0, rows.to(w.device)))
        if full.bias is not None:
            lin.bias.copy_(full.bias.detach().index_select(0, rows.to(w.device)))
    return lin.requires_grad_(False)


def _slice(n, rank, world):
    if n % world:
        raise ValueError(f"{n} does not split over {world} ranks")
    s = n // world
    return torch.arange(rank * s, (rank + 1) * s)


def shard_flux_model(model, group=None):
    """Split ``model`` (a ``FluxLikeTransformer`` with identical weights on
    every rank) in place for this rank of ``group``; returns it."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    first = model.double_blocks[0].attn if len(model.double_blocks) else model.single_blocks[0].attn
    heads = first.heads
    head_dim = first.to_q.weight.shape[0] // heads
    if heads % world:
        raise ValueError("heads must split evenly over the ranks")
    head_cols = _slice(heads * head_dim, rank, world)  # this rank's heads, contiguous
    for b in model.double_blocks:
        a = b.attn
        for name in ("to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj"):
            setattr(a, name, _column(getattr(a, name), head_cols))
        a.to_out[0] = RowParallelLinear(a.to_out[0], head_cols, group, rank)
        a.to_add_out = RowParallelLinear(a.to_add_out, head_cols, group, rank)
        a.heads = heads // world
        for ff in (b.ff_img, b.ff_txt):
            hid = _slice(ff[0].weight.shape[0], rank, world)
            ff[0] = _column(ff[0], hid)
            ff[1] = RowParallelLinear(ff[1], hid, group, rank)
    for b in model.single_blocks:
        a = b.attn
        for name in ("to_q", "to_k", "to_v"):
            setattr(a, name, _column(getattr(a, name), head_cols))
        a.heads = heads // world
        hid = _slice(b.proj_mlp.weight.shape[0], rank, world)
        b.proj_mlp = _column(b.proj_mlp, hid)
        b.proj_out = RowParallelJoined(b.proj_out, head_cols, hid, group, rank)
    model.tp_world, model.tp_rank = world, rank
    if torch.cuda.is_available() and first.to_q.weight.is_cuda:
        torch.cuda.empty_cache()
    return model


__all__ = ["RowParallelLinear", "RowParallelJoined", "shard_flux_model"]
