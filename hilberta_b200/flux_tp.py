"""Tensor-parallel FLUX.1-architecture step over P ranks (one per GPU).

The model of ``flux_model.FluxTransformer`` is split the Megatron way,
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
image and text streams), a single-stream block once.

With ``sequence_parallel=True`` the image stream (double blocks) and the joined
stream (single blocks) stay split by tokens between the layers: each rank keeps
its contiguous token range, runs the adaLN modulation and gated residuals on it
alone, all-gathers the modulated tokens before the column-parallel projections,
and the row-parallel projections of those streams reduce-scatter (the same
bytes as an all-reduce) instead of all-reducing.  The 512-token text stream of
the double blocks stays replicated.  The reference has no
multi-GPU step (it rejects diffusers' parallel attention,
hilberta/flux_adapter.py:385); this is the head-parallel split of its
attention (rank r owns heads [r*H/P, (r+1)*H/P)) carried through the block.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def _param(t):
    return torch.nn.Parameter(t.detach().contiguous(), requires_grad=False)


class TokenShards:
    """Token split of ``[B, S, C]`` streams over ``group``: rank r holds tokens
    [r*S/P, (r+1)*S/P)."""

    def __init__(self, group, world, rank):
        self.group, self.world, self.rank = group, world, rank

    def scatter(self, x):
        S = x.shape[1]
        if S % self.world:
            raise ValueError(f"{S} tokens do not split over {self.world} ranks")
        s = S // self.world
        return x[:, self.rank * s:(self.rank + 1) * s].contiguous()

    def gather(self, x):
        B, s, C = x.shape
        out = torch.empty(self.world * B, s, C, dtype=x.dtype, device=x.device)  # rank-major
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        if B == 1:
            return out.view(1, self.world * s, C)
        return out.view(self.world, B, s, C).transpose(0, 1).reshape(B, self.world * s, C)

    def reduce_scatter(self, y):
        """Sum of ``y`` [B, S, C] over the ranks, this rank's token range."""
        B, S, C = y.shape
        if S % self.world:
            raise ValueError(f"{S} tokens do not split over {self.world} ranks")
        s = S // self.world
        if B == 1:
            src = y.reshape(self.world, s, C)
        else:
            src = y.view(B, self.world, s, C).transpose(0, 1).reshape(self.world * B, s, C)
        out = torch.empty(B, s, C, dtype=y.dtype, device=y.device)
        dist.reduce_scatter_tensor(out, src, group=self.group)
        return out


class _Overlap:
    """Row-chunked GEMM + all-reduce: chunk i's all-reduce (async, on NCCL's
    stream) runs while chunk i+1's GEMM computes.  cuBLAS GEMMs of this size
    occupy every SM, so while the chunks are enqueued the matmuls are told to
    leave ``carveout`` SMs free for the collective (torch's SM carve-out for
    cuBLASLt); the previous setting is restored afterwards."""

    def __init__(self, chunks, carveout, min_rows=2048):
        self.chunks, self.carveout, self.min_rows = int(chunks), carveout, int(min_rows)

    def __call__(self, y, gemm, group):
        """``gemm(s, e)`` writes rows [s, e) of ``y`` ([M, N]); returns ``y``
        all-reduced over ``group``."""
        M = y.shape[0]
        if self.chunks <= 1 or M < self.min_rows:
            gemm(0, M)
            dist.all_reduce(y, group=group)
            return y
        step = -(-M // self.chunks)
        step = -(-step // 128) * 128  # GEMM-friendly chunk rows
        prev = torch._C._get_sm_carveout_experimental()
        use = self.carveout is not None and y.is_cuda
        if use:
            torch._C._set_sm_carveout_experimental(int(self.carveout))
        works = []
        try:
            for s in range(0, M, step):
                e = min(M, s + step)
                gemm(s, e)
                works.append(dist.all_reduce(y[s:e], group=group, async_op=True))
        finally:
            if use:
                torch._C._set_sm_carveout_experimental(prev)
        for w in works:
            w.wait()
        return y


class RowParallelLinear(torch.nn.Module):
    """``y = all_reduce(x_shard @ W[:, cols]^T (+ b on rank 0))``: ``x`` holds
    this rank's input columns ``cols`` of the full layer; the bias enters once,
    through rank 0's GEMM."""

    def __init__(self, full: torch.nn.Linear, cols: torch.Tensor, group, rank, overlap=None, shards=None):
        super().__init__()
        self.weight = _param(full.weight.index_select(1, cols.to(full.weight.device)))
        self.bias = _param(full.bias) if full.bias is not None and rank == 0 else None
        self.group = group
        self.overlap = overlap or _Overlap(1, None)
        self.shards = shards  # TokenShards: reduce-scatter over tokens instead of all-reduce

    def forward(self, x):
        x2 = x.reshape(-1, x.shape[-1])
        y = torch.empty(x2.shape[0], self.weight.shape[0], dtype=x.dtype, device=x.device)
        wt = self.weight.t()

        def gemm(s, e):
            if self.bias is None:
                torch.mm(x2[s:e], wt, out=y[s:e])
            else:
                torch.addmm(self.bias, x2[s:e], wt, out=y[s:e])

        if self.shards is not None:
            gemm(0, y.shape[0])
            return self.shards.reduce_scatter(y.view(*x.shape[:-1], -1))
        return self.overlap(y, gemm, self.group).view(*x.shape[:-1], -1)


class RowParallelJoined(torch.nn.Module):
    """Row-parallel form of ``flux_model.JoinedLinear``: this rank's attention
    columns ``cols_a`` and MLP columns ``cols_m``, partial sums all-reduced."""

    def __init__(self, full, cols_a, cols_m, group, rank, overlap=None, shards=None):
        super().__init__()
        w = full.weight
        self.weight_a = _param(w.index_select(1, cols_a.to(w.device)))
        self.weight_m = _param(w.index_select(1, (full.split + cols_m).to(w.device)))
        self.bias = _param(full.bias) if full.bias is not None and rank == 0 else None
        self.group = group
        self.overlap = overlap or _Overlap(1, None)
        self.shards = shards

    def forward(self, a, m, ops):
        a2, m2 = a.reshape(-1, a.shape[-1]), m.reshape(-1, m.shape[-1])
        y = torch.empty(a2.shape[0], self.weight_a.shape[0], dtype=a.dtype, device=a.device)

        def gemm(s, e):
            ops.joined_linear(a2[s:e], m2[s:e], self.weight_a, self.weight_m, self.bias, out=y[s:e])

        if self.shards is not None:
            gemm(0, y.shape[0])
            return self.shards.reduce_scatter(y.view(*a.shape[:-1], -1))
        return self.overlap(y, gemm, self.group).view(*a.shape[:-1], -1)


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


def shard_flux_model(model, group=None, *, chunks=1, carveout=None, min_rows=2048, sequence_parallel=False):
    """Split ``model`` (a ``FluxTransformer`` with identical weights on
    every rank) in place for this rank of ``group``; returns it.  Row-parallel
    layers over at least ``min_rows`` rows run as ``chunks`` row chunks whose
    all-reduces overlap the next chunk's GEMM, with ``carveout`` SMs kept free
    of the GEMMs meanwhile (``chunks=1``: one GEMM, then one all-reduce).
    ``sequence_parallel``: the image and joined streams split by tokens (see the
    module docstring)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    ov = _Overlap(chunks, carveout, min_rows)
    sh = TokenShards(group, world, rank) if sequence_parallel else None
    first = (model.transformer_blocks or model.single_transformer_blocks)[0].attn
    heads = first.heads
    head_dim = first.to_q.weight.shape[0] // heads
    if heads % world:
        raise ValueError("heads must split evenly over the ranks")
    head_cols = _slice(heads * head_dim, rank, world)  # this rank's heads, contiguous
    for b in model.transformer_blocks:
        a = b.attn
        for name in ("to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj"):
            setattr(a, name, _column(getattr(a, name), head_cols))
        a.to_out[0] = RowParallelLinear(a.to_out[0], head_cols, group, rank, ov, shards=sh)
        a.to_add_out = RowParallelLinear(a.to_add_out, head_cols, group, rank, ov)
        a.heads = heads // world
        for ff, stream_shards in ((b.ff_img, sh), (b.ff_txt, None)):
            hid = _slice(ff[0].weight.shape[0], rank, world)
            ff[0] = _column(ff[0], hid)
            ff[1] = RowParallelLinear(ff[1], hid, group, rank, ov, shards=stream_shards)
    for b in model.single_transformer_blocks:
        a = b.attn
        for name in ("to_q", "to_k", "to_v"):
            setattr(a, name, _column(getattr(a, name), head_cols))
        a.heads = heads // world
        hid = _slice(b.proj_mlp.weight.shape[0], rank, world)
        b.proj_mlp = _column(b.proj_mlp, hid)
        b.proj_out = RowParallelJoined(b.proj_out, head_cols, hid, group, rank, ov, shards=sh)
    model.tp_world, model.tp_rank = world, rank
    model.sequence_parallel = sh
    if torch.cuda.is_available() and first.to_q.weight.is_cuda:
        torch.cuda.empty_cache()
    return model


__all__ = ["RowParallelLinear", "RowParallelJoined", "TokenShards", "shard_flux_model"]
