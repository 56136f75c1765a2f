"""Head-parallel HilbertA attention over the ranks of one node.

Heads are independent and the paired metadata is indexed by query row only
(the reference kernel reads it by row, hilberta/paired_kernel.py:72-73), so the
attention shards by heads with no collective inside it: rank r of P owns heads
[r*H/P, (r+1)*H/P) (24 heads -> 12/6/3 per GPU at P = 2/4/8), with the metadata
replicated.  The one exchange is an all-gather of the 16-bit head outputs where
the FLUX block needs every head (before ``to_out``,
hilberta/flux_adapter.py:328-339), issued through torch.distributed (NCCL over
NVLink on GPUs; gloo works for host-side tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .paired_kernel import paired_attention


def head_range(num_heads: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of the heads owned by `rank`; heads must divide evenly."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if num_heads % world:
        raise ValueError(f"{num_heads} heads do not split evenly over {world} ranks")
    per = num_heads // world
    return rank * per, (rank + 1) * per


def local_heads(x: torch.Tensor, rank: int, world: int, dim: int = 1) -> torch.Tensor:
    """View of the heads `rank` owns ([B, H, N, D] -> [B, H/P, N, D])."""
    start, stop = head_range(x.shape[dim], rank, world)
    return x.narrow(dim, start, stop - start)


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def all_gather_heads(local_out: torch.Tensor, *, group=None, layout: str = "bhnd") -> torch.Tensor:
    """Gather every rank's head slice [B, h, N, D] into all heads.

    layout "bhnd" returns [B, P*h, N, D]; "bnhd" returns [B, N, P*h, D] (the
    processor's hidden-state order before ``flatten(2, 3)``).  Ranks must pass
    equal shapes; heads come back in rank order.
    """
    world, _ = _world(group)
    B, h, N, D = local_out.shape
    if layout == "bnhd":
        send = local_out.transpose(1, 2).contiguous()  # [B, N, h, D]
    elif layout == "bhnd":
        send = local_out.contiguous()
    else:
        raise ValueError("layout must be bhnd or bnhd")
    if world == 1:
        return send.view(B, N, h, D) if layout == "bnhd" else send
    buf = torch.empty((world, *send.shape), dtype=send.dtype, device=send.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(buf.view(-1), send.view(-1), group=group)
    else:
        dist.all_gather(list(buf.unbind(0)), send, group=group)
    if layout == "bnhd":  # [P, B, N, h, D] -> [B, N, P*h, D]
        return buf.permute(1, 2, 0, 3, 4).reshape(B, N, world * h, D)
    return buf.permute(1, 0, 2, 3, 4).reshape(B, world * h, N, D)  # [P, B, h, N, D] -> [B, P*h, N, D]


def head_parallel_attention(q, k, v, metadata, *, group=None, gather=True, layout="bhnd", **kernel_options):
    """Paired attention of this rank's heads (q/k/v are the local head slices),
    optionally followed by the all-gather of every rank's output."""
    out = paired_attention(q, k, v, metadata, **kernel_options)
    if not gather:
        return out
    return all_gather_heads(out, group=group, layout=layout)
