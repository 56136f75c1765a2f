"""Head-parallel HilbertA attention over the ranks of one node.

Heads are independent and the paired metadata is indexed by query row only
(the reference kernel reads it by row, hilberta/paired_kernel.py:72-73), so the
attention shards by heads with no collective inside it: rank r of P owns heads
[r*H/P, (r+1)*H/P) (24 heads -> 12/6/3 per GPU at P = 2/4/8), with the metadata
replicated.  The one exchange is an all-gather of the 16-bit head outputs where
the FLUX block needs every head (before ``to_out``,
hilberta/flux_adapter.py:328-339):

* ``PeerAllGather`` (the B200 path): the attention kernel itself stores every
  output row into all ranks' full-head outputs over NVLink peer memory, so the
  exchange overlaps the math; a bounded device-side flag barrier ends the call.
* ``all_gather_heads`` / ``head_parallel_attention``: the kernel followed by a
  torch.distributed all-gather (NCCL on GPUs; gloo for host-side tests).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .paired_kernel import _check_inputs, _launch_allgather, paired_attention


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


class PeerAllGather:
    """Paired attention of this rank's heads fused with the all-gather of all
    ranks' heads (``hb_paired_fwd_allgather``).

    Collective: every rank of `group` (one process per GPU, distinct GPUs of one
    node) constructs it with the same arguments and then makes the same sequence
    of calls.  ``heads`` is the total head count; each call takes this rank's
    head slice ``[B, heads/P, N, D]`` and returns the full ``[B, heads, N, D]``
    output (a view of storage in ``layout`` order: "bhnd", or "bnhd" as the
    processor's hidden states before ``flatten(2, 3)``), complete on return of
    the launch on the current stream.  Outputs alternate between two buffers.
    A returned tensor is valid for work that is ordered on the stream before
    this rank's next call: a peer may start writing the same buffer in its call
    after next as soon as this rank's next call has finished, so read or copy
    the output (or queue the work that consumes it) before making the next call.
    After a call that reports ``HB_DEV_PEER_TIMEOUT`` (``device_status``) the
    ranks' flags may disagree: close the instance and build a new one.
    """

    def __init__(self, batch, heads, tokens, head_dim, *, dtype=torch.bfloat16, layout="bhnd", group=None,
                 device=None, timeout_ms=10000):
        world, rank = _world(group)
        if world > _lib.HB_MAX_RANKS:
            raise ValueError(f"at most {_lib.HB_MAX_RANKS} ranks")
        if layout not in ("bhnd", "bnhd"):
            raise ValueError("layout must be bhnd or bnhd")
        self.head0, self.head1 = head_range(heads, rank, world)
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.world, self.rank, self.group, self.device = world, rank, group, dev
        self.shape = (batch, heads, tokens, head_dim)
        self.dtype, self.timeout_ms = dtype, int(timeout_ms)
        ids = [None] * world
        dist.all_gather_object(ids, str(torch.cuda.get_device_properties(dev).uuid), group=group)
        if len(set(ids)) != world:
            raise ValueError("PeerAllGather needs every rank on a distinct GPU")
        store = (batch, heads, tokens, head_dim) if layout == "bhnd" else (batch, tokens, heads, head_dim)
        with torch.inference_mode(False):
            self._bufs = [torch.empty(store, dtype=dtype, device=dev) for _ in range(2)]
            self._flags = torch.zeros(_lib.HB_MAX_RANKS, dtype=torch.int32, device=dev)
        self._views = [b if layout == "bhnd" else b.transpose(1, 2) for b in self._bufs]
        torch.cuda.synchronize(dev)  # flags are zero before any peer can write them
        lib = _lib.lib()
        mine = []
        for t in (*self._bufs, self._flags):
            h = ctypes.create_string_buffer(_lib.HB_IPC_HANDLE_BYTES)
            off = ctypes.c_uint64()
            _lib.check(lib.hb_ipc_export(ctypes.c_void_p(t.data_ptr()), h, ctypes.byref(off)), "hb_ipc_export")
            mine.append((h.raw, off.value))
        everyone = [None] * world
        dist.all_gather_object(everyone, mine, group=group)
        self._opened = {}  # handle bytes -> mapped allocation base (one mapping per peer allocation)
        self._ptrs = []  # rank -> [buf0, buf1, flags] device addresses usable on this GPU
        for r, handles in enumerate(everyone):
            if r == rank:
                self._ptrs.append([t.data_ptr() for t in (*self._bufs, self._flags)])
                continue
            ptrs = []
            for h, off in handles:
                if h not in self._opened:
                    base = ctypes.c_void_p()
                    _lib.check(lib.hb_ipc_open(h, 0, ctypes.byref(base)), "hb_ipc_open")
                    self._opened[h] = base.value
                ptrs.append(self._opened[h] + off)
            self._ptrs.append(ptrs)
        dist.barrier(group=group)  # every rank mapped every peer before the first call
        self.epoch = 0

    def __call__(self, q, k, v, metadata, *, global_strategy="flash", num_warps=4, num_stages=2, scale=None):
        if self._ptrs is None:
            raise RuntimeError("PeerAllGather is closed")
        B, H, N, D = self.shape
        N_, G, scale = _check_inputs(q, k, v, metadata, global_strategy, num_warps, num_stages, scale)
        if q.shape != (B, self.head1 - self.head0, N, D) or q.dtype != self.dtype or q.device != self.device:
            raise ValueError("Q/K/V must be this rank's [B, heads/P, N, D] slice in the gather's dtype and device")
        self.epoch += 1
        slot = self.epoch & 1
        full = self._views[slot]
        elem = full.element_size()
        peers = _lib.PeerOut()
        peers.n_ranks, peers.rank, peers.epoch, peers.timeout_ms = self.world, self.rank, self.epoch, self.timeout_ms
        for r in range(self.world):
            peers.out[r] = self._ptrs[r][slot] + self.head0 * full.stride(1) * elem
            peers.flags[r] = self._ptrs[r][2]
        _launch_allgather(q, k, v, full, metadata, N_, G, scale, peers)
        return full

    def measure_link_gbs(self, reps=3, method="sm"):
        """Collective, between calls only: every rank sends the bytes one call
        sends to each peer (its own head rows) into every peer's buffer, all
        ranks at once, as the fused call's stores load the links.  ``method``
        "sm": one ``hb_peer_scatter`` launch, SM stores to all peers in the fused
        kernel's pattern; "copy_engine": plain copy-engine transfers
        (``hb_peer_copy``, one stream per peer).  Returns this rank's send
        bandwidth in GB/s (bytes sent over device time, best of `reps`).  It
        overwrites the buffers' contents."""
        if self._ptrs is None:
            raise RuntimeError("PeerAllGather is closed")
        if method not in ("sm", "copy_engine"):
            raise ValueError("method must be 'sm' or 'copy_engine'")
        B, H, N, D = self.shape
        nbytes = B * (self.head1 - self.head0) * N * D * self._bufs[0].element_size()
        src = self._ptrs[self.rank][1] + self.rank * nbytes  # this rank's region of its idle second buffer
        lib = _lib.lib()
        main = torch.cuda.current_stream(self.device)
        peers = [r for r in range(self.world) if r != self.rank]
        side = [torch.cuda.Stream(self.device) for _ in peers] if method == "copy_engine" else []
        dsts = (ctypes.c_void_p * len(peers))(*[self._ptrs[r][0] + self.rank * nbytes for r in peers])
        best = float("inf")
        for _ in range(reps):
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(main)
            if method == "sm":
                _lib.check(lib.hb_peer_scatter(ctypes.c_void_p(src), dsts, len(peers), nbytes,
                                               ctypes.c_void_p(main.cuda_stream)), "hb_peer_scatter")
            else:
                for s, d in zip(side, dsts):
                    s.wait_event(e0)
                    _lib.check(lib.hb_peer_copy(ctypes.c_void_p(d), ctypes.c_void_p(src), nbytes,
                                                ctypes.c_void_p(s.cuda_stream)), "hb_peer_copy")
                    main.wait_stream(s)
            e1.record(main)
            torch.cuda.synchronize(self.device)
            best = min(best, e0.elapsed_time(e1))
        dist.barrier(group=self.group)
        return len(peers) * nbytes / (best * 1e-3) / 1e9

    def close(self):
        """Unmap the peers' buffers once every rank is done with every call (collective)."""
        if self._ptrs is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = _lib.lib()
        for base in self._opened.values():
            _lib.check(lib.hb_ipc_close(ctypes.c_void_p(base), 0), "hb_ipc_close")
        self._opened, self._ptrs = {}, None
        dist.barrier(group=self.group)  # no rank frees its buffers while a peer still maps them

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False
