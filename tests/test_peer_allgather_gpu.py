"""Attention fused with the all-gather of head outputs (hb_paired_fwd_allgather,
hilberta_b200.head_parallel.PeerAllGather).

One GPU: the C ABI driven with two "ranks" whose outputs and flag words both
live on this device — every row must land in both outputs, the flags must carry
the epoch, and a peer flag that nobody sets must end the wait with
HB_DEV_PEER_TIMEOUT (bounded; the context stays usable).  Two GPUs (skipped
with fewer): two processes, each computing half of the heads, must both end
with the full-head output bit-identical to the per-slice kernel results.
"""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch

from oracle import attention_oracle as ao

pytestmark = pytest.mark.gpu


def _setup(heads=4, grid=32, seed=11, phase=1):
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(4, 1, False, grid_size=grid)
    N, G = plan.total_tokens, plan.global_tokens
    p = plan.phases[phase]
    meta = hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=G).to("cuda")
    q, k, v = (x.cuda() for x in ao.seeded_qkv(1, heads, N, 128, seed=seed))
    return meta, q, k, v


def _loopback(q, k, v, meta, outs, flags, epoch, timeout_ms):
    from hilberta_b200 import _lib
    from hilberta_b200.paired_kernel import _launch_allgather

    peers = _lib.PeerOut()
    peers.n_ranks, peers.rank, peers.epoch, peers.timeout_ms = 2, 0, epoch, timeout_ms
    for i in range(2):
        peers.out[i] = outs[i].data_ptr()
        peers.flags[i] = flags[i].data_ptr()
    with torch.inference_mode():
        _launch_allgather(q, k, v, outs[0], meta, meta.tokens, meta.global_tokens, 128**-0.5, peers)
    torch.cuda.synchronize()


def test_loopback_writes_every_destination_and_flags():
    import hilberta_b200 as hb
    from hilberta_b200 import _lib

    meta, q, k, v = _setup()
    with torch.inference_mode():
        ref = hb.paired_attention(q, k, v, meta)
    outs = [torch.full_like(q, float("nan")) for _ in range(2)]
    flags = [torch.zeros(8, dtype=torch.int32, device="cuda") for _ in range(2)]
    flags[0][1] = 1  # "rank 1" already finished epoch 1
    _loopback(q, k, v, meta, outs, flags, 1, 2000)
    assert hb.device_status() == 0
    assert torch.equal(outs[0], ref) and torch.equal(outs[1], ref)
    assert flags[0][0].item() == 1 and flags[1][0].item() == 1  # this rank's word in both arrays
    # next epoch, BNHD outputs: a later epoch already published by the peer is accepted too
    outs = [torch.empty(1, q.shape[2], 4, 128, dtype=q.dtype, device="cuda").transpose(1, 2) for _ in range(2)]
    flags[0][1] = 3
    _loopback(q, k, v, meta, outs, flags, 2, 2000)
    assert hb.device_status() == 0
    assert torch.equal(outs[0], ref) and torch.equal(outs[1], ref)
    assert flags[1][0].item() == 2
    assert _lib.HB_DEV_PEER_TIMEOUT == 8


def test_loopback_more_items_than_ctas_matches_oracle():
    """24 heads at grid 64 give more work items than CTAs: items finished mid-launch
    go through warp 3's copy ring, each CTA's last item through the softmax warps'
    own copy; both destinations must equal the local kernel bit for bit, and
    sampled rows the fp32 oracle."""
    import hilberta_b200 as hb

    meta, q, k, v = _setup(heads=24, grid=64, seed=5, phase=2)
    with torch.inference_mode():
        ref = hb.paired_attention(q, k, v, meta)
    outs = [torch.full_like(q, float("nan")) for _ in range(2)]
    flags = [torch.zeros(8, dtype=torch.int32, device="cuda") for _ in range(2)]
    flags[0][1] = 1
    _loopback(q, k, v, meta, outs, flags, 1, 2000)
    assert hb.device_status() == 0
    assert torch.equal(outs[0], ref) and torch.equal(outs[1], ref)
    plan = hb.bridge_k_plan(4, 1, False, grid_size=64)
    p = plan.phases[2]
    N, G = plan.total_tokens, plan.global_tokens
    rows = torch.tensor([0, G - 1, G, G + 63, G + 64, N // 2, N - 1])
    mask = ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G)
    want = ao.masked_attention_fp32(q.cpu(), k.cpu(), v.cpu(), mask, rows=rows)
    err = (outs[1].cpu()[:, :, rows].float() - want).abs()
    assert float(err.max()) <= 2e-2 and float(err.mean()) <= 2e-3


def test_peer_scatter_copies_to_every_destination():
    """hb_peer_scatter (the link measurement's SM-store copy) on local buffers:
    every destination equals the source, bytes outside the range untouched."""
    import ctypes

    from hilberta_b200 import _lib

    g = torch.Generator(device="cuda").manual_seed(3)
    src = torch.randint(-(2**31), 2**31 - 1, (3 << 18,), generator=g, dtype=torch.int32, device="cuda")
    dst = [torch.zeros(src.numel() + 64, dtype=torch.int32, device="cuda") for _ in range(3)]
    ptrs = (ctypes.c_void_p * 3)(*[d.data_ptr() for d in dst])
    rc = _lib.lib().hb_peer_scatter(ctypes.c_void_p(src.data_ptr()), ptrs, 3, src.numel() * 4,
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.HB_OK
    torch.cuda.synchronize()
    for d in dst:
        assert torch.equal(d[: src.numel()], src) and not d[src.numel():].any()


def test_missing_peer_times_out_and_context_survives():
    import hilberta_b200 as hb
    from hilberta_b200 import _lib

    meta, q, k, v = _setup(seed=12)
    outs = [torch.empty_like(q) for _ in range(2)]
    flags = [torch.zeros(8, dtype=torch.int32, device="cuda") for _ in range(2)]  # nobody sets flags[0][1]
    _loopback(q, k, v, meta, outs, flags, 1, 100)
    assert hb.device_status() & _lib.HB_DEV_PEER_TIMEOUT
    with torch.inference_mode():
        ref = hb.paired_attention(q, k, v, meta)  # the device still runs kernels
    torch.cuda.synchronize()
    assert hb.device_status() == 0
    assert torch.equal(outs[0], ref) and torch.equal(outs[1], ref)  # rows were stored before the wait


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, result):
    try:
        import torch.distributed as dist

        import hilberta_b200 as hb
        from hilberta_b200.head_parallel import PeerAllGather, local_heads

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
        plan = hb.bridge_k_plan(16, 3, False, grid_size=64)
        N, G = plan.total_tokens, plan.global_tokens
        metas = [
            hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=G).to(dev) for p in plan.phases
        ]
        H = 24  # 12 heads per rank: more work items than CTAs, so both copy paths run
        full = [x.to(dev) for x in ao.seeded_qkv(1, H, N, 128, seed=21)]
        ok = True
        for layout in ("bhnd", "bnhd"):
            with PeerAllGather(1, H, N, 128, layout=layout, timeout_ms=5000) as ag, torch.inference_mode():
                for call in range(6):
                    ph = call % 4
                    mine = [local_heads(x, rank, world) for x in full]
                    got = ag(*mine, metas[ph]).clone()
                    # every slice as the owning rank computes it (same kernel, same head count)
                    want = torch.cat(
                        [hb.paired_attention(*(local_heads(x, r, world) for x in full), metas[ph]) for r in range(world)],
                        dim=1,
                    )
                    torch.cuda.synchronize()
                    ok &= bool(torch.equal(got, want))
                ok &= hb.device_status() == 0
        dist.barrier()
        dist.destroy_process_group()
        result.put((rank, "ok" if ok else "mismatch"))
    except Exception as e:
        traceback.print_exc()
        result.put((rank, f"error: {type(e).__name__}: {e}"))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_fused_allgather_matches_slices():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert res == {0: "ok", 1: "ok"}
