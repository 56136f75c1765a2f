"""Head-parallel partition + all-gather on CPU ranks (gloo, world size 2), and
the failure path: a rank that dies before the collective makes the surviving
rank's gather raise within the process-group timeout instead of hanging.
Nothing here touches a GPU."""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hilberta_b200.head_parallel import all_gather_heads, head_range, local_heads


def test_head_range_partition():
    for world in (1, 2, 4, 8):
        spans = [head_range(24, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 24
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert {s[1] - s[0] for s in spans} == {24 // world}
    with pytest.raises(ValueError):
        head_range(24, 0, 5)
    with pytest.raises(ValueError):
        head_range(24, 2, 2)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        g = torch.Generator().manual_seed(0)
        full = torch.randn(1, 24, 256, 64, generator=g)
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected rank failure before the gather")
        mine = local_heads(full, rank, world)
        if mode == "bnhd":
            mine = mine.transpose(1, 2).contiguous().transpose(1, 2)  # BNHD storage viewed as BHND
            got = all_gather_heads(mine, layout="bnhd")
            ok = torch.equal(got, full.transpose(1, 2))
        else:
            got = all_gather_heads(mine)
            ok = torch.equal(got, full)
        q.put((rank, "ok" if ok else "mismatch"))
        dist.destroy_process_group()
    except Exception as e:  # report, then exit non-zero
        q.put((rank, f"error: {type(e).__name__}: {e}"))
        if mode != "fail":
            traceback.print_exc()


@pytest.mark.parametrize("mode", ["bhnd", "bnhd"])
def test_gloo_all_gather_heads_two_ranks(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}


def test_gloo_rank_failure_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, "fail", q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1].startswith("error: RuntimeError: injected")
    assert res[0].startswith("error:"), res[0]  # the survivor's collective failed, it did not hang
