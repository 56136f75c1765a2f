"""Tensor-parallel FLUX.1-architecture step on two GPUs (NCCL): each rank runs
HilbertA attention (persistent_flux_attention, backend "paired") on its half of
the heads inside the sharded blocks, and the step's output matches the
unsharded HilbertA step of the same weights."""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, sp):
    try:
        import hilberta_b200 as hb
        from hilberta_b200.flux_model import FluxTransformer, step_inputs
        from hilberta_b200.flux_tp import shard_flux_model

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
        plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
        torch.manual_seed(0)
        model = FluxTransformer(num_double=2, num_single=2, dim=512, heads=4, text_dim=64, pooled_dim=32, device=dev)
        x = step_inputs(32, plan.text_tokens, dev, seed=3, text_dim=64, pooled_dim=32)
        with torch.inference_mode(), hb.persistent_flux_attention(model, plan, backend="paired"):
            full = model(**x).sample.float()
        shard_flux_model(model, sequence_parallel=sp)
        with torch.inference_mode(), hb.persistent_flux_attention(model, plan, backend="paired"):
            local = model(**x).sample.float()
        rel = float((local - full).norm() / full.norm())
        heads_ok = all(b.attn.heads == 4 // world for b in model.single_transformer_blocks)
        status = hb.device_status(dev)
        q.put((rank, "ok" if rel < 2e-2 and heads_ok and status == 0 else f"rel {rel} heads {heads_ok} st {status}"))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, f"error: {type(e).__name__}: {e}"))
        traceback.print_exc()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("sp", [False, True])
def test_tensor_parallel_hilberta_step_two_gpus(sp):
    """sp: image / joined streams split by tokens (all-gather, reduce-scatter)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, sp)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}
