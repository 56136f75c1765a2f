"""The allocation-free entry point ``hb_paired_fwd_noalloc`` against the
allocating one, through the C ABI.

``hb_paired_fwd_noalloc`` exists for callers that cannot allocate device memory
when they enqueue work (runtime plugins whose host owns all device memory,
fixed-budget real-time services, bindings without a CUDA allocator): it keeps
the kernel's scheduler words in a static device array owned by the library
instead of a caller workspace.  This file is collected last so that a failure
here never hides the other tests; it builds its own inputs and passes both on
its own in a fresh process and after the rest of the suite.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _strides(q, k, v, out):
    return (ctypes.c_int64 * 12)(*q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *out.stride()[:3])


@pytest.mark.gpu
def test_noalloc_matches_allocating_entry_on_two_calls():
    import hilberta_b200 as hb
    from hilberta_b200 import _lib
    from oracle import attention_oracle as ao

    lib = _lib.lib()
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    plan = hb.bridge_k_plan(16, 3, False, grid_size=64)
    N, G = plan.total_tokens, plan.global_tokens
    stream = torch.cuda.current_stream(dev).cuda_stream
    ws_bytes = lib.hb_fwd_workspace_bytes_for(1, 4, N, G, 128)
    workspace = torch.zeros(ws_bytes // 4, dtype=torch.int32, device=dev)
    scale_log2 = 128**-0.5 * 1.4426950408889634
    for call, phase in enumerate((1, 3)):  # two calls in a row, different inputs and metadata
        p = plan.phases[phase]
        meta = hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=G).to(dev)
        q, k, v = (x.to(dev) for x in ao.seeded_qkv(1, 4, N, 128, seed=40 + call, layout="bnhd"))
        ref = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        args = (meta.kv_indices.shape[1], 64, _lib.ptr(meta.kv_indices), _lib.ptr(meta.kv_flags), _lib.ptr(meta.kv_counts))
        rc = lib.hb_paired_fwd(
            _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(ref), _strides(q, k, v, ref), 1, 4, N, 128, G, *args,
            scale_log2, 1, None, _lib.ptr(workspace), ws_bytes, ctypes.c_void_p(stream),
        )
        assert rc == 0, _lib.status_text(rc)
        rc = lib.hb_paired_fwd_noalloc(
            _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(got), _strides(q, k, v, got), 1, 4, N, 128, G, *args,
            scale_log2, 1, ctypes.c_void_p(stream),
        )
        assert rc == 0, _lib.status_text(rc)
        torch.cuda.synchronize()
        assert int(workspace[2].item()) == 0
        err = (got.float() - ref.float()).abs()
        assert torch.isfinite(got.float()).all()
        assert float(err.max()) <= MAX_ABS and float(err.mean()) <= MEAN_ABS, (call, float(err.max()))


@pytest.mark.parametrize("items_log2", [30, 31])
def test_noalloc_rejects_problems_beyond_its_limit(items_log2):
    """HB_NOALLOC_MAX_ITEMS is 2^30 - 1, the scheduler's own bound: exactly 2^30
    work items (B*H*N/128) is already refused, before any CUDA call, so this
    needs no GPU and the fake pointers are never touched."""
    from hilberta_b200 import _lib

    lib = _lib.lib()
    fake = ctypes.c_void_p(1 << 20)
    strides = (ctypes.c_int64 * 12)(*([1] * 12))
    B, H = 1 << 10, 1 << 10
    N = 128 << (items_log2 - 20)
    assert B * H * (N // 128) == 1 << items_log2
    rc = lib.hb_paired_fwd_noalloc(fake, fake, fake, fake, strides, B, H, N, 128, 0, 1, 64,
                                   fake, fake, fake, 0.1, 1, None)
    assert rc == _lib.HB_ERR_UNSUPPORTED
