"""Parity of the sm_100a paired attention kernel (through the C ABI via the
``paired_attention`` shim) against the fp32 CPU dense-mask oracle.

Tolerance: max-abs <= 2e-2 and mean-abs <= 2e-3 against
the fp32 reference computed from the same bf16/fp16 inputs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ao

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _close(out, ref, what=""):
    err = (out.float().cpu() - ref.float()).abs()
    assert torch.isfinite(out.float()).all(), what
    assert float(err.max()) <= MAX_ABS, (what, float(err.max()))
    assert float(err.mean()) <= MEAN_ABS, (what, float(err.mean()))


def _meta(plan, phase, device="cuda"):
    import hilberta_b200 as hb

    p = plan.phases[phase]
    return hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=plan.total_tokens, global_tokens=plan.global_tokens).to(device), p


def _run(q, k, v, meta, **kw):
    import hilberta_b200 as hb

    with torch.inference_mode():
        out = hb.paired_attention(q.cuda(), k.cuda(), v.cuda(), meta, global_strategy="triton", num_warps=8, num_stages=2, **kw)
    torch.cuda.synchronize()
    assert hb.device_status() == 0
    return out


@pytest.mark.parametrize("phase", [0, 1, 2, 3])
def test_small_plan_all_phases_bhnd(phase):
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    meta, p = _meta(plan, phase)
    N, G = plan.total_tokens, plan.global_tokens
    q, k, v = ao.seeded_qkv(1, 2, N, 128, seed=100 + phase)
    out = _run(q, k, v, meta)
    ref = ao.masked_attention_fp32(q, k, v, ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G))
    _close(out, ref, f"phase {phase}")


def test_adapter_bnhd_view_layout_and_out_order():
    """Q/K/V as [B,H,N,D] views of [B,N,H,D] storage (flux_adapter.py:298); the
    output keeps q's storage order (empty_like)."""
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(16, 3, False, grid_size=64)
    meta, p = _meta(plan, 1)
    N, G = plan.total_tokens, plan.global_tokens
    q, k, v = ao.seeded_qkv(1, 3, N, 128, seed=5, layout="bnhd")
    out = _run(q, k, v, meta)
    assert out.stride() == q.stride()
    ref = ao.masked_attention_fp32(q, k, v, ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G))
    _close(out, ref)


def test_mixed_strides_and_given_out():
    """Contract case of test_paired_kernel_contract.py: BNHD q/v, BHND k, native out."""
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    meta, p = _meta(plan, 2)
    N, G = plan.total_tokens, plan.global_tokens
    q, _, v = ao.seeded_qkv(1, 2, N, 128, seed=9, layout="bnhd")
    _, k, _ = ao.seeded_qkv(1, 2, N, 128, seed=10)
    out = torch.empty(1, N, 2, 128, dtype=torch.bfloat16, device="cuda").transpose(1, 2)
    res = _run(q, k, v, meta, out=out)
    assert res is out
    ref = ao.masked_attention_fp32(q, k, v, ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G))
    _close(out, ref)


@pytest.mark.parametrize("dtype,D", [(torch.float16, 128), (torch.bfloat16, 64), (torch.float16, 64)])
def test_dtypes_and_head_dim(dtype, D):
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(4, 2, False, grid_size=32)
    meta, p = _meta(plan, 3)
    N, G = plan.total_tokens, plan.global_tokens
    q, k, v = ao.seeded_qkv(2, 3, N, D, seed=11, dtype=dtype)
    out = _run(q, k, v, meta)
    assert out.dtype == dtype
    ref = ao.masked_attention_fp32(q, k, v, ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G))
    _close(out, ref, str((dtype, D)))


def test_scale_argument():
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    meta, p = _meta(plan, 0)
    N, G = plan.total_tokens, plan.global_tokens
    q, k, v = ao.seeded_qkv(1, 2, N, 128, seed=12)
    out = _run(q, k, v, meta, scale=0.05)
    ref = ao.masked_attention_fp32(q, k, v, ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G), scale=0.05)
    _close(out, ref)


def _random_paired(N, G, seed, density=0.3):
    """Random valid paired metadata: every query half keeps >= 1 block; flags in
    {1,2,3} so whole half-tiles are masked, including leading entries."""
    rng = np.random.default_rng(seed)
    nb, rows = N // 64, (N - G) // 128
    lists = []
    for r in range(rows):
        blocks = np.nonzero(rng.random(nb) < density)[0]
        if len(blocks) < 2:
            blocks = np.array([0, nb - 1])
        flags = rng.integers(1, 4, len(blocks))
        flags[0] = 2  # the first entry is masked for query half 0
        if not (flags & 1).any():
            flags[-1] |= 1
        lists.append((blocks, flags))
    W = max(len(b) for b, _ in lists)
    ids = np.zeros((rows, W), np.int32)
    fl = np.zeros((rows, W), np.int32)
    cnt = np.zeros(rows, np.int32)
    for r, (b, f) in enumerate(lists):
        ids[r, : len(b)], fl[r, : len(b)], cnt[r] = b, f, len(b)
    return ids, fl, cnt


@pytest.mark.parametrize("G", [0, 128, 512])
def test_random_flags_and_masked_leading_entries(G):
    import hilberta_b200 as hb

    N = 2048
    ids, fl, cnt = _random_paired(N, G, seed=G + 1)
    meta = hb.PairedMetadata(
        torch.from_numpy(ids).cuda(), torch.from_numpy(fl).cuda(), torch.from_numpy(cnt).cuda(), N, G, 64
    )
    q, k, v = ao.seeded_qkv(1, 2, N, 128, seed=13)
    out = _run(q, k, v, meta)
    ref = ao.masked_attention_fp32(q, k, v, ao.block_mask_from_paired(ids, fl, cnt, N, G))
    _close(out, ref, f"G={G}")


def test_large_logits_force_rescaling():
    """Inputs scaled so the running max grows many times (lazy O rescale path)."""
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    meta, p = _meta(plan, 1)
    N, G = plan.total_tokens, plan.global_tokens
    q, k, v = ao.seeded_qkv(1, 2, N, 128, seed=14)
    ramp = torch.linspace(0.5, 4.0, N).view(1, 1, N, 1)
    k = (k.float() * ramp).to(torch.bfloat16)
    out = _run(q, k, v, meta)
    ref = ao.masked_attention_fp32(q, k, v, ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G))
    _close(out, ref)


def test_1024_t16k3_full_heads_subset():
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(16, 3, False, grid_size=64)
    N, G = plan.total_tokens, plan.global_tokens
    q, k, v = ao.seeded_qkv(1, 4, N, 128, seed=2707)
    for phase in (0, 3):
        meta, p = _meta(plan, phase)
        out = _run(q, k, v, meta)
        ref = ao.masked_attention_fp32(q, k, v, ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G))
        _close(out, ref, f"phase {phase}")


def test_2048_t16k3_24_heads_row_sampled():
    """BASELINE headline shape at full size; oracle on sampled rows of every head
    (global rows, both halves of ordinary pair-rows, the last row)."""
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(16, 3, False, grid_size=128)
    N, G = plan.total_tokens, plan.global_tokens
    q, k, v = ao.seeded_qkv(1, 24, N, 128, seed=2707)
    meta, p = _meta(plan, 0)
    out = _run(q, k, v, meta)
    rng = np.random.default_rng(0)
    rows = np.unique(np.concatenate([[0, 127, 511, 512, 575, 576, 639, N // 2, N - 1], rng.integers(0, N, 48)]))
    ref = ao.masked_attention_fp32(q, k, v, ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G), rows=rows)
    _close(out[:, :, torch.from_numpy(rows).cuda()], ref)


def test_repeated_calls_bitwise_deterministic():
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(16, 3, False, grid_size=64)
    meta, _ = _meta(plan, 2)
    q, k, v = (x.cuda() for x in ao.seeded_qkv(1, 24, plan.total_tokens, 128, seed=3))
    a = _run(q, k, v, meta)
    b = _run(q, k, v, meta)
    assert torch.equal(a, b)


def test_shared_workspace_across_split_shapes():
    """One workspace serving split launches of different group counts: the
    partials of a launch with few groups must not leave words where a launch with
    more groups keeps its chunk counters (result equals a fresh workspace's)."""
    import hilberta_b200 as hb
    from hilberta_b200 import paired_kernel as pk

    plan64 = hb.bridge_k_plan(16, 3, False, grid_size=64)
    meta64, _ = _meta(plan64, 2)
    q, k, v = (x.cuda() for x in ao.seeded_qkv(1, 24, plan64.total_tokens, 128, seed=7))
    pk._workspaces.clear()
    fresh = _run(q, k, v, meta64)
    plan128 = hb.bridge_k_plan(16, 3, False, grid_size=128)  # grows the workspace
    meta128, _ = _meta(plan128, 0)
    _run(*(x.cuda() for x in ao.seeded_qkv(1, 24, plan128.total_tokens, 128, seed=8)), meta128)
    _run(q[:, :2], k[:, :2], v[:, :2], meta64)  # few groups: partials right after the counters
    assert torch.equal(_run(q, k, v, meta64), fresh)
    assert torch.equal(_run(q, k, v, meta64), fresh)


def _unsplit(q, k, v, meta):
    """The same call through the C ABI with the minimal workspace (global rows run unsplit)."""
    import ctypes

    from hilberta_b200 import _lib
    from hilberta_b200.paired_kernel import LOG2E

    out = torch.empty_like(q)
    ws = torch.zeros(64, dtype=torch.int32, device=q.device)  # 256 bytes: no room for split partials
    B, H, N, D = q.shape
    strides = (ctypes.c_int64 * 12)(*q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *out.stride()[:3])
    rc = _lib.lib().hb_paired_fwd(
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), strides, B, H, N, D, meta.global_tokens,
        int(meta.kv_indices.shape[1]), 64, _lib.ptr(meta.kv_indices), _lib.ptr(meta.kv_flags),
        _lib.ptr(meta.kv_counts), float(D**-0.5 * LOG2E), 1 if q.dtype == torch.bfloat16 else 0, None,
        _lib.ptr(ws), 256, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert int(ws[2].item()) == 0
    return out


@pytest.mark.parametrize("dtype,D", [(torch.float16, 64), (torch.bfloat16, 64), (torch.float16, 128)])
def test_split_global_rows_fp16_and_d64(dtype, D):
    """Global rows split over key-block chunks (8 heads at 1024^2: 3 chunks per row)
    for fp16 and D=64, against the oracle and against the unsplit launch."""
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(16, 3, False, grid_size=64)
    meta, p = _meta(plan, 2)
    N, G = plan.total_tokens, plan.global_tokens
    q, k, v = (x.cuda() for x in ao.seeded_qkv(1, 8, N, D, seed=31, dtype=dtype))
    out = _run(q, k, v, meta)
    rows = np.concatenate([np.arange(0, G), np.arange(G, N, 11)])
    ref = ao.masked_attention_fp32(q.cpu(), k.cpu(), v.cpu(), ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G),
                                   rows=rows)
    _close(out[:, :, torch.from_numpy(rows).cuda()], ref, f"split {dtype} D{D}")
    with torch.inference_mode():
        whole = _unsplit(q, k, v, meta)
    _close(whole[:, :, torch.from_numpy(rows).cuda()], ref, "unsplit")
    assert torch.equal(out[:, :, G:], whole[:, :, G:])  # ordinary rows take the same path either way
    assert not torch.equal(out[:, :, :G], whole[:, :, :G])  # the global rows really were merged from chunks
