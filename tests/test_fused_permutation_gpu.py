"""Fused Hilbert gather/scatter (``paired_attention(token_order=...)``): with Q/K/V
kept in raster token order, the kernel gathers rows through the plan's
physical -> raster map while loading and scatters output rows, so the result
must equal permuting the inputs (``index_select``, the reference's entry pass,
hilberta/sampling_layout.py:88-103), running the kernel on the physical layout
and inverting the permutation (sampling_layout.py:105-113) — bit for bit, since
both run the same tiles in the same order."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as ao

pytestmark = pytest.mark.gpu


def _case(tiles, k, grid, heads, layout, phase, seed):
    import hilberta_b200 as hb
    from hilberta_b200.paired_kernel import token_order_map

    dev = torch.device("cuda", 0)
    plan = hb.bridge_k_plan(tiles, k, False, grid_size=grid)
    N, G = plan.total_tokens, plan.global_tokens
    p = plan.phases[phase]
    meta = hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=G).to(dev)
    rows = token_order_map(plan, dev)
    q, kk, v = (x.to(dev) for x in ao.seeded_qkv(1, heads, N, 128, seed=seed, layout=layout))  # raster order
    kw = dict(global_strategy="triton", num_warps=8, num_stages=2)
    with torch.inference_mode():
        fused = hb.paired_attention(q, kk, v, meta, token_order=rows, **kw)
        idx = rows.long()
        phys = [x.index_select(2, idx) for x in (q, kk, v)]
        out_phys = hb.paired_attention(*phys, meta, **kw)
        unperm = torch.empty_like(out_phys)
        unperm[:, :, idx] = out_phys
    torch.cuda.synchronize()
    assert hb.device_status() == 0
    return fused, unperm, (q, kk, v, p, N, G, rows)


@pytest.mark.parametrize("layout", ["bhnd", "bnhd"])
def test_fused_permutation_equals_explicit_reorder(layout):
    fused, ref, _ = _case(4, 1, 32, 2, layout, 1, 51)
    assert torch.equal(fused, ref)


def test_fused_permutation_against_oracle():
    fused, _, (q, k, v, p, N, G, rows) = _case(16, 3, 64, 3, "bnhd", 2, 52)
    # oracle in the physical layout, then scattered back to raster rows
    idx = rows.long().cpu()
    phys = [x.cpu().index_select(2, idx) for x in (q, k, v)]
    ref_phys = ao.masked_attention_fp32(*phys, ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G))
    ref = torch.empty_like(ref_phys)
    ref[:, :, idx] = ref_phys
    err = (fused.float().cpu() - ref).abs()
    assert float(err.max()) <= 2e-2 and float(err.mean()) <= 2e-3


def test_fused_permutation_2048_t16k3_all_heads():
    fused, ref, _ = _case(16, 3, 128, 24, "bnhd", 0, 53)
    assert torch.equal(fused, ref)


def test_token_order_validation():
    import hilberta_b200 as hb

    dev = torch.device("cuda", 0)
    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    N, G = plan.total_tokens, plan.global_tokens
    p = plan.phases[0]
    meta = hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=G).to(dev)
    q = torch.zeros(1, 2, N, 128, dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError, match="token_order"):
        hb.paired_attention(q, q.clone(), q.clone(), meta, token_order=torch.arange(N, device=dev))  # int64


def _raster_case(tiles, k, grid, heads, layout, phase, seed):
    import hilberta_b200 as hb
    from hilberta_b200.paired_kernel import raster_order

    dev = torch.device("cuda", 0)
    plan = hb.bridge_k_plan(tiles, k, False, grid_size=grid)
    N, G = plan.total_tokens, plan.global_tokens
    p = plan.phases[phase]
    meta = hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=G).to(dev)
    order = raster_order(plan, dev)
    q, kk, v = (x.to(dev) for x in ao.seeded_qkv(1, heads, N, 128, seed=seed, layout=layout))  # raster order
    kw = dict(global_strategy="triton", num_warps=8, num_stages=2)
    with torch.inference_mode():
        fused = hb.paired_attention(q, kk, v, meta, token_order=order, **kw)
        idx = order.rows().long()  # the kernel's own token order: row-major within each square
        out_phys = hb.paired_attention(*(x.index_select(2, idx) for x in (q, kk, v)), meta, **kw)
        ref = torch.empty_like(out_phys)
        ref[:, :, idx] = out_phys
    torch.cuda.synchronize()
    assert hb.device_status() == 0
    return fused, ref, (q, kk, v, p, N, G, idx)


@pytest.mark.parametrize("layout", ["bhnd", "bnhd"])
def test_raster_squares_equal_explicit_reorder(layout):
    fused, ref, _ = _raster_case(4, 1, 32, 2, layout, 1, 61)
    assert torch.equal(fused, ref)


def test_raster_squares_2048_t16k3_all_heads_against_oracle_rows():
    fused, ref, (q, k, v, p, N, G, idx) = _raster_case(16, 3, 128, 24, "bnhd", 3, 62)
    assert torch.equal(fused, ref)
    # sampled rows against the fp32 oracle, in physical layout
    phys = [x[:, :4].cpu().index_select(2, idx.cpu()) for x in (q, k, v)]
    mask = ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G)
    rows = torch.cat([torch.arange(0, 256), torch.arange(N - 2048, N, 7)])
    want = ao.masked_attention_fp32(*phys, mask, rows=rows.numpy())
    got = fused[:, :4].float().cpu()[:, :, idx.cpu()][:, :, rows]
    err = (got - want).abs()
    assert float(err.max()) <= 2e-2 and float(err.mean()) <= 2e-3


def test_raster_squares_bad_origin_drops_block():
    import hilberta_b200 as hb
    from hilberta_b200 import _lib
    from hilberta_b200.paired_kernel import RasterOrder, raster_order

    dev = torch.device("cuda", 0)
    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    N, G = plan.total_tokens, plan.global_tokens
    p = plan.phases[0]
    meta = hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=G).to(dev)
    good = raster_order(plan, dev)
    bad_origin = good.block_origin.clone()
    bad_origin[3] = 5  # not the corner of an aligned square
    q, k, v = (x.to(dev) for x in ao.seeded_qkv(1, 2, N, 128, seed=63))
    with torch.inference_mode():
        out = torch.full_like(q, 7.0)
        hb.paired_attention(q, k, v, meta, token_order=RasterOrder(good.text_tokens, good.grid, bad_origin), out=out)
    torch.cuda.synchronize()
    assert hb.device_status() & _lib.HB_DEV_BAD_BLOCK
    rows = good.rows().long().view(-1)
    dropped = rows[good.text_tokens + 3 * 64 : good.text_tokens + 4 * 64]
    assert bool((out[:, :, dropped] == 7.0).all())  # the bad block's rows were never written
    assert bool(torch.isfinite(out).all())


@pytest.mark.parametrize("mode", ["squares", "rows"])
def test_raster_orders_with_split_global_rows(mode):
    """Both raster-order layouts while the global rows are split over chunks
    (8 heads at 1024^2), bit-identical to the explicit reorder."""
    if mode == "squares":
        fused, ref, _ = _raster_case(16, 3, 64, 8, "bhnd", 2, 64)
    else:
        fused, ref, _ = _case(16, 3, 64, 8, "bhnd", 2, 65)
    assert torch.equal(fused, ref)
