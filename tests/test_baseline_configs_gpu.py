"""Kernel parity on every BASELINE configuration and every tile phase.

The reference's own benchmark gates each phase of each configuration on the
kernel output against a masked SDPA of sampled rows (hilberta/benchmark.py:
51-72).  Here the sm_100a kernel (through ``paired_attention`` and the C ABI)
is compared with the fp32 dense-mask oracle (``oracle/attention_oracle.py``,
the ``plan.dense_mask`` + SDPA computation of hilberta/plan.py:70-84 and
flux_adapter.py:299-307) at the north-star tolerance, max-abs <= 2e-2 and
mean-abs <= 2e-3, on the full 24 heads of the BASELINE shapes:

* 1024^2 4-tile K1 and 16-tile K3 (grid 64): every output row of every phase;
* 2048^2 4-tile K1 (the widest plan: 75 entries per pair-row) and 2048^2
  16-tile K3 (the headline shape): every phase, >= 256 sampled rows per phase
  (global rows including the first and last, both halves of 64+ pair-rows, the
  last row);
* 4096^2 16-tile K3 (performance only in BASELINE): phases 0 and 3, sampled rows,
  physical order;

each in the physical token order of the metadata and in raster token order
(8x8-square TMA boxes, ``token_order=raster_order(plan)``), where the inputs
are the same tokens scattered to their raster rows.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ao

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3
KW = dict(global_strategy="triton", num_warps=8, num_stages=2)


def _sample_rows(N, G, seed):
    """Sorted query rows: global rows (first, last and 48 random), both halves of
    72 pair-rows (the first, the last and 70 random), 64 random rows, the last row."""
    rng = np.random.default_rng(seed)
    pairs = (N - G) // 128
    glob = np.concatenate([[0, 1, 63, 64, 127, 128, G - 2, G - 1], rng.integers(0, G, 48)])
    chosen = np.concatenate([[0, pairs - 1], rng.choice(pairs, min(pairs, 70), replace=False)])
    halves = []
    for p in chosen:
        base = G + 128 * p
        halves += [base + rng.integers(0, 64), base + 64 + rng.integers(0, 64)]
    rows = np.unique(np.concatenate([glob, halves, rng.integers(G, N, 64), [G, N - 1]]))
    assert len(rows) >= 256
    return rows


def _check(got, want, what):
    assert torch.isfinite(got).all(), what
    err = (got.float() - want.float()).abs()
    assert float(err.max()) <= MAX_ABS, (what, float(err.max()))
    assert float(err.mean()) <= MEAN_ABS, (what, float(err.mean()))


def _config(tiles, k, grid, *, all_rows, seed):
    import hilberta_b200 as hb
    from hilberta_b200.paired_kernel import raster_order

    dev = torch.device("cuda", 0)
    plan = hb.bridge_k_plan(tiles, k, False, grid_size=grid)
    N, G = plan.total_tokens, plan.global_tokens
    q, kk, v = ao.seeded_qkv(1, 24, N, 128, seed=seed)  # physical token order
    order = raster_order(plan, dev)
    idx = order.rows().long()  # physical token p -> its raster row
    dq, dk, dv = (x.to(dev) for x in (q, kk, v))
    rq, rk, rv = (torch.empty_like(x).index_copy_(2, idx, x) for x in (dq, dk, dv))  # the same tokens, raster rows
    for phase in range(4):
        p = plan.phases[phase]
        meta = hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=G).to(dev)
        with torch.inference_mode():
            phys = hb.paired_attention(dq, dk, dv, meta, **KW)
            rast = hb.paired_attention(rq, rk, rv, meta, token_order=order, **KW)
        torch.cuda.synchronize()
        assert hb.device_status() == 0
        rows = np.arange(N) if all_rows else _sample_rows(N, G, seed + phase)
        want = ao.masked_attention_fp32(q, kk, v, ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G),
                                        rows=rows)
        sel = torch.from_numpy(rows).to(dev)
        _check(phys[:, :, sel].cpu(), want, f"physical order, phase {phase}")
        _check(rast[:, :, idx[sel]].cpu(), want, f"raster order, phase {phase}")


def test_1024_t4k1_all_phases_all_rows():
    _config(4, 1, 64, all_rows=True, seed=2707)


def test_2048_t4k1_all_phases_sampled_rows():
    _config(4, 1, 128, all_rows=False, seed=2708)


def test_2048_t16k3_all_phases_sampled_rows():
    _config(16, 3, 128, all_rows=False, seed=2709)


def test_1024_t16k3_all_phases_all_rows():
    _config(16, 3, 64, all_rows=True, seed=2710)


def test_4096_t16k3_sampled_rows_phases_0_and_3():
    """The performance-only BASELINE shape (66 048 tokens, 24 heads), physical
    order, phases 0 and 3: the widest rows (75 paired entries), where each
    global row's last key blocks run as separate tail chunks merged at the end."""
    import hilberta_b200 as hb

    dev = torch.device("cuda", 0)
    plan = hb.bridge_k_plan(16, 3, False, grid_size=256)
    N, G = plan.total_tokens, plan.global_tokens
    q, kk, v = ao.seeded_qkv(1, 24, N, 128, seed=2711)
    dq, dk, dv = (x.to(dev) for x in (q, kk, v))
    for phase in (0, 3):
        p = plan.phases[phase]
        meta = hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=G).to(dev)
        with torch.inference_mode():
            got = hb.paired_attention(dq, dk, dv, meta, **KW)
        torch.cuda.synchronize()
        assert hb.device_status() == 0
        rows = _sample_rows(N, G, 2711 + phase)
        want = ao.masked_attention_fp32(q, kk, v, ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G),
                                        rows=rows)
        _check(got[:, :, torch.from_numpy(rows).to(dev)].cpu(), want, f"4096^2 physical order, phase {phase}")
