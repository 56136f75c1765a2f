"""Pin the numpy oracle to the reference: every golden plan, the reference's
known-answer constants, and the reference dense-mask attention rows."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ao
from oracle import plan_oracle as po
from tests.golden_util import GOLDEN, check_plan, records


def _oracle_plan(case, kind):
    if kind == "build":
        return po.build_plan(case["tiles"], case["grid"], case["text"], case["shared"], case["bridge"], case["block"])
    return po.bridge_k_plan(case["tiles"], case["k"], case["shared"], grid_size=case["grid"])


def _pair(plan):
    def fn(i, p, kvb):
        return po.pair_metadata(
            p.kv_indices, p.kv_counts, tokens=plan.total_tokens, global_tokens=plan.global_tokens, key_block_size=kvb
        )

    return fn


NAMES = sorted(n for n in records() if records()[n]["case"].get("grid", 0) <= 128)


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_plan(name):
    rec = records()[name]
    kind = name.split("_")[0]
    if "error" in rec:
        exc = {"ValueError": ValueError, "AssertionError": AssertionError}[rec["error"]]
        with pytest.raises(exc):
            _oracle_plan(rec["case"], "build" if kind == "build" else "bridgek")
        return
    plan = _oracle_plan(rec["case"], "build" if kind == "build" else "bridgek")
    assert check_plan(name, plan, _pair(plan)) == []


@pytest.mark.slow
def test_oracle_matches_reference_plan_4096():
    name = "bridgek_tiles16_k3_shared0_grid256"
    plan = _oracle_plan(records()[name]["case"], "bridgek")
    assert check_plan(name, plan, _pair(plan)) == []


def test_known_bridge_budget():
    """``tests/test_plan.py:54-59``: extra 64x64 blocks per phase of the K=1 bridge."""
    for tiles, expected in [(4, [24, 34, 32, 34]), (16, [56, 57, 58, 55])]:
        a, b = po.build_plan(tiles, bridge=False), po.build_plan(tiles)
        delta = [int((b.dense_mask(i) & ~a.dense_mask(i)).sum()) // 4096 for i in range(4)]
        assert delta == expected
        assert a.physical_original_blocks[:4].tolist() == [15, 16, 47, 48]


def test_known_paired_toy():
    """``tests/test_paired_metadata.py:46-55``: ids [0,1,2], flags [15,9,9] (KV128)."""
    ids = np.array([[0, 1, 2, 4], [0, 1, 3, 5], [0, 1, 4, 5], [0, 1, 4, 5]], dtype=np.int32)
    pids, flags, counts = po.pair_metadata(ids, np.full(4, 4, np.int32), tokens=384, global_tokens=128, key_block_size=128)
    assert pids[0, :3].tolist() == [0, 1, 2]
    assert flags[0, :3].tolist() == [15, 9, 9]
    assert po.unpair_metadata(pids, flags, counts, 128) == ids.tolist()


def test_pair_round_trip_and_popcount():
    """``tests/test_paired_metadata.py:10-44`` on the oracle."""
    for tiles in (4, 16):
        for shared in (False, True):
            plan = po.build_plan(tiles, shared=shared, bridge=True)
            for p in plan.phases:
                exp = [p.kv_indices[r, : p.kv_counts[r]].tolist() for r in range(len(p.kv_counts))]
                for kvb in (64, 128):
                    ids, fl, cnt = po.pair_metadata(
                        p.kv_indices, p.kv_counts, tokens=plan.total_tokens, global_tokens=plan.global_tokens, key_block_size=kvb
                    )
                    assert po.unpair_metadata(ids, fl, cnt, kvb) == exp
                    bits = sum(int(f).bit_count() for r, n in zip(fl, cnt) for f in r[:n])
                    assert bits == int(p.kv_counts.sum())


def test_hilbert_rejects_bad_grid():
    for g in (0, 1, 3, 12):
        with pytest.raises(ValueError):
            po.hilbert_order(g)


def test_attention_oracle_matches_reference_rows():
    z = np.load(GOLDEN / "attention_small.npz")
    plan = po.bridge_k_plan(4, 1, False, grid_size=32)
    N = plan.total_tokens
    q, k, v = ao.seeded_qkv(1, 2, N, 64, seed=2707)
    import hashlib

    h = hashlib.sha256(torch.cat([q, k, v]).view(torch.int16).numpy().tobytes()).digest()
    assert np.frombuffer(h, np.uint8).tolist() == z["qkv_sha256"].tolist(), "seeded RNG drifted"
    rows = z["rows"]
    for phase in (0, 1):
        p = plan.phases[phase]
        bm = ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, plan.global_tokens)
        out = ao.masked_attention_fp32(q, k, v, bm, rows=rows)
        np.testing.assert_allclose(out.numpy(), z[f"out_phase{phase}"], atol=2e-6, rtol=1e-5)
        # the paired view of the same phase expands to the same block mask
        ids, fl, cnt = po.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=plan.global_tokens)
        assert np.array_equal(ao.block_mask_from_paired(ids, fl, cnt, N, plan.global_tokens), bm)
