"""CUDA metadata builder vs the reference, bit for bit (golden vectors from the
reference run by ``tests/golden/make_golden.py``), plus the reference's own
known-answer constants and error contract."""

from __future__ import annotations

import pytest
import torch

from tests.golden_util import check_plan, records

pytestmark = pytest.mark.gpu


def _plan(name):
    import hilberta_b200 as hb

    c = records()[name]["case"]
    if name.startswith("build"):
        return hb.build_plan(c["tiles"], c["grid"], c["text"], c["shared"], c["bridge"], c["block"])
    return hb.bridge_k_plan(c["tiles"], c["k"], c["shared"], grid_size=c["grid"])


def _pair(plan):
    import hilberta_b200 as hb

    def fn(i, p, kvb):
        m = hb.pair_metadata(
            p.kv_indices, p.kv_counts, tokens=plan.total_tokens, global_tokens=plan.global_tokens, key_block_size=kvb
        )
        return m.kv_indices, m.kv_flags, m.kv_counts

    return fn


@pytest.mark.parametrize("name", sorted(records()))
def test_cuda_builder_matches_reference(name):
    rec = records()[name]
    if "error" in rec:
        exc = {"ValueError": ValueError, "AssertionError": AssertionError}[rec["error"]]
        with pytest.raises(exc):
            _plan(name)
        return
    plan = _plan(name)
    assert check_plan(name, plan, _pair(plan)) == []
    assert plan.manifest()["image_order_sha256"] == rec["manifest_image_order_sha256"]


def test_known_bridge_budget_cuda():
    """``tests/test_plan.py:54-59`` against the CUDA builder and its dense mask."""
    import hilberta_b200 as hb

    for tiles, expected in [(4, [24, 34, 32, 34]), (16, [56, 57, 58, 55])]:
        a, b = hb.build_plan(tiles, bridge=False), hb.build_plan(tiles)
        delta = [int((b.dense_mask(i) & ~a.dense_mask(i)).sum()) // 4096 for i in range(4)]
        assert delta == expected
        assert a.physical_original_blocks[:4].tolist() == [15, 16, 47, 48]


def test_known_paired_toy_cuda():
    """``tests/test_paired_metadata.py:46-55``: ids [0,1,2], flags [15,9,9] (KV128)."""
    import hilberta_b200 as hb

    ids = torch.tensor([[0, 1, 2, 4], [0, 1, 3, 5], [0, 1, 4, 5], [0, 1, 4, 5]], dtype=torch.int32)
    meta = hb.pair_metadata(ids, torch.full((4,), 4, dtype=torch.int32), tokens=384, global_tokens=128, key_block_size=128)
    assert meta.kv_indices[0, :3].tolist() == [0, 1, 2]
    assert meta.kv_flags[0, :3].tolist() == [15, 9, 9]
    assert hb.unpair_metadata(meta) == ids.tolist()


def test_full_layout_gate_cuda():
    """``tests/test_plan.py:61-63``."""
    import hilberta_b200 as hb

    p = hb.full_attention_plan(hb.build_plan(16, 16, 16, True, True, 4))
    assert all(p.dense_mask(i).all() for i in range(4))


def test_hilbert_order_cuda_matches_oracle():
    import hilberta_b200.geometry as geo
    from oracle import plan_oracle as po

    for g in (2, 4, 8, 64, 256):
        assert geo.hilbert_order(g).numpy().tolist() == po.hilbert_order(g).tolist()


def test_validate_metadata_errors_cuda():
    """Device validation raises the reference's messages on the first bad row
    (``sparse_kernel.py:136-145``)."""
    import hilberta_b200 as hb

    ids = torch.tensor([[0, 1, 2, 0], [0, 1, 3, 0], [0, 1, 2, 3]], dtype=torch.int32)
    cnt = torch.tensor([3, 3, 4], dtype=torch.int32)
    st = hb.validate_metadata(ids, cnt, tokens=320, global_tokens=128)
    assert st["max_kv_blocks"] == 4 and st["min_kv_blocks"] == 3 and st["ordinary_directed_entries"] == 10 * 4096
    bad = cnt.clone()
    bad[1] = 5
    with pytest.raises(ValueError, match="Invalid K/V count in ordinary query block 1"):
        hb.validate_metadata(ids, bad, tokens=320, global_tokens=128)
    dup = ids.clone()
    dup[2, 3] = 2
    with pytest.raises(ValueError, match="duplicate K/V blocks in row 2"):
        hb.validate_metadata(dup, cnt, tokens=320, global_tokens=128)
    oor = ids.clone()
    oor[0, 2] = 5
    with pytest.raises(ValueError, match="Out-of-range"):
        hb.validate_metadata(oor, cnt, tokens=320, global_tokens=128)
    noglob = ids.clone()
    noglob[0, 0] = 4
    with pytest.raises(ValueError, match="Row 0 misses global-prefix keys"):
        hb.validate_metadata(noglob, cnt, tokens=320, global_tokens=128)
    hb.validate_metadata(noglob, cnt, tokens=320, global_tokens=128, require_global_prefix=False)


def test_explicit_mask_cuda_matches_oracle():
    import numpy as np

    import hilberta_b200 as hb
    from oracle import attention_oracle as ao

    plan = hb.bridge_k_plan(16, 3, False, grid_size=64)
    p = plan.phases[2]
    m = hb.explicit_mask(p.kv_indices, p.kv_counts, tokens=plan.total_tokens, global_tokens=plan.global_tokens)
    bm = ao.block_mask_from_rows(p.kv_indices.numpy(), p.kv_counts.numpy(), plan.total_tokens, plan.global_tokens)
    assert np.array_equal(m.numpy(), np.repeat(np.repeat(bm, 64, 0), 64, 1))
