"""Paired metadata with 128-key blocks (paired_metadata.py:26-51, key_block_size
128; accepted by the reference kernel, paired_kernel.py:65-75, 128): expanded on
the device (hb_expand_kv128) to the equivalent KV64 rows, which must equal
pair_metadata's KV64 table entry for entry, so the attention is bit-identical to
the KV64 call; and against the fp32 dense-mask oracle of the KV128 flags.

Tolerance (north star): max-abs <= 2e-2, mean-abs <= 2e-3 vs fp32."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ao

pytestmark = pytest.mark.gpu


def _pair(plan, phase, kvb):
    import hilberta_b200 as hb

    p = plan.phases[phase]
    return hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=plan.total_tokens, global_tokens=plan.global_tokens,
                            key_block_size=kvb).to("cuda")


@pytest.mark.parametrize("phase", [0, 1, 2, 3])
def test_expansion_equals_kv64_metadata(phase):
    import hilberta_b200 as hb
    from hilberta_b200.paired_kernel import _as_kv64

    plan = hb.bridge_k_plan(16, 3, False, grid_size=64)
    m128, m64 = _pair(plan, phase, 128), _pair(plan, phase, 64)
    e = _as_kv64(m128)
    assert e.key_block_size == 64
    assert torch.equal(e.kv_counts, m64.kv_counts)
    for r in range(m64.kv_counts.numel()):
        c = int(m64.kv_counts[r])
        assert torch.equal(e.kv_indices[r, :c], m64.kv_indices[r, :c]), r
        assert torch.equal(e.kv_flags[r, :c], m64.kv_flags[r, :c]), r


def test_kv128_attention_equals_kv64_and_oracle():
    import hilberta_b200 as hb

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    q, k, v = (x.cuda() for x in ao.seeded_qkv(1, 2, plan.total_tokens, 128, seed=31))
    with torch.inference_mode():
        for phase in range(4):
            m128, m64 = _pair(plan, phase, 128), _pair(plan, phase, 64)
            out128 = hb.paired_attention(q, k, v, m128)
            out64 = hb.paired_attention(q, k, v, m64)
            assert torch.equal(out128, out64), phase
    assert hb.device_status() == 0
    m128 = _pair(plan, 3, 128)
    mask = ao.block_mask_from_paired(m128.kv_indices.cpu(), m128.kv_flags.cpu(), m128.kv_counts.cpu(),
                                     plan.total_tokens, plan.global_tokens, key_block_size=128)
    ref = ao.masked_attention_fp32(q.cpu(), k.cpu(), v.cpu(), mask)
    err = (out128.float().cpu() - ref).abs()
    assert float(err.max()) <= 2e-2 and float(err.mean()) <= 2e-3


def test_reference_six_block_example():
    """tests/test_paired_metadata.py:46-55 of the reference: ids [0, 1, 2],
    flags [15, 9, 9] for KV128 over 384 tokens, 128 global."""
    import hilberta_b200 as hb

    ids = torch.tensor([[0, 1, 2, 4], [0, 1, 3, 5], [0, 1, 4, 5], [0, 1, 4, 5]], dtype=torch.int32)
    meta = hb.pair_metadata(ids, torch.full((4,), 4, dtype=torch.int32), tokens=384, global_tokens=128,
                            key_block_size=128).to("cuda")
    assert meta.kv_flags[0, :3].tolist() == [15, 9, 9]
    q, k, v = (x.cuda() for x in ao.seeded_qkv(1, 3, 384, 64, seed=32))
    with torch.inference_mode():
        out = hb.paired_attention(q, k, v, meta)
    mask = ao.block_mask_from_paired(meta.kv_indices.cpu(), meta.kv_flags.cpu(), meta.kv_counts.cpu(), 384, 128,
                                     key_block_size=128)
    ref = ao.masked_attention_fp32(q.cpu(), k.cpu(), v.cpu(), mask)
    err = (out.float().cpu() - ref).abs()
    assert float(err.max()) <= 2e-2 and float(err.mean()) <= 2e-3


def test_in_place_edit_is_re_expanded():
    import hilberta_b200 as hb
    from hilberta_b200.paired_kernel import _as_kv64

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    m128 = _pair(plan, 0, 128)
    first = _as_kv64(m128)
    assert _as_kv64(m128) is first  # cached
    m128.kv_flags[0, 0] = 1  # only query half 0 of key half 0 stays visible
    second = _as_kv64(m128)
    assert second is not first
    assert int(second.kv_flags[0, 0]) == 1 and int(second.kv_indices[0, 0]) == 2 * int(m128.kv_indices[0, 0])


def test_inference_mode_tables_are_expanded_every_call():
    import hilberta_b200 as hb
    from hilberta_b200.paired_kernel import _as_kv64

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    with torch.inference_mode():
        m128 = _pair(plan, 1, 128)
        a = _as_kv64(m128)
        m128.kv_flags[0, 0] = 2  # query half 1 only, key half 0
        b = _as_kv64(m128)
    assert b is not a and int(b.kv_flags[0, 0]) == 2
