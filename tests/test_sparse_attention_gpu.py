"""sparse_attention (the reference's unpaired operator, hilberta/sparse_kernel.py:
253-339) on this package's paired kernel: bit-identical to paired_attention on
the paired rows, within the north-star tolerance of the fp32 dense-mask oracle
(max-abs 2e-2, mean-abs 2e-3), the pairing done once per table."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as ao

pytestmark = pytest.mark.gpu


def test_sparse_attention_equals_paired_and_oracle():
    import hilberta_b200 as hb
    from hilberta_b200.sparse_kernel import _paired_rows_cache, sparse_attention

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    N, G = plan.total_tokens, plan.global_tokens
    q, k, v = (x.cuda() for x in ao.seeded_qkv(1, 2, N, 128, seed=41))
    p = plan.phases[2]
    ids, counts = p.kv_indices.cuda(), p.kv_counts.cuda()
    meta = hb.pair_metadata(ids, counts, tokens=N, global_tokens=G)
    before = len(_paired_rows_cache)
    with torch.no_grad():
        out = sparse_attention(q, k, v, ids, counts, global_tokens=G, global_strategy="triton", num_warps=8)
        again = sparse_attention(q, k, v, ids, counts, global_tokens=G)
        want = hb.paired_attention(q, k, v, meta)
    assert len(_paired_rows_cache) == before + 1  # paired once
    assert torch.equal(out, want) and torch.equal(again, want)
    assert hb.device_status() == 0
    ref = ao.masked_attention_fp32(q.cpu(), k.cpu(), v.cpu(), ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G))
    err = (out.float().cpu() - ref).abs()
    assert float(err.max()) <= 2e-2 and float(err.mean()) <= 2e-3


def test_sparse_backend_under_inference_mode_pairs_each_table_once(monkeypatch):
    """The adapter's sparse backend reads the unpaired rows from PlanBank's
    device copies.  Built on a first call under inference mode they must still
    be normal tensors (inference tensors carry no version counter), so the
    pairing cache hits and every phase is paired once, not on every call."""
    import hilberta_b200 as hb
    from hilberta_b200 import paired_metadata as pm
    from hilberta_b200 import sparse_kernel as sk

    calls = []
    real = pm.pair_metadata

    def counting(*a, **kw):
        calls.append(1)
        return real(*a, **kw)

    monkeypatch.setattr(pm, "pair_metadata", counting)
    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    N, G = plan.total_tokens, plan.global_tokens
    bank = hb.PlanBank(plan, backend="sparse")
    q, k, v = (x.cuda() for x in ao.seeded_qkv(1, 2, N, 128, seed=42))
    sk._paired_rows_cache.clear()
    outs = []
    with torch.inference_mode():
        for layer in range(12):  # three passes over the four phases
            ids, counts = bank.on_device(q.device)["phases"][layer % 4]
            assert not ids.is_inference() and not counts.is_inference()
            outs.append(sk.sparse_attention(q, k, v, ids, counts, global_tokens=G))
    assert len(calls) == 4
    for layer in range(4, 12):
        assert torch.equal(outs[layer], outs[layer % 4])
    assert hb.device_status() == 0
