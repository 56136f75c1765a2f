"""Generate the golden vectors that pin the CPU oracle and the CUDA builder.

Runs the REFERENCE implementation (wenboluu/hilberta, imported from a local
checkout given by ``--reference``; it is never vendored) and stores:

* ``plans_small.npz``  full arrays of the small plans (build_plan up to grid 64,
                       bridge_k_plan up to grid 32);
* ``plans.json``       sha256 digests + summary stats of every plan, including
                       the BASELINE-sized ones (grid 128/256), and the error
                       type of configurations the reference rejects;
* ``attention_small.npz`` rows of the reference's dense-mask fp32 attention
                       (``plan.dense_mask`` + ``F.scaled_dot_product_attention``,
                       the ``sdpa_reference`` computation) on seeded inputs.

Usage: python tests/golden/make_golden.py --reference <path-to-hilberta-checkout>
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
from oracle.attention_oracle import seeded_qkv  # noqa: E402


def digest(arr, dtype):
    a = np.ascontiguousarray(np.asarray(arr).astype(dtype))
    return hashlib.sha256(a.tobytes()).hexdigest()


BUILD_CASES = []
for grid, block, text in [(8, 4, 16), (16, 4, 16), (32, 64, 512), (64, 64, 512)]:
    for tiles in (4, 16):
        for shared in (False, True):
            for bridge in (False, True):
                BUILD_CASES.append(dict(tiles=tiles, grid=grid, text=text, shared=shared, bridge=bridge, block=block))

BRIDGE_CASES = []
for grid in (32, 64):
    for tiles in (4, 16):
        for k in (1, 2, 3, 4):
            for shared in (False, True):
                BRIDGE_CASES.append(dict(tiles=tiles, k=k, shared=shared, grid=grid))
for grid, tiles, k, shared in [(128, 4, 1, False), (128, 16, 3, False), (128, 16, 3, True), (256, 16, 3, False), (256, 4, 1, False)]:
    BRIDGE_CASES.append(dict(tiles=tiles, k=k, shared=shared, grid=grid))


def case_name(kind, c):
    return kind + "_" + "_".join(f"{k}{int(v) if isinstance(v, bool) else v}" for k, v in c.items())


def plan_record(plan, arrays, name, small, pair_sizes):
    rec = dict(
        grid_size=plan.grid_size,
        tile_count=plan.tile_count,
        text_tokens=plan.text_tokens,
        shared_tokens=plan.shared_tokens,
        block_size=plan.block_size,
        image_order=digest(plan.image_order, np.int64),
        inverse_image_order=digest(plan.inverse_image_order, np.int64),
        original_order=digest(plan.original_order, np.int64),
        physical_original_blocks=digest(plan.physical_original_blocks, np.int64),
        manifest_image_order_sha256=plan.manifest()["image_order_sha256"],
        phases=[],
    )
    if small:
        for f in ("image_order", "inverse_image_order", "original_order", "physical_original_blocks"):
            arrays[f"{name}.{f}"] = getattr(plan, f).numpy().astype(np.int64)
    from hilberta.paired_metadata import pair_metadata

    for i, p in enumerate(plan.phases):
        ph = dict(
            offset=int(p.offset),
            kv_shape=list(p.kv_indices.shape),
            kv_indices=digest(p.kv_indices, np.int32),
            kv_counts=digest(p.kv_counts, np.int32),
            kv_count_sum=int(p.kv_counts.sum()),
            bridge_original_blocks=digest(p.bridge_original_blocks, np.int64),
            bridge_shape=list(p.bridge_original_blocks.shape),
            paired={},
        )
        if small:
            arrays[f"{name}.p{i}.kv_indices"] = p.kv_indices.numpy()
            arrays[f"{name}.p{i}.kv_counts"] = p.kv_counts.numpy()
            arrays[f"{name}.p{i}.bridge_original_blocks"] = p.bridge_original_blocks.numpy()
        for kvb in pair_sizes:
            if plan.total_tokens % 128 or plan.global_tokens % 128 or plan.block_size != 64:
                continue
            m = pair_metadata(
                p.kv_indices, p.kv_counts, tokens=plan.total_tokens, global_tokens=plan.global_tokens, key_block_size=kvb
            )
            ph["paired"][str(kvb)] = dict(
                shape=list(m.kv_indices.shape),
                kv_indices=digest(m.kv_indices, np.int32),
                kv_flags=digest(m.kv_flags, np.int32),
                kv_counts=digest(m.kv_counts, np.int32),
                flag_bits=int(sum(int(f).bit_count() for r, n in zip(m.kv_flags, m.kv_counts) for f in r[: int(n)])),
            )
            if small:
                arrays[f"{name}.p{i}.kv{kvb}.ids"] = m.kv_indices.numpy()
                arrays[f"{name}.p{i}.kv{kvb}.flags"] = m.kv_flags.numpy()
                arrays[f"{name}.p{i}.kv{kvb}.counts"] = m.kv_counts.numpy()
        rec["phases"].append(ph)
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    from hilberta.plan import build_plan
    from hilberta.bridge_k import bridge_k_plan
    from hilberta.paired_metadata import pair_metadata

    torch.set_num_threads(8)
    arrays, records = {}, {}
    for c in BUILD_CASES:
        name = case_name("build", c)
        try:
            plan = build_plan(c["tiles"], c["grid"], c["text"], c["shared"], c["bridge"], c["block"])
        except (ValueError, AssertionError) as e:
            records[name] = dict(case=c, error=type(e).__name__)
            continue
        records[name] = dict(case=c, **plan_record(plan, arrays, name, True, (64, 128)))
    for c in BRIDGE_CASES:
        name = case_name("bridgek", c)
        try:
            plan = bridge_k_plan(c["tiles"], c["k"], c["shared"], grid_size=c["grid"])
        except (ValueError, AssertionError) as e:
            records[name] = dict(case=c, error=type(e).__name__)
            continue
        small = c["grid"] <= 32
        records[name] = dict(case=c, **plan_record(plan, arrays, name, small, (64,)))
        print(name, flush=True)
    # known answer: tests/test_paired_metadata.py:46-55 (6-block toy, KV128)
    ids = torch.tensor([[0, 1, 2, 4], [0, 1, 3, 5], [0, 1, 4, 5], [0, 1, 4, 5]], dtype=torch.int32)
    meta = pair_metadata(ids, torch.full((4,), 4, dtype=torch.int32), tokens=384, global_tokens=128, key_block_size=128)
    arrays["toy.ids"] = meta.kv_indices.numpy()
    arrays["toy.flags"] = meta.kv_flags.numpy()
    arrays["toy.counts"] = meta.kv_counts.numpy()
    np.savez_compressed(HERE / "plans_small.npz", **arrays)
    (HERE / "plans.json").write_text(json.dumps(records, indent=1, sort_keys=True))

    # attention: reference dense-mask path on seeded inputs, sampled rows
    plan = bridge_k_plan(4, 1, False, grid_size=32)
    N = plan.total_tokens
    q, k, v = seeded_qkv(1, 2, N, 64, seed=2707)
    rows = np.arange(0, N, 8)
    att = {}
    for phase in (0, 1):
        mask = plan.dense_mask(phase)
        ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), attn_mask=mask)
        att[f"out_phase{phase}"] = ref[:, :, rows].numpy()
    att["rows"] = rows
    att["qkv_sha256"] = np.frombuffer(
        hashlib.sha256(torch.cat([q, k, v]).view(torch.int16).numpy().tobytes()).digest(), dtype=np.uint8
    )
    np.savez_compressed(HERE / "attention_small.npz", **att)
    print("done")


if __name__ == "__main__":
    main()
