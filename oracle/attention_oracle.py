"""fp32 CPU dense-mask attention: the reference's correctness path, restated.

TEST INFRASTRUCTURE ONLY (parity checker and the timed CPU baseline of
``bench.py --impl reference``); the product path never imports it.

The reference's oracle for the sparse kernel is ``AttentionPlan.dense_mask``
(``hilberta/plan.py:70-84``) / ``explicit_mask`` (``hilberta/sparse_kernel.py:155-166``)
fed to ``F.scaled_dot_product_attention`` with a bool mask
(``hilberta/flux_adapter.py:299-307`` ``sdpa_reference``; ``hilberta/benchmark.py:59-70``).
This module builds the same block mask from paired or unpaired metadata and
evaluates softmax(Q K^T * scale + mask) V in fp32 from the bf16/fp16 inputs,
per head and per query chunk so the N x N mask never materialises.
"""

from __future__ import annotations

import numpy as np
import torch


def block_mask_from_rows(kv_indices, kv_counts, tokens, global_tokens, block_size=64):
    """[N/b, N/b] bool block mask; rows < G/b are all True (``plan.py:76-79``)."""
    nb = tokens // block_size
    g = global_tokens // block_size
    m = np.zeros((nb, nb), dtype=bool)
    m[:g] = True
    ids = np.asarray(kv_indices)
    cnt = np.asarray(kv_counts)
    for r in range(len(cnt)):
        m[g + r, ids[r, : cnt[r]]] = True
    return m


def block_mask_from_paired(ids, flags, counts, tokens, global_tokens, key_block_size=64):
    """Expand paired metadata (``paired_metadata.py:26-51``) to the 64x64 block mask."""
    nb = tokens // 64
    g = global_tokens // 64
    ratio = key_block_size // 64
    m = np.zeros((nb, nb), dtype=bool)
    m[:g] = True
    ids = np.asarray(ids)
    flags = np.asarray(flags)
    for r, c in enumerate(np.asarray(counts).tolist()):
        for j in range(c):
            for half in range(2):
                for kh in range(ratio):
                    if flags[r, j] & (1 << (half + 2 * kh)):
                        m[g + 2 * r + half, ids[r, j] * ratio + kh] = True
    return m


@torch.no_grad()
def masked_attention_fp32(q, k, v, block_mask, *, scale=None, rows=None, chunk=1024, threads=None):
    """softmax(QK^T*scale + mask) V in fp32 on CPU.

    q/k/v: [B,H,N,D] (any float dtype, any strides).  block_mask: [N/64, N/64] bool.
    rows: optional 1-D int array of query rows to evaluate (row-sampled oracle,
    like ``benchmark.py:59-70``); returns [B,H,len(rows),D] then, else [B,H,N,D].
    """
    if threads is not None:
        torch.set_num_threads(int(threads))
    B, H, N, D = q.shape
    scale = D**-0.5 if scale is None else float(scale)
    bm = torch.as_tensor(np.asarray(block_mask))
    qrows = torch.arange(N) if rows is None else torch.as_tensor(np.asarray(rows), dtype=torch.long)
    out = torch.empty(B, H, len(qrows), D, dtype=torch.float32)
    kf = k.detach().to("cpu", torch.float32)
    vf = v.detach().to("cpu", torch.float32)
    qf = q.detach().to("cpu", torch.float32)
    for s in range(0, len(qrows), chunk):
        r = qrows[s : s + chunk]
        mask = bm[r // 64].repeat_interleave(64, dim=1)  # [len(r), N]
        for b in range(B):
            for h in range(H):
                out[b, h, s : s + len(r)] = torch.nn.functional.scaled_dot_product_attention(
                    qf[b, h, r][None], kf[b, h][None], vf[b, h][None], attn_mask=mask[None], scale=scale
                )[0]
    return out


def seeded_qkv(B, H, N, D, seed=2707, dtype=torch.bfloat16, layout="bhnd"):
    """Q, K, V ~ N(0,1) drawn in that order after ``torch.manual_seed(seed)``
    (``hilberta/benchmark.py:24-28``).  layout "bnhd" returns [B,H,N,D] views of
    [B,N,H,D] storage, the adapter's layout (``flux_adapter.py:298``)."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(3):
        if layout == "bhnd":
            out.append(torch.randn(B, H, N, D, generator=g, dtype=torch.float32).to(dtype))
        else:
            out.append(torch.randn(B, N, H, D, generator=g, dtype=torch.float32).to(dtype).transpose(1, 2))
    return out
