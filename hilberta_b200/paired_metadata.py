"""Paired (128-query) metadata (API of ``hilberta/paired_metadata.py``), built on the device."""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch

from . import _lib
from .sparse_kernel import validate_metadata


@dataclass(frozen=True)
class PairedMetadata:
    kv_indices: torch.Tensor
    kv_flags: torch.Tensor
    kv_counts: torch.Tensor
    tokens: int
    global_tokens: int
    key_block_size: int

    def to(self, device):
        return replace(
            self,
            kv_indices=self.kv_indices.to(device),
            kv_flags=self.kv_flags.to(device),
            kv_counts=self.kv_counts.to(device),
        )


def pair_metadata(kv_indices, kv_counts, *, tokens, global_tokens=768, key_block_size=64):
    """Merge query rows 2i, 2i+1 into one sorted list of unique key blocks with a
    flag bit (half + 2*key_half) per original 64x64 visibility
    (``paired_metadata.py:26-51``); ``hb_pair_metadata`` does the merge.
    The result lives on the inputs' device (CPU in -> CPU out)."""
    validate_metadata(kv_indices, kv_counts, tokens=tokens, global_tokens=global_tokens)
    if key_block_size not in (64, 128) or tokens % 128 or global_tokens % 128:
        raise ValueError("Paired queries require N/global aligned to 128; KV must be 64/128")
    home = kv_indices.device
    dev = _lib.require_cuda(home if home.type == "cuda" else None)
    ids = kv_indices.to(dev).contiguous()
    cnt = kv_counts.to(dev).contiguous()
    rows = cnt.numel()
    ratio = key_block_size // 64
    cap = -(-(tokens // 64) // ratio)
    out_ids = torch.empty(rows // 2, cap, dtype=torch.int32, device=dev)
    out_flags = torch.empty_like(out_ids)
    out_counts = torch.empty(rows // 2, dtype=torch.int32, device=dev)
    info = torch.zeros(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.lib().hb_pair_metadata(
            _lib.ptr(ids), ids.shape[1], _lib.ptr(cnt), rows, int(tokens), int(global_tokens), int(key_block_size),
            _lib.ptr(out_ids), _lib.ptr(out_flags), cap, _lib.ptr(out_counts), _lib.ptr(info), _lib.stream_ptr(dev)
        )
        _lib.check(rc, "hb_pair_metadata")
        width = int(info.item())
    return PairedMetadata(
        out_ids[:, :width].contiguous().to(home),
        out_flags[:, :width].contiguous().to(home),
        out_counts.to(home),
        tokens,
        global_tokens,
        key_block_size,
    )


def unpair_metadata(meta):
    """Reconstruct the original per-64-query block lists from CPU paired metadata,
    independently checking flags (``paired_metadata.py:54-70``)."""
    if any(x.device.type != "cpu" for x in (meta.kv_indices, meta.kv_flags, meta.kv_counts)):
        raise ValueError("CPU metadata required for validation")
    ratio = meta.key_block_size // 64
    rows = []
    for row, count in enumerate(meta.kv_counts.tolist()):
        ids = meta.kv_indices[row, :count].tolist()
        flags = meta.kv_flags[row, :count].tolist()
        for half in range(2):
            rows.append(
                sorted(b * ratio + kh for b, f in zip(ids, flags) for kh in range(ratio) if f & (1 << (half + 2 * kh)))
            )
    return rows
