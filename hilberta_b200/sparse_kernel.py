"""Metadata validation, explicit mask and tensor-property guards
(API of ``hilberta/sparse_kernel.py:100-250``).

``validate_metadata`` and ``explicit_mask`` run on the GPU; the guards below are
host-side checks on tensor metadata (pointers, shapes, strides) only.  The
reference's unpaired 32/64-query kernel (``_block_sparse_fwd``) is not rebuilt:
this package has one native attention kernel, the paired one.
"""

from __future__ import annotations

from numbers import Integral

import torch

from . import _lib
from .plan import dense_block_mask


def validate_metadata(
    kv_indices, kv_counts, *, tokens, global_tokens=768, block_size=64, require_global_prefix=True
):
    """Checks of ``sparse_kernel.py:100-152`` (same exceptions and messages);
    the per-row checks run in ``hb_validate_metadata``.  Returns the same stats dict.
    Accepts CPU or CUDA int32 tensors."""
    if block_size != 64:
        raise ValueError("This kernel currently requires 64-token physical blocks")
    if any(isinstance(v, bool) or not isinstance(v, Integral) for v in (tokens, global_tokens)):
        raise TypeError("tokens and global_tokens must be integers")
    if not (0 <= global_tokens < tokens) or tokens % block_size or global_tokens % block_size:
        raise ValueError("tokens/global prefix must be block-aligned with at least one ordinary block")
    if kv_indices.dtype != torch.int32 or kv_counts.dtype != torch.int32:
        raise TypeError("Block metadata must use int32")
    rows = (tokens - global_tokens) // block_size
    if kv_indices.ndim != 2 or kv_indices.shape[0] != rows or kv_indices.shape[1] < 1:
        raise ValueError("kv_indices must be [ordinary_query_blocks, max_KV_blocks]")
    if kv_counts.shape != (rows,):
        raise ValueError("kv_counts must have one entry per ordinary query block")
    if not kv_indices.is_contiguous() or not kv_counts.is_contiguous():
        raise ValueError("Metadata must be contiguous")
    dev = _lib.require_cuda(kv_indices.device if kv_indices.is_cuda else None)
    ids = kv_indices.to(dev)
    cnt = kv_counts.to(dev)
    res = torch.empty(4, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.lib().hb_validate_metadata(
            _lib.ptr(ids), ids.shape[1], ids.shape[1], _lib.ptr(cnt), rows, int(tokens),
            int(global_tokens) if require_global_prefix else 0, _lib.ptr(res), _lib.stream_ptr(dev)
        )
        _lib.check(rc, "hb_validate_metadata")
        first, cmin, cmax, total = res.cpu().tolist()
    if first != 2**31 - 1:
        row, code = divmod(first, 4)
        if code == 1:
            raise ValueError(f"Invalid K/V count in ordinary query block {row}")
        if code == 2:
            raise ValueError(f"Out-of-range or duplicate K/V blocks in row {row}")
        raise ValueError(f"Row {row} misses global-prefix keys")
    ordinary = total * block_size * block_size
    return {
        "tokens": tokens,
        "global_tokens": global_tokens,
        "block_size": block_size,
        "ordinary_query_blocks": rows,
        "min_kv_blocks": cmin,
        "max_kv_blocks": cmax,
        "global_directed_entries": global_tokens * tokens,
        "ordinary_directed_entries": ordinary,
        "total_directed_entries": global_tokens * tokens + ordinary,
    }


def explicit_mask(kv_indices, kv_counts, *, tokens, global_tokens=768, block_size=64):
    """CPU bool [tokens, tokens] correctness mask (``sparse_kernel.py:155-166``)."""
    validate_metadata(kv_indices, kv_counts, tokens=tokens, global_tokens=global_tokens, block_size=block_size)
    return dense_block_mask(kv_indices, kv_counts, tokens, global_tokens, block_size)


def _tensor_byte_span(tensor):
    """[begin, end) byte interval a strided tensor can touch (``sparse_kernel.py:169-174``)."""
    begin = tensor.data_ptr()
    extent = 1 + sum((size - 1) * stride for size, stride in zip(tensor.shape, tensor.stride()))
    return begin, begin + extent * tensor.element_size()


def _non_overlapping_strides(tensor):
    """True when no two indices share storage (``sparse_kernel.py:177-185``)."""
    extent = 1
    for stride, size in sorted((stride, size) for stride, size in zip(tensor.stride(), tensor.shape) if size > 1):
        if stride < extent:
            return False
        extent += (size - 1) * stride
    return True
