"""Metadata validation, explicit mask and tensor-property guards
(API of ``hilberta/sparse_kernel.py:100-250``).

``validate_metadata`` and ``explicit_mask`` run on the GPU; the guards below are
host-side checks on tensor metadata (pointers, shapes, strides) only.  The
reference's unpaired 32/64-query kernel (``_block_sparse_fwd``) is not rebuilt:
this package has one native attention kernel, the paired one.
``sparse_attention`` keeps the reference's operator (``sparse_kernel.py:
253-339``: signature, checks, messages) and computes the same masked attention
with that kernel: the 64-query rows are paired once per table on the device.
"""

from __future__ import annotations

import math
from numbers import Integral, Real

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


def _check_inputs(q, k, v, kv_indices, kv_counts, global_tokens, block_size, out):
    """Host checks of ``sparse_attention`` (``sparse_kernel.py:188-250``: same
    exception types and messages); no device work."""
    if q.ndim != 4 or k.shape != q.shape or v.shape != q.shape or any(size <= 0 for size in q.shape):
        raise ValueError("Q/K/V must have equal, nonempty [B,H,N,D] shapes")
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("Q/K/V must share FP16 or BF16 dtype")
    if not q.is_cuda or k.device != q.device or v.device != q.device:
        raise ValueError("Q/K/V must be on one CUDA device")
    if torch.is_grad_enabled() and any(x.requires_grad for x in (q, k, v)):
        raise ValueError("sparse_attention is inference-only; disable autograd before calling")
    if q.shape[-1] not in (64, 128) or any(x.stride(-1) != 1 for x in (q, k, v)):
        raise ValueError("D must be64 or128 and contiguous; outer strides may differ")
    if any(any(st <= 0 for st in x.stride()[:3]) for x in (q, k, v)):
        raise ValueError("Q/K/V outer strides must be positive")
    if any(isinstance(x, bool) or not isinstance(x, Integral) for x in (global_tokens, block_size)):
        raise TypeError("global_tokens and block_size must be integers")
    n = q.shape[-2]
    if block_size != 64 or n % block_size or global_tokens % block_size or not 0 <= global_tokens < n:
        raise ValueError("N and global_tokens must align to64, with ordinary queries remaining")
    rows = (n - global_tokens) // block_size
    if kv_indices.ndim != 2 or kv_indices.shape[0] != rows or kv_indices.shape[1] < 1 or kv_counts.shape != (rows,):
        raise ValueError("Metadata shape does not match the ordinary query partition")
    if any(x.device != q.device or x.dtype != torch.int32 or not x.is_contiguous() for x in (kv_indices, kv_counts)):
        raise ValueError("Metadata must be cached contiguous CUDA int32 tensors on the Q device")
    if out is not None:
        if out.shape != q.shape or out.dtype != q.dtype or out.device != q.device or out.stride(-1) != 1:
            raise ValueError("Provided output must match Q shape/dtype/device with contiguous last dimension")
        if any(st <= 0 for st in out.stride()) or not _non_overlapping_strides(out):
            raise ValueError("Provided output must have positive, non-overlapping strides")
        if torch.is_grad_enabled() and out.requires_grad:
            raise ValueError("An inference output cannot require gradients")
        lo, hi = _tensor_byte_span(out)
        for t in (q, k, v, kv_indices, kv_counts):
            a, b = _tensor_byte_span(t)
            if lo < b and a < hi:
                raise ValueError("Provided output must not alias Q/K/V or metadata storage")


_paired_rows_cache = {}


def _paired_rows(kv_indices, kv_counts, tokens, global_tokens):
    """The paired form of a 64-query table (``pair_metadata``), once per table:
    cached with the source tensors, keyed by storage, version counters and
    shape (tables made under inference mode have no version counter and are
    paired on every call)."""
    from .paired_metadata import pair_metadata

    src = (kv_indices, kv_counts)
    key = None
    if not any(x.is_inference() for x in src):
        key = (tokens, global_tokens) + tuple((x.data_ptr(), x._version, tuple(x.shape)) for x in src)
        hit = _paired_rows_cache.get(key)
        if hit is not None:
            return hit[1]
    meta = pair_metadata(kv_indices, kv_counts, tokens=tokens, global_tokens=global_tokens, key_block_size=64)
    if key is not None:
        if len(_paired_rows_cache) >= 16:
            _paired_rows_cache.pop(next(iter(_paired_rows_cache)))
        _paired_rows_cache[key] = (src, meta)
    return meta


def sparse_attention(q, k, v, kv_indices, kv_counts, global_tokens=768, block_size=64, *, global_strategy="flash",
                     query_block_size=64, num_warps=4, num_stages=2, scale=None, out=None):
    """The reference's block-sparse operator (``sparse_kernel.py:253-339``):
    exact attention of the 64-query rows' block lists (global-prefix queries see
    every key), in Q's shape and dtype.  Both ``global_strategy`` values and the
    tuning arguments are validated and then run the one native path: the rows
    paired on the device once per table (which also validates them, one
    synchronisation), then the sm_100a paired kernel (``paired_attention``).
    Pairing needs N and ``global_tokens`` to be multiples of 128, as every FLUX
    resolution gives."""
    _check_inputs(q, k, v, kv_indices, kv_counts, global_tokens, block_size, out)
    if global_strategy not in ("flash", "triton"):
        raise ValueError("global_strategy must be flash or triton")
    if any(isinstance(x, bool) or not isinstance(x, Integral) for x in (query_block_size, num_warps, num_stages)):
        raise TypeError("Kernel tuning arguments must be integers")
    if query_block_size not in (32, 64) or num_warps not in (4, 8) or num_stages not in (1, 2, 3, 4):
        raise ValueError("Supported tuning: query_block_size32/64, warps4/8, stages1..4")
    if scale is not None and (isinstance(scale, bool) or not isinstance(scale, Real)):
        raise TypeError("scale must be a real Python/NumPy scalar, never a tensor")
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    if not math.isfinite(scale) or scale <= 0:
        raise ValueError("Softmax scale must be positive and finite")
    n, global_tokens = q.shape[-2], int(global_tokens)
    if n % 128 or global_tokens % 128:
        raise NotImplementedError("sparse_attention runs the paired kernel: N and global_tokens must be multiples of 128")
    from .paired_kernel import paired_attention

    meta = _paired_rows(kv_indices, kv_counts, n, global_tokens)
    return paired_attention(q, k, v, meta, scale=scale, out=out)
