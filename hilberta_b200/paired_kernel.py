"""Exact Q128 paired block-sparse attention (API of ``hilberta/paired_kernel.py:97-205``).

``paired_attention`` keeps the reference signature, argument meaning and host
checks (same exception types and messages) and launches the sm_100a kernel of
``hb_paired_fwd`` on the current stream.  Both ``global_strategy`` values run
the single native launch (global rows are handled in-kernel); ``num_warps`` and
``num_stages`` are validated and otherwise ignored.  No host<->device
transfer, no synchronisation, no CPU path.
"""

from __future__ import annotations

import ctypes
import math
from numbers import Integral, Real

import torch

from . import _lib
from .sparse_kernel import _non_overlapping_strides, _tensor_byte_span

LOG2E = 1.4426950408889634

_workspaces: dict = {}


def _workspace(device: torch.device, stream_handle: int, nbytes: int) -> torch.Tensor:
    """Per-(device, stream) scheduler words and split-row partials: zeroed when
    (re)allocated, self-resetting after; grown when a call needs more."""
    key = (device.index, stream_handle)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() * 4 < nbytes:
        n = max(64, -(-max(nbytes, _lib.lib().hb_fwd_workspace_bytes()) // 4))
        if ws is not None:
            torch.cuda.current_stream(device).synchronize()  # the old buffer may still be in use
        with torch.inference_mode(False):  # a normal tensor: device_status clears it in place
            ws = torch.zeros(n, dtype=torch.int32, device=device)
        _workspaces[key] = ws
    return ws


def device_status(device=None, *, clear=True) -> int:
    """OR of the HB_DEV_* bits the kernel reported on `device` (synchronises).

    With ``clear``, resets the status word; a workspace whose launch gave up on a
    wait (HB_DEV_TIMEOUT) may hold stale scheduler words and is zeroed whole."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    bits = 0
    for (index, _), ws in _workspaces.items():
        if index == dev.index:
            word = int(ws[2].item())
            bits |= word
            if clear:
                (ws if word & _lib.HB_DEV_TIMEOUT else ws[2]).zero_()
    return bits


def _launch(q, k, v, out, metadata, N, G, scale, row_map=None):
    """The one native call of the attention path."""
    dev = q.device
    stream = torch.cuda.current_stream(dev)
    B, H, _, D = q.shape
    lib = _lib.lib()
    ws = _workspace(dev, stream.cuda_stream, lib.hb_fwd_workspace_bytes_for(B, H, N, G, D))
    strides = (ctypes.c_int64 * 12)(*q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *out.stride()[:3])
    rc = lib.hb_paired_fwd(
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), strides, B, H, N, D, G,
        int(metadata.kv_indices.shape[1]), int(metadata.key_block_size),
        _lib.ptr(metadata.kv_indices), _lib.ptr(metadata.kv_flags), _lib.ptr(metadata.kv_counts),
        float(scale * LOG2E), 1 if q.dtype == torch.bfloat16 else 0, _lib.ptr(row_map), _lib.ptr(ws),
        ws.numel() * 4, ctypes.c_void_p(stream.cuda_stream),
    )
    if rc == _lib.HB_ERR_TMA:
        raise ValueError("Q/K/V need 16-byte aligned base pointers and strides for TMA tiles")
    if rc == _lib.HB_ERR_UNSUPPORTED:
        raise NotImplementedError(f"paired_attention: {_lib.status_text(rc)} (key_block_size 64, D 64/128)")
    _lib.check(rc, "hb_paired_fwd")


def _launch_allgather(q, k, v, full, metadata, N, G, scale, peers):
    """hb_paired_fwd_allgather: `full` is this rank's [B, H_all, N, D] view (its
    strides describe every rank's output); `peers` an _lib.PeerOut."""
    dev = q.device
    stream = torch.cuda.current_stream(dev)
    B, H, _, D = q.shape
    lib = _lib.lib()
    ws = _workspace(dev, stream.cuda_stream, lib.hb_fwd_workspace_bytes_for(B, H, N, G, D))
    strides = (ctypes.c_int64 * 12)(*q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *full.stride()[:3])
    rc = lib.hb_paired_fwd_allgather(
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), strides, B, H, N, D, G,
        int(metadata.kv_indices.shape[1]), int(metadata.key_block_size),
        _lib.ptr(metadata.kv_indices), _lib.ptr(metadata.kv_flags), _lib.ptr(metadata.kv_counts),
        float(scale * LOG2E), 1 if q.dtype == torch.bfloat16 else 0, ctypes.byref(peers), _lib.ptr(ws),
        ws.numel() * 4, ctypes.c_void_p(stream.cuda_stream),
    )
    if rc == _lib.HB_ERR_TMA:
        raise ValueError("Q/K/V need 16-byte aligned base pointers and strides for TMA tiles")
    _lib.check(rc, "hb_paired_fwd_allgather")


def token_order_map(plan, device) -> torch.Tensor:
    """Physical -> raster row map of a plan for ``paired_attention(token_order=...)``:
    text rows first (identity), then ``text_tokens + image_order`` (plan.py:147)."""
    t = int(plan.text_tokens)
    order = torch.as_tensor(plan.image_order).to(torch.int64)
    rows = torch.cat([torch.arange(t, dtype=torch.int64), t + order.cpu()])
    return rows.to(torch.int32).to(device).contiguous()


def paired_attention(
    q, k, v, metadata, *, global_strategy="flash", num_warps=4, num_stages=2, scale=None, out=None, token_order=None
):
    """Exact inference; pair metadata must be validated on CPU before transfer.

    Q/K/V ``[B,H,N,D]`` (D 64 or 128, contiguous D, any positive outer strides,
    e.g. BNHD storage viewed as BHND), fp16/bf16.  Returns ``out`` (allocated
    with ``torch.empty_like(q)`` when not given, preserving q's storage order).

    ``token_order`` (extension, keyword only): int32 CUDA tensor [N] mapping each
    physical token of the metadata's layout to its row in q/k/v/out, e.g.
    ``token_order_map(plan, device)`` for tensors kept in raster order; the
    kernel then gathers rows while loading and scatters output rows, replacing
    the reference's separate reorder pass (sampling_layout.py:88-116).
    """
    N, G, scale = _check_inputs(q, k, v, metadata, global_strategy, num_warps, num_stages, scale)
    if out is not None:
        if out.shape != q.shape or out.dtype != q.dtype or out.device != q.device or out.stride(-1) != 1:
            raise ValueError("Output must match Q shape/dtype/device with contiguous D")
        if any(s <= 0 for s in out.stride()) or not _non_overlapping_strides(out):
            raise ValueError("Positive non-overlapping output strides required")
        if torch.is_grad_enabled() and out.requires_grad:
            raise ValueError("Inference output cannot require gradients")
        begin, end = _tensor_byte_span(out)
        for x in (q, k, v, metadata.kv_indices, metadata.kv_flags, metadata.kv_counts):
            first, last = _tensor_byte_span(x)
            if begin < last and first < end:
                raise ValueError("Output cannot alias inputs or metadata")
    else:
        out = torch.empty_like(q)
    if token_order is not None:
        if (
            not isinstance(token_order, torch.Tensor)
            or token_order.dtype != torch.int32
            or token_order.device != q.device
            or token_order.shape != (N,)
            or not token_order.is_contiguous()
        ):
            raise ValueError("token_order must be a contiguous int32 [N] tensor on the Q device")
        if any(s % q.shape[-1] for x in (q, k, v) for s in x.stride()[:3]):
            raise ValueError("token_order needs Q/K/V outer strides that are multiples of D")
    _launch(q, k, v, out, metadata, N, G, scale, token_order)
    return out


def _check_inputs(q, k, v, metadata, global_strategy, num_warps, num_stages, scale):
    """The reference's host checks of Q/K/V, metadata, tuning and scale
    (paired_kernel.py:106-152); returns (N, G, scale)."""
    if q.ndim != 4 or k.shape != q.shape or v.shape != q.shape or any(x <= 0 for x in q.shape):
        raise ValueError("Equal nonempty B,H,N,D Q/K/V required")
    if q.shape[-1] not in (64, 128) or any(x.stride(-1) != 1 for x in (q, k, v)):
        raise ValueError("D64 or128 must be contiguous")
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("Q/K/V must share BF16/FP16 dtype")
    if not q.is_cuda or k.device != q.device or v.device != q.device:
        raise ValueError("Q/K/V must be on the same CUDA device")
    if any(any(s <= 0 for s in x.stride()[:3]) for x in (q, k, v)):
        raise ValueError("Positive Q/K/V outer strides required")
    if torch.is_grad_enabled() and any(x.requires_grad for x in (q, k, v)):
        raise ValueError("Inference only; disable autograd")
    for name in ("tokens", "global_tokens", "key_block_size"):
        value = getattr(metadata, name)
        if isinstance(value, bool) or not isinstance(value, Integral):
            raise TypeError("Integer metadata shape fields required")
    N, G = metadata.tokens, metadata.global_tokens
    if q.shape[-2] != N or G % 128 or N % 128 or not 0 <= G < N or metadata.key_block_size not in (64, 128):
        raise ValueError("Metadata/token shape mismatch or invalid128-token alignment")
    rows = (N - G) // 128
    if metadata.kv_indices.ndim != 2 or metadata.kv_indices.shape[0] != rows or metadata.kv_indices.shape[1] < 1:
        raise ValueError("Paired index shape must match ordinary query pairs")
    if metadata.kv_flags.shape != metadata.kv_indices.shape or metadata.kv_counts.shape != (rows,):
        raise ValueError("Paired flag/count shape mismatch")
    for x in (metadata.kv_indices, metadata.kv_flags, metadata.kv_counts):
        if x.device != q.device or x.dtype != torch.int32 or not x.is_contiguous():
            raise ValueError("Cached CUDA contiguous int32 metadata required")
    if global_strategy not in ("flash", "triton"):
        raise ValueError("Invalid global strategy")
    if any(isinstance(x, bool) or not isinstance(x, Integral) for x in (num_warps, num_stages)):
        raise TypeError("Integer launch tuning required")
    if num_warps not in (4, 8) or num_stages not in (1, 2, 3, 4):
        raise ValueError("Invalid launch tuning")
    if scale is not None and (isinstance(scale, bool) or not isinstance(scale, Real)):
        raise TypeError("scale must be a real scalar, never a tensor")
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    if not math.isfinite(scale) or scale <= 0:
        raise ValueError("Positive finite scale required")
    return N, G, scale
