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
                (ws if word & (_lib.HB_DEV_TIMEOUT | _lib.HB_DEV_SMEM_ALIGN) else ws[2]).zero_()
    return bits


_kv64_cache = {}


def _as_kv64(metadata):
    """KV64 form of a KV128 paired table (hb_expand_kv128, once per table: the
    result is cached with the source tensors, keyed by their storage and version
    counters, so an in-place edit of the table is re-expanded; tables made under
    inference mode have no version counter and are expanded on every call)."""
    if metadata.key_block_size == 64:
        return metadata
    src = (metadata.kv_indices, metadata.kv_flags, metadata.kv_counts)
    # inference tensors carry no version counter: expanded on every call instead
    key = None if any(x.is_inference() for x in src) else tuple((x.data_ptr(), x._version, tuple(x.shape)) for x in src)
    hit = _kv64_cache.get(key) if key is not None else None
    if hit is not None:
        return hit[1]
    from .paired_metadata import PairedMetadata

    rows, width = metadata.kv_indices.shape
    dev = metadata.kv_indices.device
    ids = torch.zeros(rows, 2 * width, dtype=torch.int32, device=dev)
    flags, counts = torch.zeros_like(ids), torch.zeros(rows, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.lib().hb_expand_kv128(
            _lib.ptr(metadata.kv_indices), _lib.ptr(metadata.kv_flags), width, width, _lib.ptr(metadata.kv_counts),
            rows, _lib.ptr(ids), _lib.ptr(flags), 2 * width, _lib.ptr(counts), _lib.stream_ptr(dev))
    _lib.check(rc, "hb_expand_kv128")
    meta64 = PairedMetadata(ids, flags, counts, metadata.tokens, metadata.global_tokens, 64)
    if key is not None:
        if len(_kv64_cache) >= 16:
            _kv64_cache.pop(next(iter(_kv64_cache)))
        _kv64_cache[key] = (src, meta64)  # holding `src` keeps its storage (and key) from being reused
    return meta64


def _launch(q, k, v, out, metadata, N, G, scale, row_map=None, raster=None):
    """The one native call of the attention path."""
    metadata = _as_kv64(metadata)
    dev = q.device
    stream = torch.cuda.current_stream(dev)
    B, H, _, D = q.shape
    lib = _lib.lib()
    ws = _workspace(dev, stream.cuda_stream, lib.hb_fwd_workspace_bytes_for(B, H, N, G, D))
    strides = (ctypes.c_int64 * 12)(*q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *out.stride()[:3])
    common = (
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), strides, B, H, N, D, G,
        int(metadata.kv_indices.shape[1]), int(metadata.key_block_size),
        _lib.ptr(metadata.kv_indices), _lib.ptr(metadata.kv_flags), _lib.ptr(metadata.kv_counts),
        float(scale * LOG2E), 1 if q.dtype == torch.bfloat16 else 0,
    )
    tail = (_lib.ptr(ws), ws.numel() * 4, ctypes.c_void_p(stream.cuda_stream))
    if raster is not None:
        order = _lib.RasterOrderC(raster.text_tokens, raster.grid, raster.block_origin.data_ptr())
        rc = lib.hb_paired_fwd_raster(*common, ctypes.byref(order), *tail)
    else:
        rc = lib.hb_paired_fwd(*common, _lib.ptr(row_map), *tail)
    if rc == _lib.HB_ERR_TMA:
        raise ValueError("Q/K/V need 16-byte aligned base pointers and strides for TMA tiles")
    if rc == _lib.HB_ERR_UNSUPPORTED:
        raise NotImplementedError(f"paired_attention: {_lib.status_text(rc)} (D 64/128)")
    _lib.check(rc, "hb_paired_fwd")


def _launch_allgather(q, k, v, full, metadata, N, G, scale, peers):
    """hb_paired_fwd_allgather: `full` is this rank's [B, H_all, N, D] view (its
    strides describe every rank's output); `peers` an _lib.PeerOut."""
    metadata = _as_kv64(metadata)
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


class RasterOrder:
    """Raster token layout of a plan for ``paired_attention(token_order=...)``:
    ``text_tokens`` text tokens, then the ``grid x grid`` image in row-major
    order.  ``block_origin`` (int32, on the device) holds, for each physical
    64-token image block, the image row y0*grid + x0 of the aligned 8x8 square it
    covers; the kernel loads each block as one square and writes its output rows
    back into it."""

    def __init__(self, text_tokens: int, grid: int, block_origin: torch.Tensor):
        self.text_tokens, self.grid, self.block_origin = int(text_tokens), int(grid), block_origin

    @property
    def tokens(self) -> int:
        return self.text_tokens + self.grid * self.grid

    def rows(self) -> torch.Tensor:
        """The equivalent row map for the kernel's token order: physical token p
        of block b at row-major position i of its square -> raster row."""
        o = self.block_origin.to(torch.int64)
        i = torch.arange(64, device=o.device)
        img = self.text_tokens + o[:, None] + (i // 8)[None, :] * self.grid + (i % 8)[None, :]
        return torch.cat([torch.arange(self.text_tokens, device=o.device), img.reshape(-1)]).to(torch.int32)


def raster_order(plan, device) -> RasterOrder:
    """RasterOrder of a plan; raises ValueError when a physical image block is not
    an aligned 8x8 square of the image (every plan of build_plan / bridge_k_plan
    has this property: the Hilbert walk fills aligned squares 64 cells at a time)."""
    t = int(plan.text_tokens)
    order = torch.as_tensor(plan.image_order).to(torch.int64).cpu()
    g = int(round(order.numel() ** 0.5))
    if g * g != order.numel() or g % 8 or t % 64:
        raise ValueError("raster_order needs a square image with a side divisible by 8 and a 64-aligned text prefix")
    blocks = order.view(-1, 64)
    y, x = blocks // g, blocks % g
    x0, y0 = x.min(dim=1).values, y.min(dim=1).values
    i = torch.arange(64)
    want = (y0[:, None] + i // 8) * g + x0[:, None] + i % 8
    if (x0 % 8).any() or (y0 % 8).any() or not torch.equal(blocks.sort(dim=1).values, want):
        raise ValueError("plan image blocks are not aligned 8x8 squares; use token_order_map")
    return RasterOrder(t, g, (y0 * g + x0).to(torch.int32).to(device).contiguous())


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

    ``token_order`` (extension, keyword only), for q/k/v/out kept in raster token
    order instead of the metadata's physical order, replacing the reference's
    separate reorder passes (sampling_layout.py:88-116):

    * ``raster_order(plan, device)`` (fast): each 64-token block is loaded as one
      aligned 8x8 image square and its output rows are written back into it;
    * an int32 CUDA tensor [N] mapping each physical token to its row, e.g.
      ``token_order_map(plan, device)`` (any permutation; rows are gathered four
      at a time, Q/K/V outer strides must be multiples of D).
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
    if isinstance(token_order, RasterOrder):
        bo = token_order.block_origin
        if token_order.tokens != N or bo.dtype != torch.int32 or bo.device != q.device or not bo.is_contiguous():
            raise ValueError("token_order must describe N tokens with int32 block origins on the Q device")
        if bo.shape != (token_order.grid * token_order.grid // 64,):
            raise ValueError("token_order block_origin needs one entry per 64-token image block")
        _launch(q, k, v, out, metadata, N, G, scale, raster=token_order)
        return out
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
