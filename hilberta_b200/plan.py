"""Static HilbertA block plans built by the CUDA metadata builder.

Same dataclasses, fields and methods as ``hilberta/plan.py:17-111`` so code that
consumes an ``AttentionPlan`` works unchanged.  The physical token stream is
[text, shared image blocks, remaining image blocks]; tile membership and bridge
tie-breaking use the ORIGINAL composite-Hilbert ordering.  Construction runs on
the device (``hb_plan_build``) and returns CPU tensors, like the reference.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, replace

import torch

from . import _lib


@dataclass(frozen=True)
class PhasePlan:
    offset: int
    kv_indices: torch.Tensor
    kv_counts: torch.Tensor
    bridge_original_blocks: torch.Tensor

    def to(self, device):
        return replace(
            self,
            kv_indices=self.kv_indices.to(device),
            kv_counts=self.kv_counts.to(device),
            bridge_original_blocks=self.bridge_original_blocks.to(device),
        )


@dataclass(frozen=True)
class AttentionPlan:
    grid_size: int
    tile_count: int
    text_tokens: int
    shared_tokens: int
    block_size: int
    image_order: torch.Tensor
    inverse_image_order: torch.Tensor
    original_order: torch.Tensor
    physical_original_blocks: torch.Tensor
    phases: tuple
    bridge: bool
    full: bool = False

    @property
    def image_tokens(self):
        return self.grid_size**2

    @property
    def global_tokens(self):
        return self.text_tokens + self.shared_tokens

    @property
    def total_tokens(self):
        return self.text_tokens + self.image_tokens

    def to(self, device):
        return replace(
            self,
            image_order=self.image_order.to(device),
            inverse_image_order=self.inverse_image_order.to(device),
            original_order=self.original_order.to(device),
            physical_original_blocks=self.physical_original_blocks.to(device),
            phases=tuple(p.to(device) for p in self.phases),
        )

    def dense_mask(self, phase, device=None):
        """Explicit physical-identity bool mask [N, N], correctness only
        (``plan.py:70-84``); expanded on the GPU by ``hb_dense_mask``."""
        p = self.phases[phase % 4]
        device = p.kv_indices.device if device is None else device
        return dense_block_mask(
            p.kv_indices, p.kv_counts, self.total_tokens, self.global_tokens, self.block_size
        ).to(device)

    def manifest(self):
        """Same dictionary as ``plan.py:86-111``."""
        glob = self.global_tokens // self.block_size
        return dict(
            grid_size=self.grid_size,
            tile_count=self.tile_count,
            text_tokens=self.text_tokens,
            shared_tokens=self.shared_tokens,
            block_size=self.block_size,
            bridge=self.bridge,
            full=self.full,
            image_order_sha256=hashlib.sha256(self.image_order.cpu().numpy().tobytes()).hexdigest(),
            physical_original_blocks=self.physical_original_blocks.cpu().tolist(),
            phases=[
                dict(
                    offset=p.offset,
                    kv_count_min=int(p.kv_counts.min()),
                    kv_count_max=int(p.kv_counts.max()),
                    directed_entries=(glob * (self.total_tokens // self.block_size) + int(p.kv_counts.sum()))
                    * self.block_size**2,
                    bridge_original_blocks=p.bridge_original_blocks.cpu().tolist(),
                )
                for p in self.phases
            ],
        )


def dense_block_mask(kv_indices, kv_counts, tokens, global_tokens, block_size, device=None):
    """[tokens, tokens] bool: rows < global all True, ordinary rows their blocks."""
    dev = _lib.require_cuda(device if device is not None else (kv_indices.device if kv_indices.is_cuda else None))
    ids = kv_indices.to(dev, torch.int32).contiguous()
    cnt = kv_counts.to(dev, torch.int32).contiguous()
    mask = torch.empty(tokens, tokens, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.lib().hb_dense_mask(
            _lib.ptr(ids), ids.shape[1] if ids.ndim == 2 else 0, _lib.ptr(cnt), int(cnt.numel()), int(tokens),
            int(global_tokens), int(block_size), _lib.ptr(mask), _lib.stream_ptr(dev)
        )
    _lib.check(rc, "hb_dense_mask")
    return mask.bool().cpu()


def _check_positive(**values):
    for name, value in values.items():
        if isinstance(value, bool) or int(value) != value or value <= 0:
            raise ValueError(f"{name} must be a positive integer")


def _build(tile_count, grid_size, text_tokens, shared, bridge_k, reciprocal, block_size, device=None):
    """Run ``hb_plan_build`` and return CPU plan tensors."""
    dims = _lib.PlanDims()
    rc = _lib.lib().hb_plan_dims(int(grid_size), int(tile_count), int(text_tokens), int(block_size), int(bool(shared)),
                                 _lib.ctypes.byref(dims))
    if rc == _lib.HB_ERR_ARG:
        raise ValueError("grid_size must be a power of two >= 8")
    if rc == _lib.HB_ERR_ALIGN:
        raise ValueError("Tile quarter offsets and text prefix must be block aligned")
    if rc == _lib.HB_ERR_SHARED:
        raise ValueError("Shared square must be a union of complete original blocks")
    _lib.check(rc, "hb_plan_dims")
    dev = _lib.require_cuda(device)
    n, nb, rows, cap = dims.image_tokens, dims.image_blocks, dims.rows, dims.row_capacity
    kout = max(1, int(bridge_k))
    i64 = dict(dtype=torch.int64, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    image_order, inverse, original = (torch.empty(n, **i64) for _ in range(3))
    packed = torch.empty(nb, **i64)
    kv = torch.empty(4, rows, cap, **i32)
    counts = torch.empty(4, rows, **i32)
    bridge = torch.empty(4, nb, kout, **i64)
    info = torch.zeros(8, **i32)
    ws = torch.empty(int(dims.workspace_bytes), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.lib().hb_plan_build(
            int(grid_size), int(tile_count), int(text_tokens), int(block_size), int(bool(shared)), int(bridge_k),
            int(reciprocal), _lib.ptr(image_order), _lib.ptr(inverse), _lib.ptr(original), _lib.ptr(packed),
            _lib.ptr(kv), _lib.ptr(counts), _lib.ptr(bridge), _lib.ptr(info), _lib.ptr(ws), ws.numel(),
            _lib.stream_ptr(dev),
        )
        _lib.check(rc, "hb_plan_build")
        info_h = info.cpu().tolist()  # synchronises: setup-time only
    if info_h[0] == _lib.HB_ERR_SHARED:
        raise ValueError("Shared square must be a union of complete original blocks")
    if info_h[0] == _lib.HB_ERR_CROSS:
        raise AssertionError("A physical block crosses a tile boundary")
    _lib.check(info_h[0], "hb_plan_build (device)")
    width = n // tile_count
    phases = []
    for ph in range(4):
        w = info_h[2 + ph]
        phases.append(
            (
                (0, width // 4, width // 2, 3 * width // 4)[ph],
                kv[ph, :, :w].contiguous().cpu(),
                counts[ph].cpu(),
                bridge[ph].cpu(),
            )
        )
    return dict(
        image_order=image_order.cpu(),
        inverse_image_order=inverse.cpu(),
        original_order=original.cpu(),
        physical_original_blocks=packed.cpu(),
        shared_tokens=int(info_h[1]) * int(block_size),
        phases=phases,
    )


def build_plan(tile_count=4, grid_size=64, text_tokens=512, shared=True, bridge=True, block_size=64, *, device=None):
    """``hilberta/plan.py:114-197`` on the device: composite order, shared packing,
    4 sliding tile phases, per-row sorted block lists, optional K=1 bridge."""
    _check_positive(tile_count=tile_count, grid_size=grid_size, text_tokens=text_tokens, block_size=block_size)
    tile_count, grid_size, text_tokens, block_size = map(int, (tile_count, grid_size, text_tokens, block_size))
    if grid_size < 8 or grid_size & (grid_size - 1):
        raise ValueError("grid_size must be a power of two >= 8")
    r = _build(tile_count, grid_size, text_tokens, shared, 1 if bridge else 0, 0, block_size, device)
    phases = tuple(PhasePlan(off, ids, cnt, br[:, 0].contiguous()) for off, ids, cnt, br in r["phases"])
    return AttentionPlan(
        grid_size,
        tile_count,
        text_tokens,
        r["shared_tokens"],
        block_size,
        r["image_order"],
        r["inverse_image_order"],
        r["original_order"],
        r["physical_original_blocks"],
        phases,
        bool(bridge),
    )


def full_attention_plan(plan):
    """Same persistent layout, all connections: permutation-equivalence gate
    (``plan.py:200-212``)."""
    nb = plan.total_tokens // plan.block_size
    nq = (plan.total_tokens - plan.global_tokens) // plan.block_size
    ids = torch.arange(nb, dtype=torch.int32).repeat(nq, 1)
    counts = torch.full((nq,), nb, dtype=torch.int32)
    return replace(
        plan,
        phases=tuple(replace(p, kv_indices=ids.clone(), kv_counts=counts.clone()) for p in plan.phases),
        full=True,
    )
