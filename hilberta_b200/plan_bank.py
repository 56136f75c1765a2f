"""Validated, device-cached plan metadata for the attention processors.

API of the reference adapter's ``_PlanBank`` (hilberta/flux_adapter.py:26-146):
the same constructor checks in the same order with the same messages, the same
``on_device`` / ``dense_mask`` / ``clear`` methods and ``info`` counters.  The
per-row metadata checks (ids in range and unique, the global prefix present)
run in the device validator (``hb_validate_metadata``) instead of a Python loop
over rows; paired metadata is built on the device too.  ``on_device`` also
caches the plan's raster layout (``paired_kernel.raster_order``) when its
blocks are aligned image squares, for callers that keep tokens in raster order.
"""

from __future__ import annotations

import hashlib

import torch

from . import _lib
from .paired_metadata import pair_metadata
from .paired_kernel import raster_order
from .sparse_kernel import explicit_mask


class PlanBank:
    """Validate and copy immutable CPU metadata once; cache device copies."""

    def __init__(self, plan, info=None, *, backend="paired", device=None):
        self.image_tokens = int(plan.image_tokens)
        self.text_tokens = int(plan.text_tokens)
        self.shared_tokens = int(plan.shared_tokens)
        self.global_tokens = int(plan.global_tokens)
        self.total_tokens = int(plan.total_tokens)
        self.block_size = int(plan.block_size)
        self.info = {"backend": backend} if info is None else info
        self.info.setdefault("backend", backend)
        if self.image_tokens <= 0 or self.text_tokens <= 0 or not 0 <= self.shared_tokens <= self.image_tokens:
            raise ValueError("Plan requires nonempty image/text tokens and a valid shared-image count")
        if (
            self.global_tokens != self.text_tokens + self.shared_tokens
            or self.total_tokens != self.text_tokens + self.image_tokens
        ):
            raise ValueError("Plan global/total token counts are inconsistent")
        if self.block_size <= 0 or self.total_tokens % self.block_size or self.global_tokens % self.block_size:
            raise ValueError("Total tokens and global prefix must be block-aligned")
        self.order = torch.as_tensor(plan.image_order).detach().to(device="cpu", dtype=torch.int64).clone()
        self.inverse = torch.as_tensor(plan.inverse_image_order).detach().to(device="cpu", dtype=torch.int64).clone()
        expected = torch.arange(self.image_tokens)
        if self.order.shape != expected.shape or not torch.equal(self.order.sort().values, expected):
            raise ValueError("image_order must contain every image-token identity exactly once")
        if self.inverse.shape != expected.shape or not torch.equal(self.inverse[self.order], expected):
            raise ValueError("inverse_image_order is not the inverse of image_order")
        if len(plan.phases) != 4:
            raise ValueError("Exactly four phase metadata tables are required")
        query_blocks = (self.total_tokens - self.global_tokens) // self.block_size
        self.phases = []
        for phase in plan.phases:
            ids = torch.as_tensor(phase.kv_indices).detach().to(device="cpu", dtype=torch.int32).contiguous().clone()
            counts = torch.as_tensor(phase.kv_counts).detach().to(device="cpu", dtype=torch.int32).contiguous().clone()
            if ids.ndim != 2 or ids.shape[0] != query_blocks or counts.shape != (query_blocks,):
                raise ValueError("KV metadata must have one row per ordinary physical query block")
            if bool(((counts <= 0) | (counts > ids.shape[1])).any()):
                raise ValueError("KV block counts are outside their metadata width")
            self.phases.append((ids, counts))
        # per-row checks of every phase on the device, in the reference's order
        dev = _lib.require_cuda(device)
        for ids, counts in self.phases:
            self._check_rows(ids, counts, dev)
        self.paired_phases = None
        if self.info["backend"] == "paired":
            if self.block_size != 64:
                raise ValueError("Paired backend requires 64-token physical blocks")
            self.paired_phases = [
                pair_metadata(ids.to(dev), counts.to(dev), tokens=self.total_tokens,
                              global_tokens=self.global_tokens, key_block_size=64).to("cpu")
                for ids, counts in self.phases
            ]
        try:
            self._raster = raster_order(plan, "cpu") if self.block_size == 64 else None
        except ValueError:
            self._raster = None
        self.device_cache, self.mask_cache = {}, {}
        self.order_hash = hashlib.sha256(self.order.numpy().tobytes()).hexdigest()

    def _check_rows(self, ids, counts, dev):
        res = torch.empty(4, dtype=torch.int32, device=dev)
        d_ids, d_counts = ids.to(dev), counts.to(dev)
        with torch.cuda.device(dev):
            rc = _lib.lib().hb_validate_metadata(
                _lib.ptr(d_ids), ids.shape[1], ids.shape[1], _lib.ptr(d_counts), ids.shape[0],
                self.total_tokens, self.global_tokens, _lib.ptr(res), _lib.stream_ptr(dev))
            _lib.check(rc, "hb_validate_metadata")
            first = int(res[0].item())
        if first == 2**31 - 1:
            return
        code = first % 4
        if code == 1:
            raise ValueError("KV block counts are outside their metadata width")
        if code == 2:
            raise ValueError("Active KV block IDs must be valid and unique")
        raise ValueError("Every ordinary query must retain every text/shared global key block")

    def on_device(self, device):
        key = str(device)
        if key not in self.device_cache:
            # Normal tensors even when the first call runs under inference mode:
            # the caches keyed on a table's version counter (the sparse
            # backend's pairing, the KV128 expansion) skip inference tensors.
            with torch.inference_mode(False):
                self.device_cache[key] = self._device_entry(device)
            self.info["metadata_device_copies"] = len(self.device_cache)
        return self.device_cache[key]

    def _device_entry(self, device):
        entry = {
            "order": self.order.to(device, copy=True),
            "inverse": self.inverse.to(device, copy=True),
            "phases": [(ids.to(device, copy=True), counts.to(device, copy=True)) for ids, counts in self.phases],
        }
        if self.paired_phases is not None:
            entry["paired_phases"] = [p.to(device) for p in self.paired_phases]
        if self._raster is not None:
            r = self._raster
            entry["raster"] = type(r)(r.text_tokens, r.grid, r.block_origin.to(device, copy=True))
        return entry

    def dense_mask(self, phase, device):
        """Dense [N, N] boolean mask of a phase (correctness reference only),
        built from the validated sparse metadata."""
        key = (phase, str(device))
        if key not in self.mask_cache:
            ids, counts = self.phases[phase]
            dev = _lib.require_cuda(device if torch.device(device).type == "cuda" else None)
            mask = explicit_mask(ids.to(dev), counts.to(dev), tokens=self.total_tokens,
                                 global_tokens=self.global_tokens, block_size=self.block_size)
            self.mask_cache[key] = mask.to(device)
            self.info["reference_masks_prepared"] = len(self.mask_cache)
        return self.mask_cache[key]

    def clear(self):
        self.device_cache.clear()
        self.mask_cache.clear()
