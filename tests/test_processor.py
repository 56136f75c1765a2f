"""HilbertAProcessor host checks (no GPU): the reference processor's refusals
of external attention masks and of autograd (hilberta/flux_adapter.py:270-277)."""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from hilberta_b200.processor import HilbertAProcessor


def test_rejects_masks_and_autograd():
    proc = HilbertAProcessor(bank=SimpleNamespace(total_tokens=1536), layer=3)
    assert proc.phase == 3
    with pytest.raises(ValueError, match="attention masks"):
        proc(object(), torch.zeros(1, 4, 8), attention_mask=torch.ones(1))
    with torch.enable_grad(), pytest.raises(RuntimeError, match="inference-only"):
        proc.attention(object(), torch.zeros(1, 4, 8))
