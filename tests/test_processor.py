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


def test_rms_norm_restatement_against_torch_rms_norm():
    """The oracle's RMSNorm (diffusers' op order: fp32 mean of squares, x * rsqrt,
    rounded to 16 bits, times the 16-bit weight) against torch's own rms_norm for
    the normalisation: equal up to the last-bit effect of the reduction order."""
    from oracle import processor_oracle as po

    g = torch.Generator().manual_seed(4)
    x = (torch.randn(2, 96, 4, 128, generator=g) * 3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    want = torch.nn.functional.rms_norm(x.float(), (128,), eps=1e-6).to(torch.bfloat16) * w
    got = po.rms_norm(x, w, 1e-6)
    d = (got.view(torch.int16).to(torch.int32) - want.view(torch.int16).to(torch.int32)).abs()
    assert int(d.max()) <= 1 and float((d > 0).float().mean()) < 0.01
