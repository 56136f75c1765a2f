"""Pin of the processor-maths restatement against diffusers itself.

The FLUX processor's steps between the projections and the attention
(hilberta/flux_adapter.py:280-295) use diffusers 0.36.0's ``RMSNorm`` and
``apply_rotary_emb``.  ``oracle/processor_oracle.py`` restates them from the
published algorithm, and ``hb_norm_rope_pack`` is tested against that
restatement (tests/test_prep_gpu.py).  Where diffusers can be imported, this
file checks the restatement and the kernel against diffusers' own functions on
the same inputs: the restatement bit for bit, the kernel within the 2-ulp bound
of its normalisation order.  diffusers is absent from this image (no network to
install it), so here these tests skip with that reason and the restatement stays
unpinned against diffusers.
"""

from __future__ import annotations

import pytest
import torch

from oracle import processor_oracle as po

diffusers = pytest.importorskip("diffusers", reason="diffusers (the reference pins 0.36.0) is not installed in this image")

pytestmark = pytest.mark.gpu


def _inputs(B=1, S=192, H=4, D=128, seed=3, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(B, S, H, D, generator=g) * 3).to(dtype)
    w = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    ang = torch.rand(S, D // 2, generator=g, dtype=torch.float64) * 6.28
    cos = torch.cos(ang).repeat_interleave(2, dim=1).float()
    sin = torch.sin(ang).repeat_interleave(2, dim=1).float()
    return x, w, cos, sin


def test_rms_norm_restatement_equals_diffusers():
    from diffusers.models.normalization import RMSNorm

    x, w, _, _ = _inputs()
    norm = RMSNorm(x.shape[-1], eps=1e-6, elementwise_affine=True).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(w)
        want = norm(x)
    assert torch.equal(po.rms_norm(x, w, 1e-6), want)


def test_rotary_restatement_equals_diffusers():
    from diffusers.models.embeddings import apply_rotary_emb

    x, _, cos, sin = _inputs()
    want = apply_rotary_emb(x, (cos, sin), sequence_dim=1)
    assert torch.equal(po.apply_rope(x, cos, sin), want)


def test_kernel_against_diffusers_steps():
    from diffusers.models.embeddings import apply_rotary_emb
    from diffusers.models.normalization import RMSNorm

    from hilberta_b200 import prep

    x, w, cos, sin = _inputs()
    B, S, H, D = x.shape
    norm = RMSNorm(D, eps=1e-6, elementwise_affine=True).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(w)
        want = apply_rotary_emb(norm(x), (cos, sin), sequence_dim=1)
    dev = torch.device("cuda", 0)
    with torch.inference_mode():
        got = prep.norm_rope_pack(None, x.flatten(2).to(dev), heads=H, weight_txt=w.to(dev), weight_img=w.to(dev), eps=1e-6,
                                  cos=cos.to(dev), sin=sin.to(dev)).cpu()
    ia, ib = got.view(torch.int16).to(torch.int32), want.view(torch.int16).to(torch.int32)
    assert int((ia - ib).abs().max()) <= 2
