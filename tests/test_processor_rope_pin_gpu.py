"""Pin of the rotary step against an independent implementation.

diffusers (whose ``apply_rotary_emb`` the FLUX processor calls,
hilberta/flux_adapter.py:290-291) is absent from this image, so the
restatement in ``oracle/processor_oracle.py`` cannot be checked against it.
FLUX's rotation is the interleaved ("GPT-J") convention: pair (2i, 2i+1) of
each head turned by angle theta_i of its token, out = x cos + rot(x) sin with
rot(x)_(2i, 2i+1) = (-x_(2i+1), x_2i).  flashinfer (in this image) ships a kernel
for exactly that convention (``apply_rope_with_cos_sin_cache(..., is_neox=False)``,
per-token cos/sin read from a cache indexed by position), so the restatement
and ``hb_norm_rope_pack``'s rotation are checked against it here, with FLUX's
3-axis angles.  flashinfer rounds a fused multiply-add where the restatement
(like diffusers' torch ops) rounds each product, so a 16-bit result may differ
in its last place, and by a few fp32 rounding errors where the pair's two
products cancel; the test allows exactly that, on a small fraction of
elements.  The normalisation step is checked against torch's own ``rms_norm``
on the CPU (test_processor.py).
"""

from __future__ import annotations

import pytest
import torch

from oracle import processor_oracle as po

pytestmark = pytest.mark.gpu


def _flux_angles(S, D, seed):
    """Per-token angles of FLUX's 3-axis rotary embedding (axes 16/56/56 of
    D = 128, theta 10000) for random (t, y, x) position ids."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, 128, (S, 3), generator=g).double()
    parts = []
    for axis, dim in enumerate((16, 56, 56)):
        freqs = 1.0 / (10000.0 ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
        parts.append(ids[:, axis : axis + 1] * freqs[None, :])
    ang = torch.cat(parts, dim=1)  # [S, D/2]
    assert ang.shape[1] == D // 2
    return ang


def _flashinfer_rope(x, cos_half, sin_half):
    flashinfer = pytest.importorskip("flashinfer", reason="flashinfer is not importable")
    B, S, H, D = x.shape
    cache = torch.cat([cos_half, sin_half], dim=1).float().contiguous().cuda()  # [S, D] (cos | sin)
    flat = x.reshape(B * S, H * D).cuda()
    pos = torch.arange(S, device="cuda", dtype=torch.int64).repeat(B)
    try:
        out, _ = flashinfer.rope.apply_rope_with_cos_sin_cache(pos, flat, flat.clone(), D, cache, is_neox=False)
    except Exception as e:  # its kernels are compiled on first use; no compiler or cache -> skip
        pytest.skip(f"flashinfer rope unavailable: {type(e).__name__}: {e}")
    torch.cuda.synchronize()
    return out.reshape(B, S, H, D).cpu()


def _check_close(got, want, x):
    """got equals want but for rounding: each element within one 16-bit step of
    want, or, where the pair's two products cancel, within a few fp32 rounding
    errors of their magnitudes; differing elements rare.  A wrong pairing, sign
    or angle gives errors of the order of the values themselves."""
    eps = torch.finfo(x.dtype).eps
    mag = x.float().reshape(*x.shape[:-1], -1, 2).abs().sum(-1).repeat_interleave(2, dim=-1)
    diff = (got.float() - want.float()).abs()
    assert bool((diff <= eps * want.float().abs() + 2.0**-18 * mag).all()), float(diff.max())
    assert float((got != want).float().mean()) < 0.02


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rotation_matches_flashinfer_interleaved_rope(dtype):
    B, S, H, D = 1, 640, 4, 128
    g = torch.Generator().manual_seed(11)
    x = (torch.randn(B, S, H, D, generator=g) * 2).to(dtype)
    ang = _flux_angles(S, D, seed=5)
    cos_half, sin_half = torch.cos(ang).float(), torch.sin(ang).float()
    cos, sin = cos_half.repeat_interleave(2, dim=1), sin_half.repeat_interleave(2, dim=1)
    want = _flashinfer_rope(x, cos_half, sin_half)
    # the CPU restatement (diffusers' op order)
    _check_close(po.apply_rope(x, cos, sin), want, x)
    # the kernel's rotation (no normalisation weights: rotation and packing only)
    from hilberta_b200 import prep

    dev = torch.device("cuda", 0)
    with torch.inference_mode():
        got = prep.norm_rope_pack(None, x.flatten(2).to(dev), heads=H, cos=cos.to(dev), sin=sin.to(dev)).cpu()
    _check_close(got, want, x)
