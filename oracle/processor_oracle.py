"""CPU restatement of the FLUX processor's Q/K/V preparation (test infrastructure).

Checker for ``hb_norm_rope_pack`` / ``hilberta_b200.prep``; only tests, smoke()
and bench.py's CPU legs use it.

The steps are hilberta/flux_adapter.py:280-298.  The arithmetic of ``norm_q`` /
``norm_k`` (RMSNorm) and of ``apply_rotary_emb`` lives in diffusers 0.36.0
(pinned by the reference's requirements, absent from this image and from the
reference tree), restated here from its published algorithm, one tensor op per
step, in the order and dtypes those ops use:

  RMSNorm (elementwise affine, 16-bit weight):
    v = mean(x.float() ** 2 over D); y = (x * rsqrt(v + eps)).to(x.dtype); y = y * weight
  apply_rotary_emb (real cos/sin [S, D], pairs interleaved, sequence dim 1):
    (x_re, x_im) = x.reshape(..., D/2, 2).unbind(-1); x_rot = stack([-x_im, x_re], -1).flatten(-2)
    out = (x.float() * cos + x_rot.float() * sin).to(x.dtype)

Parity is unpinned against diffusers itself (it cannot be imported here); the
reference's own checks at this boundary (tests/test_adapter.py) need it too.
"""

from __future__ import annotations

import torch


def rms_norm(x: torch.Tensor, weight: torch.Tensor | None, eps: float) -> torch.Tensor:
    """x [..., D] 16-bit -> same shape and dtype."""
    var = x.to(torch.float32).pow(2).mean(-1, keepdim=True)
    y = x * torch.rsqrt(var + eps)  # 16-bit * fp32 -> fp32
    if weight is None:
        return y.to(x.dtype)
    y = y.to(weight.dtype)
    return y * weight  # 16-bit product, rounded once


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, S, H, D]; cos/sin fp32 [S, D]."""
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    re, im = x.reshape(*x.shape[:-1], -1, 2).unbind(-1)
    rot = torch.stack([-im, re], dim=-1).flatten(3)
    return (x.float() * c + rot.float() * s).to(x.dtype)


def norm_rope_pack(txt, img, *, heads, weight_txt=None, weight_img=None, eps=1e-6, cos=None, sin=None,
                   image_rows=None):
    """[B, T, H*D] + [B, n, H*D] -> [B, T+n, H, D], the processor's order of ops."""
    parts = []
    if txt is not None:
        t = txt.unflatten(-1, (heads, -1))
        parts.append(rms_norm(t, weight_txt, eps) if weight_txt is not None else t)
    if img is not None:
        i = img.unflatten(-1, (heads, -1))
        i = rms_norm(i, weight_img, eps) if weight_img is not None else i
        if image_rows is not None:  # image token j -> position image_rows[j]
            placed = torch.empty_like(i)
            placed[:, image_rows.long()] = i
            i = placed
        parts.append(i)
    x = torch.cat(parts, dim=1)
    if cos is not None:
        x = apply_rope(x, cos, sin)
    return x
