"""Q/K/V preparation in front of the attention (``hb_norm_rope_pack``).

The FLUX processor (hilberta/flux_adapter.py:280-298) turns the six projections
of a double-stream block into the attention inputs:

* split each projection into heads (``unflatten(-1, (heads, -1))``);
* RMS-normalise query and key rows over the head dimension (``norm_q`` /
  ``norm_k`` for the image stream, ``norm_added_q`` / ``norm_added_k`` for the
  text stream; learned weight, eps 1e-6 in FLUX);
* concatenate text tokens first, image tokens after;
* rotate query and key by the rotary embedding (``apply_rotary_emb`` with real
  cos/sin of shape [S, D]);
* hand ``transpose(1, 2)`` views ([B, H, S, D] of [B, S, H, D] storage) to the
  attention.

``prepare_qkv`` does all of it with one pass over HBM per tensor and returns
those views, ready for ``paired_attention``.  ``image_rows`` optionally writes
image token i to token ``T + image_rows[i]`` (for instance the plan's inverse
order, giving the physical layout the plain kernel reads).  No CPU path.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return 1
    if t.dtype == torch.float16:
        return 0
    raise TypeError("16-bit (bf16/fp16) projections required")


def norm_rope_pack(txt, img, *, heads, weight_txt=None, weight_img=None, eps=1e-6, cos=None, sin=None,
                   image_rows=None, out=None):
    """One of Q/K/V: ``txt`` [B, T, heads*D] and ``img`` [B, n, heads*D] (D
    contiguous, 16-bit) -> [B, T+n, heads, D] (``out`` if given).  Weights [D]
    in the inputs' dtype (both or neither); cos/sin fp32 [T+n, D] by output
    token (both or neither)."""
    ref = img if img is not None else txt
    if ref is None or not ref.is_cuda:
        raise ValueError("CUDA projections required")
    B = ref.shape[0]
    HD = ref.shape[-1]
    if HD % heads:
        raise ValueError("projection width must split into heads")
    D = HD // heads
    T = 0 if txt is None else txt.shape[1]
    n = 0 if img is None else img.shape[1]
    for x in (txt, img):
        if x is not None and (x.ndim != 3 or x.shape[0] != B or x.shape[2] != HD or x.stride(-1) != 1
                              or x.dtype != ref.dtype or x.device != ref.device):
            raise ValueError("txt/img must be [B, tokens, heads*D] with contiguous last dim, same dtype/device")
    if (weight_txt is None) != (weight_img is None):
        raise ValueError("give both stream weights or neither")
    for w in (weight_txt, weight_img):
        if w is not None and (w.shape != (D,) or w.dtype != ref.dtype or w.device != ref.device or not w.is_contiguous()):
            raise ValueError("norm weights must be contiguous [D] in the projections' dtype")
    if (cos is None) != (sin is None):
        raise ValueError("give both cos and sin or neither")
    for c in (cos, sin):
        if c is not None and (c.shape != (T + n, D) or c.dtype != torch.float32 or c.device != ref.device
                              or not c.is_contiguous()):
            raise ValueError("cos/sin must be contiguous fp32 [T+n, D] on the projections' device")
    if image_rows is not None and (image_rows.shape != (n,) or image_rows.dtype != torch.int32
                                   or image_rows.device != ref.device or not image_rows.is_contiguous()):
        raise ValueError("image_rows must be a contiguous int32 [n] tensor on the projections' device")
    if out is None:
        out = torch.empty((B, T + n, heads, D), dtype=ref.dtype, device=ref.device)
    elif out.shape != (B, T + n, heads, D) or out.dtype != ref.dtype or out.stride(-1) != 1:
        raise ValueError("out must be [B, T+n, heads, D] with contiguous D")
    status = None
    rc = _lib.lib().hb_norm_rope_pack(
        _lib.ptr(txt), 0 if txt is None else txt.stride(0), 0 if txt is None else txt.stride(1),
        _lib.ptr(img), 0 if img is None else img.stride(0), 0 if img is None else img.stride(1),
        B, T, n, heads, D, _lib.ptr(weight_txt), _lib.ptr(weight_img), float(eps), _lib.ptr(cos), _lib.ptr(sin),
        _lib.ptr(image_rows), _lib.ptr(out), out.stride(0), out.stride(1), out.stride(2), _dtype_code(ref), status,
        ctypes.c_void_p(torch.cuda.current_stream(ref.device).cuda_stream),
    )
    if rc == _lib.HB_ERR_ALIGN:
        raise ValueError("hb_norm_rope_pack needs 16-byte aligned rows (strides multiples of 8 elements)")
    if rc == _lib.HB_ERR_UNSUPPORTED:
        raise NotImplementedError("hb_norm_rope_pack supports D 64 or 128, fp16/bf16")
    _lib.check(rc, "hb_norm_rope_pack")
    return out


def prepare_qkv(q_txt, k_txt, v_txt, q_img, k_img, v_img, *, heads, norm_q, norm_k, norm_added_q, norm_added_k,
                rotary=None, eps=1e-6, image_rows=None):
    """The processor's Q/K/V for the attention: [B, H, S, D] views of [B, S, H, D]
    storage, text tokens first.  norm_* are the [D] RMSNorm weights; rotary is
    (cos, sin), fp32 [S, D] by output token, or None."""
    cos, sin = (None, None) if rotary is None else rotary
    q = norm_rope_pack(q_txt, q_img, heads=heads, weight_txt=norm_added_q, weight_img=norm_q, eps=eps, cos=cos,
                       sin=sin, image_rows=image_rows)
    k = norm_rope_pack(k_txt, k_img, heads=heads, weight_txt=norm_added_k, weight_img=norm_k, eps=eps, cos=cos,
                       sin=sin, image_rows=image_rows)
    v = norm_rope_pack(v_txt, v_img, heads=heads, image_rows=image_rows)
    return q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
