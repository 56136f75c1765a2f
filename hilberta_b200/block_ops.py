"""The FLUX blocks' adaLN modulation and gated residuals on the native library
(``hb_adaln_residual``), and the block-level operations the FLUX-architecture
step uses around the attention (``NativeBlockOps``).

``adaln(x, shift, scale)``              h = LayerNorm(x) * (1 + scale) + shift
``gate_residual(x, y, gate)``           x += gate * y            (in place)
``gate_residual_adaln(x, y, gate, shift, scale)``
                                        x += gate * y; h = LayerNorm(x) * (1 + scale) + shift

``x``/``y``: ``[B, S, C]`` (or ``[S, C]``) 16-bit with unit element stride;
``shift``/``scale``/``gate``: ``[B, C]`` with unit element stride (chunks of a
modulation output are fine).  LayerNorm without affine weights.
"""

from __future__ import annotations

import torch

from . import _lib

_DTYPES = {torch.float16: 0, torch.bfloat16: 1}


def _rows(t, name):
    """(pointer, row stride, B, S) of a [B, S, C] / [S, C] tensor whose rows
    are equally spaced."""
    if t.dim() == 2:
        t = t.unsqueeze(0)
    if t.dim() != 3 or t.stride(-1) != 1:
        raise ValueError(f"{name} must be [B, S, C] with a contiguous last dimension")
    B, S, _ = t.shape
    if B > 1 and S > 0 and t.stride(0) != S * t.stride(1):
        raise ValueError(f"{name} rows must be equally spaced across the batch")
    return t, t.stride(1), B, S


def _mod(m, B, C, x, name):
    if m.dim() == 1:
        m = m.unsqueeze(0)
    if m.dim() != 2 or m.shape[1] != C or m.stride(-1) != 1 or m.shape[0] not in (1, B):
        raise ValueError(f"{name} must be [B, C] with a contiguous last dimension")
    if m.dtype != x.dtype or m.device != x.device:
        raise ValueError(f"{name} must match x's dtype and device")
    if m.shape[0] == 1 and B > 1:
        raise ValueError(f"{name} must have one row per batch entry")
    return m, (m.stride(0) if B > 1 else 0)


def _call(x, y, gate, shift, scale, x_out, h_out, eps):
    if not x.is_cuda:
        raise ValueError("CUDA tensors required")
    if x.dtype not in _DTYPES:
        raise ValueError("x must be float16 or bfloat16")
    x3, x_rs, B, S = _rows(x, "x")
    C = x3.shape[-1]
    strides = {}
    mod_bs = None
    for name, m in (("gate", gate), ("shift", shift), ("scale", scale)):
        if m is not None:
            _, bs = _mod(m, B, C, x, name)
            if mod_bs is not None and bs != mod_bs:
                raise ValueError("gate, shift and scale must share one batch stride")
            mod_bs = bs
    for name, t in (("y", y), ("x_out", x_out), ("h_out", h_out)):
        if t is not None:
            if t.shape != x.shape or t.dtype != x.dtype or t.device != x.device:
                raise ValueError(f"{name} must match x's shape, dtype and device")
            strides[name] = _rows(t, name)[1]
    dev = x.device
    with torch.cuda.device(dev):
        rc = _lib.lib().hb_adaln_residual(
            _lib.ptr(x), x_rs, _lib.ptr(y) if y is not None else None, strides.get("y", 0),
            _lib.ptr(gate) if gate is not None else None, _lib.ptr(shift) if shift is not None else None,
            _lib.ptr(scale) if scale is not None else None, mod_bs or 0,
            _lib.ptr(x_out) if x_out is not None else None, strides.get("x_out", 0),
            _lib.ptr(h_out) if h_out is not None else None, strides.get("h_out", 0),
            B * S, S, C, float(eps), _DTYPES[x.dtype], _lib.stream_ptr(dev))
    _lib.check(rc, "hb_adaln_residual")


def adaln(x, shift, scale, eps=1e-6, out=None):
    h = torch.empty_like(x, memory_format=torch.contiguous_format) if out is None else out
    _call(x, None, None, shift, scale, None, h, eps)
    return h


def gate_residual(x, y, gate):
    _call(x, y, gate, None, None, x, None, 0.0)
    return x


def gate_residual_adaln(x, y, gate, shift, scale, eps=1e-6, out=None):
    h = torch.empty_like(x, memory_format=torch.contiguous_format) if out is None else out
    _call(x, y, gate, shift, scale, x, h, eps)
    return x, h


class NativeBlockOps:
    """Block-level operations of the FLUX-architecture step on CUDA tensors:
    the fused adaLN kernels above, MLP input projections with the tanh-GELU in
    the cuBLASLt epilogue, and the single-stream output projection over
    [attention | MLP] as two accumulating GEMMs instead of a concatenation."""

    @staticmethod
    def modulate(x, shift, scale):
        return adaln(x, shift, scale)

    @staticmethod
    def gate_add(x, y, gate):
        return gate_residual(x, y, gate)

    @staticmethod
    def gate_add_modulate(x, y, gate, shift, scale):
        return gate_residual_adaln(x, y, gate, shift, scale)

    @staticmethod
    def linear_gelu(x, weight, bias):
        """tanh-GELU(x @ weight^T + bias) with the activation in the GEMM epilogue."""
        y = torch._addmm_activation(bias, x.reshape(-1, x.shape[-1]), weight.t(), use_gelu=True)
        return y.view(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def joined_linear(a, m, weight_a, weight_m, bias, out=None):
        """[a | m] @ [weight_a | weight_m]^T (+ bias) without materialising
        [a | m]: two GEMMs, the second accumulating into the first's output
        (``out``, rows x out-features, if given)."""
        a2, m2 = a.reshape(-1, a.shape[-1]), m.reshape(-1, m.shape[-1])
        if out is None:
            out = torch.empty(a2.shape[0], weight_a.shape[0], dtype=a.dtype, device=a.device)
        if bias is None:
            torch.mm(a2, weight_a.t(), out=out)
        else:
            torch.addmm(bias, a2, weight_a.t(), out=out)
        out.addmm_(m2, weight_m.t())
        return out.view(*a.shape[:-1], weight_a.shape[0])


__all__ = ["adaln", "gate_residual", "gate_residual_adaln", "NativeBlockOps"]
