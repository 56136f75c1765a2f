"""hb_adaln_residual (hilberta_b200/block_ops.py) against fp32 references of the
FLUX blocks' adaLN-Zero steps: h = LayerNorm(x) * (1 + scale) + shift and
x += gate * y.  Each output is one rounding of an fp32 computation, so it must
lie within half a 16-bit ulp (2^-8 relative for bf16, 2^-11 for fp16) of the
fp32 reference, plus a small absolute slack for fp32 differences."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

_REL = {torch.bfloat16: 2.0**-8, torch.float16: 2.0**-11}


def _check(got, ref, dtype, slack=1e-5):
    err = (got.float() - ref).abs()
    bound = ref.abs() * _REL[dtype] * 1.01 + slack
    assert bool((err <= bound).all()), float((err - bound).max())


def _mods(B, C, dtype, g):
    m = (torch.randn(B, 6 * C, generator=g) * 0.5).to(dtype).cuda()
    return m.chunk(6, dim=-1)  # views with batch stride 6C


def _ln_ref(x, shift, scale):
    return F.layer_norm(x.float(), x.shape[-1:], eps=1e-6) * (1 + scale.float()[:, None]) + shift.float()[:, None]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("C", [256, 3072, 4096])
def test_adaln(dtype, C):
    from hilberta_b200.block_ops import adaln

    g = torch.Generator().manual_seed(C)
    x = (torch.randn(2, 333, C, generator=g) * 3 + 1).to(dtype).cuda()
    shift, scale, *_ = _mods(2, C, dtype, g)
    h = adaln(x, shift, scale)
    _check(h, _ln_ref(x, shift, scale), dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gate_residual_in_place(dtype):
    from hilberta_b200.block_ops import gate_residual

    g = torch.Generator().manual_seed(2)
    x = torch.randn(2, 257, 3072, generator=g).to(dtype).cuda()
    y = torch.randn(2, 257, 3072, generator=g).to(dtype).cuda()
    _, _, gate, *_ = _mods(2, 3072, dtype, g)
    ref = x.float() + gate.float()[:, None] * y.float()
    ptr = x.data_ptr()
    out = gate_residual(x, y, gate)
    assert out.data_ptr() == ptr
    _check(x, ref, dtype, slack=1e-6)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gate_residual_adaln(dtype):
    from hilberta_b200.block_ops import gate_residual_adaln

    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 515, 3072, generator=g).to(dtype).cuda()
    y = torch.randn(2, 515, 3072, generator=g).to(dtype).cuda()
    shift, scale, gate, *_ = _mods(2, 3072, dtype, g)
    x_ref = x.float() + gate.float()[:, None] * y.float()
    x_new, h = gate_residual_adaln(x, y, gate, shift, scale)
    _check(x_new, x_ref, dtype, slack=1e-6)
    _check(h, _ln_ref(x_new, shift, scale), dtype)  # the LayerNorm reads the rounded stream


def test_strided_rows_and_single_batch():
    from hilberta_b200.block_ops import adaln, gate_residual_adaln

    g = torch.Generator().manual_seed(4)
    big = torch.randn(1, 600, 2 * 1024, generator=g).to(torch.bfloat16).cuda()
    x = big[:, :, :1024]  # row stride 2048
    y = torch.randn(1, 600, 2 * 1024, generator=g).to(torch.bfloat16).cuda()[:, :, 1024:]
    shift, scale, gate, *_ = _mods(1, 1024, torch.bfloat16, g)
    _check(adaln(x, shift, scale), _ln_ref(x, shift, scale), torch.bfloat16)
    untouched = big[:, :, 1024:].clone()
    x_ref = x.float() + gate.float()[:, None] * y.float()
    gate_residual_adaln(x, y, gate, shift, scale)
    _check(x, x_ref, torch.bfloat16, slack=1e-6)
    assert torch.equal(big[:, :, 1024:], untouched)  # only the view's columns are written


def test_argument_errors():
    from hilberta_b200.block_ops import adaln

    x = torch.zeros(1, 8, 128, dtype=torch.bfloat16, device="cuda")
    m = torch.zeros(1, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(Exception):
        adaln(x, m, m)  # C = 128 is not a multiple of 256
    x = torch.zeros(2, 8, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="one row per batch"):
        adaln(x, m[:, :1].expand(1, 256).contiguous(), m[:, :1].expand(1, 256).contiguous())


def test_native_block_ops_gemms():
    from hilberta_b200.block_ops import NativeBlockOps

    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 300, 512, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(1024, 512, generator=g) * 0.05).to(torch.bfloat16).cuda()
    b = (torch.randn(1024, generator=g) * 0.1).to(torch.bfloat16).cuda()
    got = NativeBlockOps.linear_gelu(x, w, b).float()
    ref = F.gelu(x.float() @ w.float().t() + b.float(), approximate="tanh")
    assert got.shape == (2, 300, 1024)
    assert float((got - ref).abs().max()) < 2e-2 * float(ref.abs().max())
    m = torch.randn(2, 300, 1024, generator=g).to(torch.bfloat16).cuda()
    wj = (torch.randn(512, 512 + 1024, generator=g) * 0.05).to(torch.bfloat16).cuda()
    got = NativeBlockOps.joined_linear(x, m, wj[:, :512], wj[:, 512:], b[:512]).float()
    ref = torch.cat([x, m], -1).float() @ wj.float().t() + b[:512].float()
    assert float((got - ref).abs().max()) < 2e-2 * float(ref.abs().max())
