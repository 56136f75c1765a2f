"""hb_norm_rope_pack / hilberta_b200.prep against the CPU restatement of the FLUX
processor's Q/K/V preparation (oracle/processor_oracle.py).

Exact where the arithmetic is elementwise: packing (V), rotation, and rotation
of the kernel's own normalised rows are bit-identical.  The normalisation sums
the D squares in its own order (fused multiply-adds, a lane-pair shuffle)
rather than torch's CPU reduction order, so x * rsqrt may round to the
neighbouring 16-bit value; multiplied by a weight below 1 that one-unit step
can land one binade lower, i.e. two units of the result.  Bound: at most 2 ulp,
on well under 1 % of elements.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import attention_oracle as ao
from oracle import processor_oracle as po

pytestmark = pytest.mark.gpu


def _inputs(B=1, T=128, n=256, H=4, D=128, dtype=torch.bfloat16, seed=5):
    g = torch.Generator().manual_seed(seed)
    txt = (torch.randn(B, T, H * D, generator=g) * 3).to(dtype)
    img = (torch.randn(B, n, H * D, generator=g) * 3).to(dtype)
    wt = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    wi = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    ang = torch.rand(T + n, D // 2, generator=g, dtype=torch.float64) * 6.28
    cos = torch.cos(ang).repeat_interleave(2, dim=1).float()
    sin = torch.sin(ang).repeat_interleave(2, dim=1).float()
    return txt, img, wt, wi, cos, sin


def _ulps(a, b):
    """Distance in units in the last place between two 16-bit tensors of one dtype."""
    ia = a.view(torch.int16).to(torch.int32)
    ib = b.view(torch.int16).to(torch.int32)
    ia = torch.where(ia < 0, -32768 - ia, ia)  # sign-magnitude -> monotone integers
    ib = torch.where(ib < 0, -32768 - ib, ib)
    return (ia - ib).abs()


def test_pack_and_rotation_are_exact():
    from hilberta_b200 import prep

    txt, img, wt, wi, cos, sin = _inputs()
    v = prep.norm_rope_pack(txt.cuda(), img.cuda(), heads=4)
    assert torch.equal(v.cpu(), po.norm_rope_pack(txt, img, heads=4))
    r = prep.norm_rope_pack(txt.cuda(), img.cuda(), heads=4, cos=cos.cuda(), sin=sin.cuda())
    assert torch.equal(r.cpu(), po.norm_rope_pack(txt, img, heads=4, cos=cos, sin=sin))


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 128), (torch.bfloat16, 64)])
def test_norm_within_two_ulp_and_rotation_exact_on_top(dtype, D):
    from hilberta_b200 import prep

    txt, img, wt, wi, cos, sin = _inputs(D=D, dtype=dtype, seed=6)
    kw = dict(heads=4, weight_txt=wt, weight_img=wi)
    normed = prep.norm_rope_pack(txt.cuda(), img.cuda(), heads=4, weight_txt=wt.cuda(), weight_img=wi.cuda()).cpu()
    u = _ulps(normed, po.norm_rope_pack(txt, img, **kw))
    assert int(u.max()) <= 2
    assert float((u > 0).float().mean()) < 0.01
    # rotation of the kernel's own normalised rows is exact (a 1-ulp difference
    # upstream can be many ulps of y0*cos - y1*sin when the two terms cancel)
    both = prep.norm_rope_pack(txt.cuda(), img.cuda(), heads=4, weight_txt=wt.cuda(), weight_img=wi.cuda(),
                               cos=cos.cuda(), sin=sin.cuda()).cpu()
    assert torch.equal(both, po.apply_rope(normed, cos, sin))


def test_image_rows_place_tokens_and_strided_inputs():
    from hilberta_b200 import prep

    txt, img, wt, wi, cos, sin = _inputs(n=256, seed=7)
    perm = torch.randperm(256, generator=torch.Generator().manual_seed(1)).to(torch.int32)
    # projections as column slices of one fused [B, S, 3*H*D] matmul output (row stride 3*H*D)
    big = torch.zeros(1, 256, 3 * 512, dtype=img.dtype)
    big[:, :, 512:1024] = img
    got = prep.norm_rope_pack(txt.cuda(), big.cuda()[:, :, 512:1024], heads=4, cos=cos.cuda(), sin=sin.cuda(),
                              image_rows=perm.cuda()).cpu()
    assert torch.equal(got, po.norm_rope_pack(txt, img, heads=4, cos=cos, sin=sin, image_rows=perm))
    normed = prep.norm_rope_pack(txt.cuda(), big.cuda()[:, :, 512:1024], heads=4, weight_txt=wt.cuda(),
                                 weight_img=wi.cuda(), image_rows=perm.cuda()).cpu()
    want = po.norm_rope_pack(txt, img, heads=4, weight_txt=wt, weight_img=wi, image_rows=perm)
    assert int(_ulps(normed, want).max()) <= 2


def test_bad_image_row_is_dropped_and_flagged():
    from hilberta_b200 import _lib

    txt, img, _, _, _, _ = _inputs(T=0, n=64, H=2, seed=8)
    img = img.cuda()
    rows = torch.arange(64, dtype=torch.int32, device="cuda")
    rows[5] = 64  # out of range
    out = torch.full((1, 64, 2, 128), 3.0, dtype=img.dtype, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _lib.lib().hb_norm_rope_pack(
        None, 0, 0, ctypes.c_void_p(img.data_ptr()), img.stride(0), img.stride(1), 1, 0, 64, 2, 128, None, None,
        1e-6, None, None, ctypes.c_void_p(rows.data_ptr()), ctypes.c_void_p(out.data_ptr()), out.stride(0),
        out.stride(1), out.stride(2), 1, ctypes.c_void_p(status.data_ptr()), None)
    torch.cuda.synchronize()
    assert rc == 0 and int(status.item()) == _lib.HB_DEV_BAD_BLOCK
    assert bool((out[0, 5] == 3.0).all())  # row 5 is the one no valid token maps to
    keep = [i for i in range(64) if i != 5]
    assert torch.equal(out[0, keep].cpu(), img.cpu().view(1, 64, 2, 128)[0, keep])


def test_prepare_qkv_feeds_paired_attention():
    """End to end on a 32x32 plan: the processor's prepared Q/K/V through the
    kernel match the oracle's preparation through the fp32 attention oracle."""
    import hilberta_b200 as hb
    from hilberta_b200 import prep

    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    N, G, T, n = plan.total_tokens, plan.global_tokens, plan.text_tokens, plan.total_tokens - plan.text_tokens
    p = plan.phases[1]
    meta = hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=G).to("cuda")
    g = torch.Generator().manual_seed(9)
    H, D = 2, 128
    proj = [(torch.randn(1, T if i < 3 else n, H * D, generator=g) * 2).to(torch.bfloat16) for i in range(6)]
    w = [(1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16) for _ in range(4)]
    ang = torch.rand(N, D // 2, generator=g, dtype=torch.float64) * 6.28
    cos = torch.cos(ang).repeat_interleave(2, dim=1).float()
    sin = torch.sin(ang).repeat_interleave(2, dim=1).float()
    q, k, v = prep.prepare_qkv(*(x.cuda() for x in proj), heads=H, norm_q=w[0].cuda(), norm_k=w[1].cuda(),
                               norm_added_q=w[2].cuda(), norm_added_k=w[3].cuda(), rotary=(cos.cuda(), sin.cuda()))
    assert q.shape == (1, H, N, D) and q.stride(1) == D  # BNHD storage viewed as BHND
    with torch.inference_mode():
        out = hb.paired_attention(q, k, v, meta)
    qo = po.norm_rope_pack(proj[0], proj[3], heads=H, weight_txt=w[2], weight_img=w[0], cos=cos, sin=sin)
    ko = po.norm_rope_pack(proj[1], proj[4], heads=H, weight_txt=w[3], weight_img=w[1], cos=cos, sin=sin)
    vo = po.norm_rope_pack(proj[2], proj[5], heads=H)
    ref = ao.masked_attention_fp32(*(x.transpose(1, 2) for x in (qo, ko, vo)),
                                   ao.block_mask_from_rows(p.kv_indices, p.kv_counts, N, G))
    err = (out.float().cpu() - ref).abs()
    assert float(err.max()) <= 2e-2 and float(err.mean()) <= 2e-3
