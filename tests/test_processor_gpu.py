"""HilbertAProcessor (the reference adapter's processor call, hilberta/flux_adapter.py:
259-340) on an attention module with FluxAttention's attribute names built from
plain torch layers: the attention part against the CPU oracle of the processor's
steps (oracle/processor_oracle.py + the fp32 dense-mask attention), and the full
call against the module's own output projections applied to that part."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as ao
from oracle import processor_oracle as po

pytestmark = pytest.mark.gpu


class _Norm(torch.nn.Module):
    def __init__(self, d, g):
        super().__init__()
        self.weight = torch.nn.Parameter((1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16), requires_grad=False)
        self.eps = 1e-6


class _Attn(torch.nn.Module):
    """Attribute layout of diffusers' FluxAttention (double- or single-stream)."""

    def __init__(self, dim, heads, d, double, g):
        super().__init__()
        lin = lambda i, o: torch.nn.Linear(i, o).to(torch.bfloat16).requires_grad_(False)
        self.heads = heads
        self.to_q, self.to_k, self.to_v = lin(dim, heads * d), lin(dim, heads * d), lin(dim, heads * d)
        self.norm_q, self.norm_k = _Norm(d, g), _Norm(d, g)
        self.added_kv_proj_dim = dim if double else None
        if double:
            self.add_q_proj, self.add_k_proj, self.add_v_proj = lin(dim, heads * d), lin(dim, heads * d), lin(dim, heads * d)
            self.norm_added_q, self.norm_added_k = _Norm(d, g), _Norm(d, g)
            self.to_out = torch.nn.ModuleList([lin(heads * d, dim), torch.nn.Dropout(0.0)])
            self.to_add_out = lin(heads * d, dim)


def _setup(double):
    import hilberta_b200 as hb

    torch.manual_seed(0)
    g = torch.Generator().manual_seed(1)
    plan = hb.bridge_k_plan(4, 1, False, grid_size=32)
    T, N = plan.text_tokens, plan.total_tokens
    H, D, dim = 2, 128, 256
    attn = _Attn(dim, H, D, double, g).cuda()
    ang = torch.rand(N, D // 2, generator=g, dtype=torch.float64) * 6.28
    rot = (torch.cos(ang).repeat_interleave(2, 1).float().cuda(), torch.sin(ang).repeat_interleave(2, 1).float().cuda())
    bank = hb.PlanBank(plan)
    return plan, bank, attn, rot, T, N, H, D, dim, g


def _oracle_attention(plan, phase, q, k, v):
    p = plan.phases[phase]
    mask = ao.block_mask_from_rows(p.kv_indices, p.kv_counts, plan.total_tokens, plan.global_tokens)
    out = ao.masked_attention_fp32(*(x.transpose(1, 2) for x in (q, k, v)), mask)  # [B, H, S, D]
    return out.transpose(1, 2).flatten(2, 3)


def test_double_stream_block():
    from hilberta_b200.processor import HilbertAProcessor

    plan, bank, attn, rot, T, N, H, D, dim, g = _setup(True)
    hidden = torch.randn(1, N - T, dim, generator=g).to(torch.bfloat16).cuda()
    enc = torch.randn(1, T, dim, generator=g).to(torch.bfloat16).cuda()
    proc = HilbertAProcessor(bank, layer=5)  # phase 1
    with torch.inference_mode():
        att = proc.attention(attn, hidden, enc, rot)
        image, text = proc(attn, hidden, enc, image_rotary_emb=rot)
        proj = [m(x).cpu() for m, x in ((attn.add_q_proj, enc), (attn.to_q, hidden), (attn.add_k_proj, enc),
                                         (attn.to_k, hidden), (attn.add_v_proj, enc), (attn.to_v, hidden))]
        want_image = attn.to_out[1](attn.to_out[0](att[:, T:].to(hidden.dtype)))
        want_text = attn.to_add_out(att[:, :T].to(hidden.dtype))
    torch.cuda.synchronize()
    cos, sin = (x.cpu() for x in rot)
    w = lambda m: m.weight.detach().cpu()
    q = po.norm_rope_pack(proj[0], proj[1], heads=H, weight_txt=w(attn.norm_added_q), weight_img=w(attn.norm_q), cos=cos, sin=sin)
    k = po.norm_rope_pack(proj[2], proj[3], heads=H, weight_txt=w(attn.norm_added_k), weight_img=w(attn.norm_k), cos=cos, sin=sin)
    v = po.norm_rope_pack(proj[4], proj[5], heads=H)
    ref = _oracle_attention(plan, 1, q, k, v)
    err = (att.float().cpu() - ref).abs()
    assert float(err.max()) <= 2e-2 and float(err.mean()) <= 2e-3
    assert image.shape == (1, N - T, dim) and text.shape == (1, T, dim)
    assert torch.equal(image, want_image) and torch.equal(text, want_text)


def test_single_stream_block():
    from hilberta_b200.processor import HilbertAProcessor

    plan, bank, attn, rot, T, N, H, D, dim, g = _setup(False)
    hidden = torch.randn(1, N, dim, generator=g).to(torch.bfloat16).cuda()  # text + image already joined
    proc = HilbertAProcessor(bank, layer=2)  # phase 2
    with torch.inference_mode():
        out = proc(attn, hidden, image_rotary_emb=rot)
        proj = [m(hidden).cpu() for m in (attn.to_q, attn.to_k, attn.to_v)]
    torch.cuda.synchronize()
    cos, sin = (x.cpu() for x in rot)
    w = lambda m: m.weight.detach().cpu()
    q = po.norm_rope_pack(None, proj[0], heads=H, weight_img=w(attn.norm_q), weight_txt=w(attn.norm_q), cos=cos, sin=sin)
    k = po.norm_rope_pack(None, proj[1], heads=H, weight_img=w(attn.norm_k), weight_txt=w(attn.norm_k), cos=cos, sin=sin)
    v = po.norm_rope_pack(None, proj[2], heads=H)
    ref = _oracle_attention(plan, 2, q, k, v)
    err = (out.float().cpu() - ref).abs()
    assert out.shape == (1, N, H * D)
    assert float(err.max()) <= 2e-2 and float(err.mean()) <= 2e-3
