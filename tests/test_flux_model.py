"""Host-side checks of the FLUX.1-architecture model and of the adapter entry's
argument checks (hilberta/flux_adapter.py:359-388), which run before any plan
or device work.  No GPU."""

from __future__ import annotations

import pytest
import torch

from hilberta_b200.flux_adapter import _ACTIVE, persistent_flux_attention
from hilberta_b200.flux_model import FluxTransformer, image_ids, parameter_count, rotary_3axis, timestep_features


def test_full_configuration_has_flux1_size():
    # 19 double + 38 single blocks, hidden 3072: FLUX.1-dev's 11.9 B parameters
    model = FluxTransformer(device="meta")
    assert len(model.transformer_blocks) == 19 and len(model.single_transformer_blocks) == 38
    assert 11.85e9 < parameter_count(model) < 11.95e9
    assert not model.training and not model.gradient_checkpointing
    assert all(m.processor is not None for m in model.attention_modules())


def test_rotary_axes_and_positions():
    ids = torch.tensor([[0, 0, 0], [0, 3, 5]])
    cos, sin = rotary_3axis(ids)
    assert cos.shape == sin.shape == (2, 128)
    assert torch.equal(cos[0], torch.ones(128)) and torch.equal(sin[0], torch.zeros(128))
    # axis 1 (rows) covers dims 16..71 in pairs; its first pair turns by the row index
    assert torch.allclose(cos[1, 16:18], torch.cos(torch.tensor([3.0, 3.0])))
    # axis 2 (columns) covers dims 72..127
    assert torch.allclose(sin[1, 72:74], torch.sin(torch.tensor([5.0, 5.0])))
    assert torch.equal(cos[1, :16], torch.ones(16))
    assert torch.equal(image_ids(4)[6], torch.tensor([0, 1, 2]))


def test_timestep_features():
    f = timestep_features(torch.tensor([0.0, 0.5]))
    assert f.shape == (2, 256)
    assert torch.equal(f[0, :128], torch.ones(128)) and torch.equal(f[0, 128:], torch.zeros(128))
    assert torch.allclose(f[1, 0], torch.cos(torch.tensor(500.0)))


def _small():
    return FluxTransformer(num_double=1, num_single=1, dim=256, heads=2, device="meta")


def _enter(model, **kw):
    with persistent_flux_attention(model, None, **kw):
        pass


def test_adapter_argument_checks():
    model = _small()
    with pytest.raises(ValueError, match="layout_scope"):
        _enter(model, layout_scope="image")
    with pytest.raises(ValueError, match="backend must be"):
        _enter(model, backend="flash")
    with pytest.raises(ValueError, match="backend must be"):
        _enter(model, backend="paired", sdpa_backend="flash")
    model.train()
    with pytest.raises(ValueError, match="eval mode"):
        _enter(model, backend="paired")
    model.eval()
    model.gradient_checkpointing = True
    with pytest.raises(ValueError, match="eval mode"):
        _enter(model, backend="paired")
    model.gradient_checkpointing = False
    setattr(model, _ACTIVE, True)
    with pytest.raises(RuntimeError, match="Nested"):
        _enter(model, backend="paired")
    delattr(model, _ACTIVE)
    model._cache_config = {"any": 1}
    with pytest.raises(ValueError, match="cache state"):
        _enter(model, backend="paired")


def test_adapter_block_checks():
    no_single = FluxTransformer(num_double=1, num_single=0, dim=256, heads=2, device="meta")
    with pytest.raises(ValueError, match="joint and single blocks"):
        _enter(no_single, backend="paired")
    model = _small()
    model.transformer_blocks[0].attn.processor._parallel_config = object()
    with pytest.raises(ValueError, match="non-parallel"):
        _enter(model, backend="paired")
    model = _small()
    model.single_transformer_blocks[0].attn.added_kv_proj_dim = 256
    with pytest.raises(ValueError, match="disagree"):
        _enter(model, backend="paired")
