"""Host-side checks of the FLUX.1-architecture step model (no GPU): the full
configuration's size, and argument errors."""

from __future__ import annotations

import pytest
import torch

from hilberta_b200.flux_model import FluxLikeTransformer, parameter_count, rotary_3axis, timestep_features


def test_full_configuration_has_flux1_size():
    # 19 double + 38 single blocks, hidden 3072: FLUX.1-dev's 11.9 B parameters
    model = FluxLikeTransformer(128, None, attention="dense", device="meta")
    assert len(model.double_blocks) == 19 and len(model.single_blocks) == 38
    assert 11.85e9 < parameter_count(model) < 11.95e9
    assert model.rot[0].shape == (512 + 128 * 128, 128)


def test_attention_modes_need_a_bank():
    with pytest.raises(ValueError, match="PlanBank"):
        FluxLikeTransformer(8, None, attention="hilberta", num_double=1, num_single=1, dim=256, heads=2, device="meta")
    model = FluxLikeTransformer(8, None, attention="dense", num_double=1, num_single=1, dim=256, heads=2, device="meta")
    with pytest.raises(ValueError, match="attention must be"):
        model.set_attention("sparse")
    with pytest.raises(ValueError, match="PlanBank"):
        model.set_attention("masked")


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


def test_timestep_features():
    f = timestep_features(torch.tensor([0.0, 0.5]))
    assert f.shape == (2, 256)
    assert torch.equal(f[0, :128], torch.ones(128)) and torch.equal(f[0, 128:], torch.zeros(128))
    assert torch.allclose(f[1, 0], torch.cos(torch.tensor(500.0)))
