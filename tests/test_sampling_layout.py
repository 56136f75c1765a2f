"""Host-side checks of sample_flux_persistent (hilberta/sampling_layout.py:
21-60): pipelines without the needed hooks, stochastic schedulers, nesting,
unpacked callbacks and IP-adapter inputs are refused before any work.  No GPU."""

from __future__ import annotations

import pytest

from hilberta_b200.sampling_layout import _ACTIVE, sample_flux_persistent
from tests._tiny_pipe import Scheduler, TinyPipe


class _NoHooks:
    transformer = None
    scheduler = Scheduler()


def _pipe():
    p = TinyPipe.__new__(TinyPipe)
    p.transformer, p.scheduler = None, Scheduler()
    return p


def test_refusals():
    with pytest.raises(TypeError, match="prepare_latents"):
        sample_flux_persistent(_NoHooks(), None)
    p = _pipe()
    p.scheduler = Scheduler(stochastic=True)
    with pytest.raises(ValueError, match="Stochastic"):
        sample_flux_persistent(p, None)
    p = _pipe()
    setattr(p, _ACTIVE, True)
    with pytest.raises(RuntimeError, match="Nested"):
        sample_flux_persistent(p, None)
    with pytest.raises(ValueError, match="packed_callback_on_step_end"):
        sample_flux_persistent(_pipe(), None, callback_on_step_end=lambda *a: {})
    with pytest.raises(ValueError, match="IP-adapter"):
        sample_flux_persistent(_pipe(), None, ip_adapter_image=object())
