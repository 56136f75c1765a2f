"""The package's path modules carry the reference's public names: every public
function and class of hilberta's geometry, plan, bridge_k, paired_metadata,
sparse_kernel, paired_kernel, flux_adapter and sampling_layout modules exists
in the same-named module of hilberta_b200 (the list below is that set)."""

from __future__ import annotations

import importlib

import pytest

REFERENCE_PUBLIC = {
    "geometry": ["hilbert_order", "neighbor_pairs"],
    "plan": ["PhasePlan", "AttentionPlan", "build_plan", "full_attention_plan"],
    "bridge_k": ["bridge_k_plan"],
    "paired_metadata": ["PairedMetadata", "pair_metadata", "unpair_metadata"],
    "sparse_kernel": ["validate_metadata", "explicit_mask", "sparse_attention"],
    "paired_kernel": ["paired_attention"],
    "flux_adapter": ["PersistentFluxProcessor", "persistent_flux_attention"],
    "sampling_layout": ["sample_flux_persistent"],
}


@pytest.mark.parametrize("module", sorted(REFERENCE_PUBLIC))
def test_reference_names_exist(module):
    ours = importlib.import_module(f"hilberta_b200.{module}")
    assert [n for n in REFERENCE_PUBLIC[module] if not hasattr(ours, n)] == []


def test_private_helpers_the_reference_tests_import():
    from hilberta_b200.sparse_kernel import _check_inputs  # noqa: F401
