"""hilberta_b200 — B200-native HilbertA inference attention.

Drop-in for the reference's operator API (``hilberta``): plan builders
(``build_plan``, ``bridge_k_plan``), metadata (``pair_metadata``,
``validate_metadata``) and the paired block-sparse attention
(``paired_attention``), all executed by the sm_100a library in ``lib/``.
"""

from .bridge_k import bridge_k_plan
from .paired_kernel import device_status, paired_attention
from .paired_metadata import PairedMetadata, pair_metadata, unpair_metadata
from .plan import AttentionPlan, PhasePlan, build_plan, full_attention_plan
from .sparse_kernel import explicit_mask, validate_metadata

__version__ = "0.1.0"

__all__ = [
    "bridge_k_plan",
    "build_plan",
    "full_attention_plan",
    "AttentionPlan",
    "PhasePlan",
    "PairedMetadata",
    "pair_metadata",
    "unpair_metadata",
    "validate_metadata",
    "explicit_mask",
    "paired_attention",
    "device_status",
]
