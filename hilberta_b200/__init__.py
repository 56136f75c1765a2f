"""hilberta_b200 — B200-native HilbertA inference attention.

Drop-in for the reference's operator API (``hilberta``): plan builders
(``build_plan``, ``bridge_k_plan``), metadata (``pair_metadata``,
``validate_metadata``) and the paired block-sparse attention
(``paired_attention``), all executed by the sm_100a library in ``lib/``.

Additions beyond that API: raster-order tensors (``raster_order``,
``token_order_map`` for ``paired_attention(token_order=...)``), the adapter's
plan cache (``PlanBank``), plans on disk (``save_plan``, ``load_plan``,
``PlanCache``), the processor's Q/K/V preparation
(``prepare_qkv``), and head-parallel attention over several GPUs with the head
all-gather fused into the kernel (``PeerAllGather``), and the FLUX processor
built from them (``HilbertAProcessor``), the reference adapter's entry
(``persistent_flux_attention``) and sampling wrapper (``sample_flux_persistent``),
and a FLUX.1-architecture transformer with
random weights and diffusers' interface to run it on
(``hilberta_b200.flux_model.FluxTransformer``).
"""

from .bridge_k import bridge_k_plan
from .head_parallel import PeerAllGather, all_gather_heads, head_parallel_attention
from .paired_kernel import RasterOrder, device_status, paired_attention, raster_order, token_order_map
from .paired_metadata import PairedMetadata, pair_metadata, unpair_metadata
from .plan import AttentionPlan, PhasePlan, build_plan, full_attention_plan
from .plan_bank import PlanBank
from .plan_cache import PlanCache, load_plan, save_plan
from .prep import norm_rope_pack, prepare_qkv
from .processor import HilbertAProcessor
from .flux_adapter import persistent_flux_attention
from .sampling_layout import sample_flux_persistent
from .sparse_kernel import explicit_mask, sparse_attention, validate_metadata

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
    "sparse_attention",
    "device_status",
    "RasterOrder",
    "raster_order",
    "token_order_map",
    "PlanBank",
    "PlanCache",
    "save_plan",
    "load_plan",
    "prepare_qkv",
    "norm_rope_pack",
    "PeerAllGather",
    "all_gather_heads",
    "head_parallel_attention",
    "HilbertAProcessor",
    "persistent_flux_attention",
    "sample_flux_persistent",
]
