"""orthocache_b200 — B200-native (sm_100a) OrthoCache eviction + attention hot path.

Drop-in functions with the reference's names (j-arndt/orthocache v0.3.0,
``src/orthocache/__init__.py:5-23``), backed by hand-written CUDA kernels in
``liborthocache_b200.so``.  Inputs are torch CUDA tensors (NumPy arrays and
CPU tensors are copied to the current device).  There is no CPU fallback:
without the library or a GPU every call raises.
"""
__version__ = "0.1.0"

from .fwht import fwht_512
from .spectral_energy import (
    compute_block_energy_jax,
    generate_threshold_mask,
    compute_query_aware_bounds,
    compute_query_aware_mask,
    compute_spectral_bands,
    compute_spectral_decay_ratio,
    compute_multiband_mask,
    score_blocks,
    BAND_LOW, BAND_MID, BAND_HIGH,
)
from .sparse_attention import jax_block_sparse_attention, compile_pallas_sparse_attention
from .compaction import stream_compact, stream_decompact, compact_and_attend
from .pipeline import orthocache_forward
from .indirect_attention import indirect_attention, compile_indirect_attention
from .adaptive_attention import orthocache_attention, orthocache_attention_batched
from .metadata_cache import SpectralMetadataCache
from .paged import PagedKVCache
from . import nvlink_model

__all__ = [
    "fwht_512", "compute_block_energy_jax", "generate_threshold_mask", "compute_query_aware_bounds",
    "compute_query_aware_mask", "compute_spectral_bands", "compute_spectral_decay_ratio",
    "compute_multiband_mask", "score_blocks", "jax_block_sparse_attention",
    "compile_pallas_sparse_attention", "stream_compact", "stream_decompact", "compact_and_attend",
    "orthocache_forward", "indirect_attention", "compile_indirect_attention", "orthocache_attention",
    "orthocache_attention_batched", "SpectralMetadataCache", "PagedKVCache",
]
