"""OrthoCache adaptive indirect attention drop-in (reference: src/orthocache/adaptive_attention.py).

The reference dispatches between a per-head vmap and a multi-head loop by
sequence length (``adaptive_attention.py:126-177``), a TPU tuning choice.  On
B200 one split-KV kernel serves every length: work items are (retained block,
128-token chunk, kv head), taken by a persistent grid; the results are
merged in log-sum-exp form.  Output is bfloat16 as in the reference
(``:76, :120``).
"""
from __future__ import annotations

import torch

from . import _core, _lib

BS = 512
_SEQ_THRESHOLD = 16384  # adaptive_attention.py:126 (kept for reference; not used for dispatch)


def stream_compact(block_mask):
    """(active_indices, num_active int) for a (num_blocks,) mask (``adaptive_attention.py:29-40``)."""
    perm, count = _core.compact(block_mask)
    return perm[0], int(count[0].item())


def orthocache_attention(q, k_cache, v_cache, block_mask, block_size: int = BS):
    """Indirect attention over the blocks kept by a (num_blocks,) mask.

    q (Sq, H, D); k_cache, v_cache (S, H, D).  Returns (bf16 output, stats).
    """
    qq, k, v, _ = _core.batched_qkv(q, k_cache, v_cache)
    nb = k.shape[1] // block_size
    perm, count = _core.compact(block_mask)
    out = _core.attend(qq, k, v, perm, count, block_size, out_dtype=torch.bfloat16)[0]
    n = count[0]
    stats = _core.Meta(num_active=n, num_blocks=nb,
                       eviction_rate=lambda: 1.0 - float(n.item()) / nb,
                       path="b200_split_kv")
    return out, stats


def orthocache_attention_batched(q, k_cache, v_cache, block_mask, block_size: int = BS):
    """Batched form (``adaptive_attention.py:212-260``): q (B, Sq, H, D), caches
    (B, S, H, D), one (num_blocks,) mask shared by the batch."""
    qq, k, v, batched = _core.batched_qkv(q, k_cache, v_cache)
    if not batched:
        raise ValueError("orthocache_attention_batched expects 4-D inputs")
    B = k.shape[0]
    nb = k.shape[1] // block_size
    perm, count = _core.compact(block_mask)
    out = _core.attend(qq, k, v, perm, count, block_size, idx_stride=0, count_stride=0,
                       out_dtype=torch.bfloat16)
    n = count[0]
    stats = _core.Meta(num_active=n, num_blocks=nb,
                       eviction_rate=lambda: 1.0 - float(n.item()) / nb,
                       batch_size=B, path="b200_split_kv_batched")
    return out, stats
