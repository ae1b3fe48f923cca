"""Predicated block-sparse attention drop-in (reference: src/orthocache/sparse_attention.py).

The reference masks evicted logits with -1e9 per (block, head) and takes a
softmax over all tokens (``sparse_attention.py:5-64``).  Here each head's
kept blocks are compacted into their own index list and only those blocks are
read (per-head indirect attention); the softmax over the kept tokens is the
same.  A head whose mask keeps no block gets the uniform average of all its
value rows, which is what the reference's all -1e9 logit row gives.
"""
from __future__ import annotations

from . import _core, _lib


def jax_block_sparse_attention(q, keys, values, block_mask, block_size: int = 512):
    """Per-head masked attention; block_mask (nb, Hkv) bool.  Output in q's dtype."""
    qq, k, v, batched = _core.batched_qkv(q, keys, values)
    B, S, Hkv, D = k.shape
    nb = S // block_size
    m = _lib.as_device(block_mask)
    if not batched:
        m = m.unsqueeze(0)
    if m.dim() == 2:  # (B, nb) -> same mask for all heads
        m = m.unsqueeze(-1).expand(B, nb, Hkv)
    if tuple(m.shape) != (B, nb, Hkv):
        raise ValueError(f"block_mask {tuple(block_mask.shape)} does not match (nb={nb}, Hkv={Hkv})")
    perm, count = _core.compact_per_head(m)
    out = _core.attend(qq, k, v, perm, count, block_size, idx_stride=Hkv * nb, idx_head_stride=nb,
                       count_stride=Hkv, count_head_stride=1)
    _core.fill_empty_heads(out, v, count, Hkv, 1)
    return out if batched else out[0]


compile_pallas_sparse_attention = jax_block_sparse_attention
