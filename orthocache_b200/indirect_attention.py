"""Indirect attention drop-in (reference: src/orthocache/indirect_attention.py).

No copy of the KV cache: the attention reads the retained blocks in place
through an index table, like the reference's Pallas kernel.  The device-side
count never leaves the GPU; the metadata synchronises only when read.
"""
from __future__ import annotations

import torch

from . import _core, _lib

BUCKETS = [1, 2, 4, 8, 16, 32, 64, 128, 256, 512]  # indirect_attention.py:20


def _next_bucket(n):
    """Smallest bucket >= n, or n beyond the largest (``indirect_attention.py:22-26``)."""
    for b in BUCKETS:
        if b >= n:
            return b
    return n


def compile_indirect_attention(q, keys, values, active_indices, bucket_size: int, block_size: int = 512):
    """Attention over exactly ``bucket_size`` table entries per head
    (``indirect_attention.py:86-124``); active_indices (bucket_size, H) int32."""
    qq, k, v, batched = _core.batched_qkv(q, keys, values)
    B, S, Hkv, D = k.shape
    tab = _lib.as_device(active_indices, device=k.device, dtype=torch.int32)
    if tab.dim() == 1:
        tab = tab[:, None].expand(tab.shape[0], Hkv)
    tab = tab[:bucket_size].t().contiguous()  # (H, bucket)
    cnt = torch.full((Hkv,), int(bucket_size), dtype=torch.int32, device=k.device)
    out = _core.attend(qq, k, v, tab, cnt, block_size, max_blocks=int(bucket_size), idx_stride=0,
                       idx_head_stride=int(bucket_size), count_stride=0, count_head_stride=1)
    return out if batched else out[0]


def indirect_attention(q, keys, values, block_mask, block_size: int = 512):
    """Top-level indirect attention (``indirect_attention.py:127-170``).

    Union mask over heads -> stable active-first permutation -> the reference's
    power-of-two bucket of the active count -> attention over the first
    ``bucket`` permutation entries (as the reference's kernel does, the
    entries between the active count and the bucket are the first evicted
    blocks, and they are attended too).  No active block -> zeros.
    Returns (output in q's dtype, metadata num_active / bucket / num_blocks /
    eviction_rate).
    """
    qq, k, v, batched = _core.batched_qkv(q, keys, values)
    nb = k.shape[1] // block_size
    perm, count = _core.compact(block_mask, batched=batched)
    bcount = torch.empty_like(count)
    _lib.call("oc_bucket_count", _lib.ptr(count), count.numel(), nb, _lib.ptr(bcount),
              _lib.stream_ptr(k.device))
    out = _core.attend(qq, k, v, perm, bcount, block_size)
    if not batched:
        out = out[0]
    n = count if batched else count[0]

    def _bucket():
        c = int(count[0].item()) if not batched else [int(x) for x in count.tolist()]
        return (_next_bucket(c) if c else 0) if not batched else [(_next_bucket(x) if x else 0) for x in c]

    meta = _core.Meta(num_active=n, bucket=_bucket, num_blocks=nb,
                      eviction_rate=lambda: 1.0 - float(n.float().mean().item()) / nb)
    return out, meta
