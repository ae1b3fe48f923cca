"""Stream compaction drop-ins (reference: src/orthocache/compaction.py)."""
from __future__ import annotations

import torch

from . import _core, _lib


def stream_compact(keys, values=None, block_mask=None, block_size: int = 512):
    """Compact the KV cache to its retained blocks (``compaction.py:28-100``).

    ``stream_compact(keys, values, block_mask, block_size)`` returns
    (compact_keys, compact_values, active_indices, num_active):
    compact tensors are (num_blocks, block_size, H, D) with the active blocks
    first (in ascending original order) and zeros after; active_indices
    (num_blocks,) int32 is the full stable permutation (active first, then
    inactive ascending); num_active a 0-d int32 device tensor.  A block is
    active if any head keeps it (``compaction.py:65``).

    ``stream_compact(block_mask)`` (the mask-only form of ``alltoallv.py:44``)
    returns (active_indices, num_active).
    """
    if values is None and block_mask is None:
        perm, count = _core.compact(keys)
        return perm[0], count[0]
    k = _lib.as_device(keys)
    v = _lib.as_device(values, device=k.device)
    S, H, D = k.shape
    nb = S // block_size
    perm, count = _core.compact(block_mask)
    ck = _core.gather_blocks(k.unsqueeze(0), perm, count, nb, block_size)[0]
    cv = _core.gather_blocks(v.unsqueeze(0), perm, count, nb, block_size)[0]
    return (ck.reshape(nb, block_size, H, D), cv.reshape(nb, block_size, H, D), perm[0], count[0])


def stream_decompact(compact_output, active_indices, num_active, num_blocks_original: int,
                     block_size: int = 512):
    """Scatter compacted blocks back to their original positions, zeros elsewhere
    (``compaction.py:103-154``)."""
    c = _lib.as_device(compact_output)
    nbc, bs, H, D = c.shape
    perm = _lib.as_device(active_indices, device=c.device, dtype=torch.int32)
    cnt = _core.count_tensor(num_active, c.device)
    out = torch.empty((num_blocks_original, bs, H, D), dtype=c.dtype, device=c.device)
    _lib.call("oc_scatter_blocks", _lib.ptr(c), _lib.dtype_code(c), 1, nbc, bs * H * D, _lib.ptr(perm),
              perm.shape[-1], _lib.ptr(cnt), _lib.ptr(out), num_blocks_original, _lib.stream_ptr(c.device))
    return out


def compact_and_attend(q, keys, values, block_mask, block_size: int = 512):
    """Compaction + attention over the retained blocks (``compaction.py:157-222``).

    The reference copies the retained blocks into a compact tensor and runs
    masked attention on it; here the attention reads the retained blocks in
    place through the index list (same result, no copy).  Returns
    (output (Sq, H, D) in q's dtype, metadata with num_active, num_blocks,
    eviction_rate).
    """
    qq, k, v, batched = _core.batched_qkv(q, keys, values)
    nb = k.shape[1] // block_size
    perm, count = _core.compact(block_mask, batched=batched)
    out = _core.attend(qq, k, v, perm, count, block_size)
    if not batched:
        out = out[0]
    n = count if batched else count[0]
    meta = _core.Meta(num_active=n, num_blocks=nb,
                      eviction_rate=lambda: 1.0 - float(n.float().mean().item()) / nb)
    return out, meta
