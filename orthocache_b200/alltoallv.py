"""Sequence-parallel exchange protocol over ``torch.distributed``: the
drop-in counterpart of the reference's ``orthocache.alltoallv``
(j-arndt/orthocache v0.3.0, ``src/orthocache/alltoallv.py``):

  stream_compact :44-75, count_sync :80-108, compute_offsets :113-145,
  pack_active_blocks :150-212, alltoallv_exchange :217-259,
  unpack_received_blocks :264-335, alltoallv_kv_exchange :340-440

The reference's ``axis_name`` (a pmap axis) becomes a ``torch.distributed``
process group: NCCL between GPUs (one process per GPU), gloo for host-side
tests.  Block data moves only through the CUDA kernels of
``liborthocache_b200.so`` (block gather, exchange index); the collectives are
``torch.distributed`` calls; the only host-side arithmetic is on the P
per-device counts.

Exchange semantics.  ``alltoallv_exchange`` returns every device's packed
buffer concatenated in rank order (the (P * max_tokens, H, D) layout that
``unpack_received_blocks`` and the reference's docstring describe), i.e. an
all-gather of the packed buffers.  The per-peer AllToAllv (each rank receives
only its own KV heads) is ``orthocache_b200.distributed.alltoallv_heads``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from . import _core

BLOCK_SIZE = 512


# ---------------------------------------------------------------------------
# collectives (any device: NCCL for CUDA tensors, gloo for CPU tensors)
# ---------------------------------------------------------------------------
def _world(group):
    return dist.get_world_size(group)


def _all_gather_cat(t, group=None):
    """Concatenate every rank's ``t`` along dim 0, in rank order."""
    t = t.contiguous()
    P = _world(group)
    out = torch.empty((P * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    if t.is_cuda:
        dist.all_gather_into_tensor(out, t, group=group)
    else:
        dist.all_gather(list(out.chunk(P, dim=0)), t, group=group)
    return out


# ---------------------------------------------------------------------------
# a9 (mask only), a15: compaction, count sync, offsets
# ---------------------------------------------------------------------------
def stream_compact(block_mask):
    """(active_indices int32 (nb,), num_active int32 (1,)) of a (nb,) or
    (nb, H) block mask (``alltoallv.py:44-75``; union over H)."""
    perm, count = _core.compact(block_mask)
    return perm[0], count


def count_sync(local_num_active, group=None):
    """Every rank's active-block count, int32 (P,) (``alltoallv.py:80-108``)."""
    c = torch.as_tensor(local_num_active).reshape(1).to(torch.int32)
    return _all_gather_cat(c, group)


def compute_offsets(all_counts):
    """(offsets (P,), total_active (1,)) int32: the exclusive prefix sum of the
    counts and their sum (``alltoallv.py:113-145``).  Arithmetic on P integers."""
    c = torch.as_tensor(all_counts).to(torch.int64).reshape(-1)
    inc = torch.cumsum(c, 0)
    offsets = (inc - c).to(torch.int32)
    total = inc[-1:].to(torch.int32) if c.numel() else torch.zeros(1, dtype=torch.int32, device=c.device)
    return offsets, total


# ---------------------------------------------------------------------------
# a14, a16: pack, exchange, unpack
# ---------------------------------------------------------------------------
def pack_active_blocks(kv_shard, active_indices, num_active, max_blocks: int, block_size: int = BLOCK_SIZE):
    """Blocks active_indices[:num_active] of kv_shard (S, H, D) copied to the
    front of a (max_blocks * block_size, H, D) buffer whose tail is zero
    (``alltoallv.py:150-212``; ``distributed_attention.py:49-75``)."""
    kv = _lib.as_device(kv_shard).contiguous()
    idx = _lib.as_device(active_indices, device=kv.device, dtype=torch.int32).reshape(1, -1).contiguous()
    cnt = _core.count_tensor(_lib.as_device(num_active, device=kv.device), kv.device)
    out = _core.gather_blocks(kv.unsqueeze(0), idx, cnt, int(max_blocks), block_size, zero_tail=True)
    return out[0]


def alltoallv_exchange(k_packed, v_packed, group=None):
    """Every rank's packed K and V, concatenated in rank order:
    (P * max_tokens, H, D) each (``alltoallv.py:217-259``)."""
    return _all_gather_cat(k_packed, group), _all_gather_cat(v_packed, group)


def global_block_index(all_counts, slots_per_device: int):
    """(order (P * slots,), total (1,)) int32 over a gathered buffer of P
    chunks of ``slots_per_device`` blocks: valid slots (j % slots <
    counts[j // slots]) first in ascending order, then the rest
    (``distributed_attention.py:179-191``; ``phase_e_stratified.py:220-226``)."""
    c = _lib.as_device(all_counts, dtype=torch.int32).reshape(-1).contiguous()
    P = c.numel()
    order = torch.empty((P * slots_per_device,), dtype=torch.int32, device=c.device)
    total = torch.empty((1,), dtype=torch.int32, device=c.device)
    offsets = torch.empty((P,), dtype=torch.int32, device=c.device)
    _lib.call("oc_exchange_index", _lib.ptr(c), P, int(slots_per_device), _lib.ptr(order), _lib.ptr(total),
              _lib.ptr(offsets), _lib.stream_ptr(c.device))
    return order, total, offsets


def unpack_received_blocks(kv_received, all_counts, num_devices: int, max_blocks: int,
                           block_size: int = BLOCK_SIZE):
    """(active_kv, device_offsets): the valid blocks of each device's chunk
    moved to the front in device order, zero tail; token offsets of each
    device's run (``alltoallv.py:264-335``).  Bit-exact block copies."""
    kv = _lib.as_device(kv_received).contiguous()
    order, total, offsets = global_block_index(_lib.as_device(all_counts, device=kv.device),
                                               int(max_blocks))
    nslots = int(num_devices) * int(max_blocks)
    out = _core.gather_blocks(kv.unsqueeze(0), order.reshape(1, -1), total, nslots, block_size, zero_tail=True)
    return out[0], offsets * block_size


def alltoallv_kv_exchange(k_shard, v_shard, block_mask, group=None, block_size: int = BLOCK_SIZE):
    """End-to-end exchange (``alltoallv.py:340-440``): returns
    ``(k_active, v_active, all_counts, offsets, stats)``.  The first
    total_active * block_size tokens of k_active / v_active are the retained
    blocks of every rank in rank order; stats holds device tensors
    (local_num_active, total_active, bytes_saved) and ints (dense_blocks,
    bytes_dense) as the reference's dict does."""
    k = _lib.as_device(k_shard).contiguous()
    v = _lib.as_device(v_shard, device=k.device).contiguous()
    nb = k.shape[0] // block_size
    active_indices, num_active = stream_compact(block_mask)
    all_counts = count_sync(num_active, group)
    offsets, total_active = compute_offsets(all_counts)
    kp = pack_active_blocks(k, active_indices, num_active, nb, block_size)
    vp = pack_active_blocks(v, active_indices, num_active, nb, block_size)
    kr, vr = alltoallv_exchange(kp, vp, group)
    P = all_counts.numel()
    k_active, _ = unpack_received_blocks(kr, all_counts, P, nb, block_size)
    v_active, _ = unpack_received_blocks(vr, all_counts, P, nb, block_size)
    H, D = k.shape[1], k.shape[2]
    per_block = block_size * H * D * k.element_size() * 2  # K + V
    dense_blocks = P * nb
    bytes_dense = dense_blocks * per_block
    stats = {
        "local_num_active": num_active,
        "total_active": total_active,
        "dense_blocks": dense_blocks,
        "bytes_saved": bytes_dense - total_active.to(torch.int64) * per_block,
        "bytes_dense": bytes_dense,
    }
    return k_active, v_active, all_counts, offsets, stats


__all__ = [
    "BLOCK_SIZE", "stream_compact", "count_sync", "compute_offsets", "pack_active_blocks", "alltoallv_exchange",
    "global_block_index", "unpack_received_blocks", "alltoallv_kv_exchange",
]
