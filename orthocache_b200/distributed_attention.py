"""Attention across sequence shards over ``torch.distributed``: the drop-in
counterpart of the reference's ``orthocache.distributed_attention``
(j-arndt/orthocache v0.3.0, ``src/orthocache/distributed_attention.py``:
distributed_orthocache_attention :131-195, ici_data_volume :198-223) and of
``benchmarks/phase_e_stratified.py``'s build_stratified (:164-273).

Three ways to run attention across P sequence shards:
``distributed_orthocache_attention`` (the reference's replicated gather of
the packed K/V), ``stratified_allgather_attention`` (``build_stratified``:
the gather sized to the smallest capacity bucket that holds the largest
count) and ``sequence_parallel_attention`` (no K/V movement: each rank
attends to its own retained blocks and the per-row (m, l, o) partials are
merged in log-sum-exp form after an all-gather of P * rows * (D + 2)
floats).  All three give the attention of the query over the union of the
retained blocks of all shards.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from . import _core
from .alltoallv import (  # noqa: F401
    BLOCK_SIZE, _world, _all_gather_cat, stream_compact, count_sync, compute_offsets, pack_active_blocks,
    alltoallv_exchange, global_block_index, unpack_received_blocks, alltoallv_kv_exchange,
)


# ---------------------------------------------------------------------------
# a17, a18: attention across shards
# ---------------------------------------------------------------------------
def _attend_gathered(q, k_all, v_all, order, total, block_size):
    q4, k4, v4, _ = _core.batched_qkv(q, k_all, v_all)
    out = _core.attend(q4, k4, v4, order.reshape(1, -1), total, block_size, out_dtype=torch.bfloat16)
    return out[0]


def distributed_orthocache_attention(q_shard, k_shard, v_shard, block_mask, group=None,
                                     block_size: int = BLOCK_SIZE):
    """Attention of the (replicated) query over the retained blocks of every
    rank (``distributed_attention.py:131-195``): local compaction and
    packing, all-gather of the counts and of the packed K/V, the valid-slot
    index over the gathered buffer, then indirect attention.  Returns
    (Sq, Hq, D) bfloat16 on every rank."""
    k = _lib.as_device(k_shard).contiguous()
    v = _lib.as_device(v_shard, device=k.device).contiguous()
    nb = k.shape[0] // block_size
    active_indices, num_active = stream_compact(block_mask)
    kp = pack_active_blocks(k, active_indices, num_active, nb, block_size)
    vp = pack_active_blocks(v, active_indices, num_active, nb, block_size)
    all_counts = count_sync(num_active, group)
    k_all, v_all = alltoallv_exchange(kp, vp, group)
    order, total, _ = global_block_index(all_counts, nb)
    return _attend_gathered(q_shard, k_all, v_all, order, total, block_size)


def stratified_buckets(nb_per_dev: int):
    """The four capacities of ``build_stratified`` (``phase_e_stratified.py:182-197``):
    max(1, nb/4), max(1, nb/2), max(1, 3nb/4), nb, duplicates removed, the
    last repeated to four entries."""
    out = []
    for b in (max(1, nb_per_dev // 4), max(1, nb_per_dev // 2), max(1, (nb_per_dev * 3) // 4), nb_per_dev):
        if b not in out:
            out.append(b)
    while len(out) < 4:
        out.append(out[-1])
    return tuple(out)


def stratified_bucket(gmax: int, nb_per_dev: int) -> int:
    """The smallest bucket that holds ``gmax`` blocks (``phase_e_stratified.py:262-265``)."""
    return int(_lib.query("oc_stratified_bucket", int(nb_per_dev), int(gmax)))


def stratified_allgather_attention(q, k_shard, v_shard, active_indices, num_active, group=None,
                                   block_size: int = BLOCK_SIZE):
    """``build_stratified`` (``phase_e_stratified.py:164-273``): the global max
    count (all-reduce MAX, the reference's pmax) picks a capacity bucket;
    every rank sends its first ``bucket`` retained blocks; the gathered
    blocks at local position < count of their rank are attended to.
    Returns ((Sq, Hq, D) bfloat16, bucket).  The bucket is read on the host
    (one integer) because it sizes the collective."""
    k = _lib.as_device(k_shard).contiguous()
    v = _lib.as_device(v_shard, device=k.device).contiguous()
    nb = k.shape[0] // block_size
    na = _lib.as_device(num_active, device=k.device, dtype=torch.int32).reshape(1)
    gmax = na.clone()
    dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=group)
    bucket = stratified_bucket(int(gmax.item()), nb)
    kp = pack_active_blocks(k, active_indices, na, bucket, block_size)
    vp = pack_active_blocks(v, active_indices, na, bucket, block_size)
    all_counts = count_sync(na, group)
    k_all, v_all = alltoallv_exchange(kp, vp, group)
    order, total, _ = global_block_index(all_counts, bucket)
    return _attend_gathered(q, k_all, v_all, order, total, block_size), bucket


def sequence_parallel_attention(q, k_shard, v_shard, block_mask, group=None, block_size: int = BLOCK_SIZE):
    """Attention over the union of all ranks' retained blocks with no K/V
    movement: each rank attends to its own retained blocks, producing the
    unnormalised (m, l, o) of every query row; an all-gather of those P
    partials and a log-sum-exp merge give the result (the online-softmax
    combine of ``distributed_attention.py:95-128`` across shards).  Returns
    (Sq, Hq, D) bfloat16 on every rank."""
    q4, k4, v4, _ = _core.batched_qkv(q, k_shard, v_shard)
    active_indices, num_active = stream_compact(block_mask)
    nb = k4.shape[1] // block_size
    m, l, o = _core.partial_attend(q4, k4, v4, active_indices.reshape(1, -1), num_active, block_size,
                                   max_blocks=nb)
    P = _world(group)
    gm = _all_gather_cat(m.unsqueeze(0), group)
    gl = _all_gather_cat(l.unsqueeze(0), group)
    go = _all_gather_cat(o.unsqueeze(0), group)
    out = _core.merge_partials(gm.reshape(P, -1), gl.reshape(P, -1), go.reshape(P, -1, o.shape[-1]),
                               tuple(q4.shape[1:]), torch.bfloat16)
    return out


def ici_data_volume(num_blocks_per_device: int, num_devices: int, active_counts, num_heads: int,
                    head_dim: int, dtype_bytes: int = 2):
    """Exchange byte accounting (``distributed_attention.py:198-223``)."""
    per_block = BLOCK_SIZE * num_heads * head_dim * dtype_bytes
    dense = num_blocks_per_device * num_devices * per_block
    sparse = sum(int(c) for c in active_counts) * per_block
    return {
        "dense_bytes": dense,
        "sparse_bytes": sparse,
        "savings_bytes": dense - sparse,
        "savings_pct": (1 - sparse / dense) * 100 if dense > 0 else 0.0,
    }


__all__ = [
    "BLOCK_SIZE", "stream_compact", "distributed_orthocache_attention", "stratified_buckets", "stratified_bucket",
    "stratified_allgather_attention", "sequence_parallel_attention", "ici_data_volume",
]
