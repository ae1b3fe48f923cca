"""Sequence-parallel exchange and attention over ``torch.distributed``.

Drop-in counterparts of the reference's multi-device path (j-arndt/orthocache
v0.3.0):

  ``alltoallv.py``             stream_compact :44-75, count_sync :80-108,
                               compute_offsets :113-145, pack_active_blocks
                               :150-212, alltoallv_exchange :217-259,
                               unpack_received_blocks :264-335,
                               alltoallv_kv_exchange :340-440
  ``distributed_attention.py`` distributed_orthocache_attention :131-195,
                               ici_data_volume :198-223
  ``benchmarks/phase_e_stratified.py``  build_stratified :164-273

The reference's ``axis_name`` (a pmap axis) becomes a ``torch.distributed``
process group: NCCL between GPUs (one process per GPU), gloo for host-side
tests.  Block data moves only through the CUDA kernels of
``liborthocache_b200.so`` (block gather, exchange index, attention, merge);
the collectives are ``torch.distributed`` calls; the only host-side
arithmetic is on the P per-device counts.

Exchange semantics.  ``alltoallv_exchange`` returns every device's packed
buffer concatenated in rank order (the (P * max_tokens, H, D) layout that
``unpack_received_blocks`` and the reference's docstring describe), i.e. an
all-gather of the packed buffers.

Three ways to run attention across P sequence shards are provided:
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


# ---------------------------------------------------------------------------
# the same exchanges through the C ABI over NCCL (orthocache_b200.comm.NcclComm)
# ---------------------------------------------------------------------------
def _exchange_buffers(k, P, nb, heads, block_size):
    cap = P * nb * block_size
    kr = torch.empty((cap, heads, k.shape[2]), dtype=k.dtype, device=k.device)
    vr = torch.empty_like(kr)
    ws_bytes = _lib.query("oc_exchange_workspace_bytes", nb, k.shape[1], k.shape[2], _lib.dtype_code(k), block_size)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=k.device)
    counts = torch.empty((P,), dtype=torch.int32, device=k.device)
    return kr, vr, ws, ws_bytes, counts


def stratified_exchange(comm, k_shard, v_shard, active_indices, num_active, block_size: int = BLOCK_SIZE):
    """``build_stratified``'s exchange (``phase_e_stratified.py:164-273``) in one
    C-ABI call (``oc_exchange_stratified``): count all-gather, bucket, packed
    all-gather of every rank's first ``bucket`` retained K/V blocks, valid-slot
    index.  Returns (k_recv, v_recv, all_counts, order, total, bucket); k_recv
    holds P chunks of ``bucket`` blocks in rank order."""
    import ctypes
    k = _lib.as_device(k_shard).contiguous()
    v = _lib.as_device(v_shard, device=k.device).contiguous()
    nb = k.shape[0] // block_size
    P = comm.size
    idx = _lib.as_device(active_indices, device=k.device, dtype=torch.int32).contiguous()
    cnt = _core.count_tensor(_lib.as_device(num_active, device=k.device), k.device)
    kr, vr, ws, ws_bytes, counts = _exchange_buffers(k, P, nb, k.shape[1], block_size)
    order = torch.empty((P * nb,), dtype=torch.int32, device=k.device)
    total = torch.empty((1,), dtype=torch.int32, device=k.device)
    bucket = ctypes.c_int(0)
    _lib.call("oc_exchange_stratified", comm.ptr, _lib.ptr(k), _lib.ptr(v), _lib.dtype_code(k), _lib.ptr(idx),
              _lib.ptr(cnt), nb, k.shape[1], k.shape[2], block_size, _lib.ptr(kr), _lib.ptr(vr), _lib.ptr(counts),
              _lib.ptr(order), _lib.ptr(total), ctypes.byref(bucket), _lib.ptr(ws), ws_bytes,
              _lib.stream_ptr(k.device))
    b = bucket.value
    return kr[:P * b * block_size], vr[:P * b * block_size], counts, order[:P * b], total, b


def alltoallv_heads(comm, k_shard, v_shard, active_indices, num_active, block_size: int = BLOCK_SIZE):
    """AllToAllv of the retained blocks by KV head (``oc_alltoallv_heads``):
    rank r receives every rank's retained blocks of its own KV heads
    r*H/P .. (r+1)*H/P - 1, in rank order.  Returns (k_recv, v_recv,
    all_counts, total) with k_recv (total * block_size, H/P, D)."""
    import ctypes
    k = _lib.as_device(k_shard).contiguous()
    v = _lib.as_device(v_shard, device=k.device).contiguous()
    nb, H = k.shape[0] // block_size, k.shape[1]
    P = comm.size
    if H % P:
        raise ValueError(f"kv_heads {H} is not a multiple of the {P} ranks")
    idx = _lib.as_device(active_indices, device=k.device, dtype=torch.int32).contiguous()
    cnt = _core.count_tensor(_lib.as_device(num_active, device=k.device), k.device)
    kr, vr, ws, ws_bytes, counts = _exchange_buffers(k, P, nb, H // P, block_size)
    total = ctypes.c_int(0)
    _lib.call("oc_alltoallv_heads", comm.ptr, _lib.ptr(k), _lib.ptr(v), _lib.dtype_code(k), _lib.ptr(idx),
              _lib.ptr(cnt), nb, H, k.shape[2], block_size, _lib.ptr(kr), _lib.ptr(vr), _lib.ptr(counts),
              ctypes.byref(total), _lib.ptr(ws), ws_bytes, _lib.stream_ptr(k.device))
    t = total.value
    return kr[:t * block_size], vr[:t * block_size], counts, t


def head_partitioned_attention(q, k_shard, v_shard, block_mask, comm, block_size: int = BLOCK_SIZE):
    """Attention over the union of all ranks' retained blocks with the KV heads
    partitioned across ranks: ``alltoallv_heads`` brings each rank the
    retained blocks of its KV heads from every shard, each rank attends for
    the query heads of those KV heads, and the outputs are all-gathered.
    Returns (Sq, Hq, D) bfloat16 on every rank."""
    q4, k4, v4, _ = _core.batched_qkv(q, k_shard, v_shard)
    Sq, Hq, D = q4.shape[1:]
    Hkv = k4.shape[2]
    P, r = comm.size, comm.rank
    G, hper = Hq // Hkv, Hkv // P
    active_indices, num_active = stream_compact(block_mask)
    kr, vr, _, total = alltoallv_heads(comm, k4[0], v4[0], active_indices, num_active, block_size)
    q_mine = q4[:, :, r * hper * G:(r + 1) * hper * G].contiguous()
    if total == 0:
        mine = torch.zeros((Sq, hper * G, D), dtype=torch.bfloat16, device=q4.device)
    else:
        idx = torch.arange(total, dtype=torch.int32, device=q4.device).reshape(1, -1)
        cnt = torch.tensor([total], dtype=torch.int32, device=q4.device)
        mine = _core.attend(q_mine, kr.unsqueeze(0), vr.unsqueeze(0), idx, cnt, block_size,
                            out_dtype=torch.bfloat16)[0]
    gathered = torch.empty((P,) + tuple(mine.shape), dtype=mine.dtype, device=mine.device)
    dist.all_gather_into_tensor(gathered, mine.contiguous(), group=comm.group)
    return gathered.permute(1, 0, 2, 3).reshape(Sq, Hq, D)


class ShardedDecoder:
    """Sequence-parallel decode through ``oc_decode_step_sharded``.

    ``peer=True`` (default) maps every rank's exchange region into every
    other rank (``oc_sharded_connect``, collective): each layer is then one
    fused kernel that merges the shards' (m, l, o) partials over NVLink peer
    stores.  Otherwise (or if mapping fails on any rank) each layer is the
    fused kernel, an NCCL all-gather of the partials and a merge kernel.
    Holds the zero-filled workspace between calls."""

    def __init__(self, comm, q_heads, kv_heads, head_dim, seq_len, batch=1, q_len=1, peer=True):
        self.comm = comm
        self.shape = (batch, q_len, q_heads, kv_heads, head_dim, seq_len)
        dev = comm.device
        self.ws_bytes = _lib.query("oc_decode_step_sharded_workspace_bytes", comm.size, batch, q_len, q_heads,
                                   kv_heads, head_dim, seq_len)
        self.ws = torch.zeros((self.ws_bytes,), dtype=torch.uint8, device=dev)
        self.peer = False
        if peer:
            lib = _lib.load()
            rc = lib.oc_sharded_connect(comm.ptr, _lib.ptr(self.ws), self.ws_bytes, batch, q_len, q_heads, kv_heads,
                                        head_dim, seq_len, _lib.stream_ptr(dev))
            self.peer = rc == 0
            self.connect_error = None if rc == 0 else lib.oc_last_error().decode(errors="replace")
        nb = seq_len // BLOCK_SIZE
        self.keep = torch.empty((batch, nb, kv_heads), dtype=torch.uint8, device=dev)
        self.perm = torch.empty((batch, nb), dtype=torch.int32, device=dev)
        self.count = torch.empty((batch,), dtype=torch.int32, device=dev)
        self.out = torch.empty((batch, q_len, q_heads, head_dim), dtype=torch.bfloat16, device=dev)

    def __call__(self, q, k, v, tau, zeta_max):
        B, Sq, Hq, Hkv, D, S = self.shape
        _lib.call("oc_decode_step_sharded", self.comm.ptr, _lib.ptr(q), _lib.ptr(k), _lib.ptr(v),
                  _lib.dtype_code(k), B, Sq, Hq, Hkv, D, S, float(tau), float(zeta_max), _lib.ptr(self.keep),
                  _lib.ptr(self.perm), _lib.ptr(self.count), _lib.ptr(self.out), 1, _lib.ptr(self.ws),
                  self.ws_bytes, _lib.stream_ptr(k.device))
        return self.out

    def close(self):
        if self.peer:
            _lib.load().oc_sharded_disconnect(_lib.ptr(self.ws))
            self.peer = False


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
    "stream_compact", "count_sync", "compute_offsets", "pack_active_blocks", "alltoallv_exchange",
    "global_block_index", "unpack_received_blocks", "alltoallv_kv_exchange",
    "distributed_orthocache_attention", "stratified_buckets", "stratified_bucket",
    "stratified_allgather_attention", "sequence_parallel_attention", "ici_data_volume",
    "stratified_exchange", "alltoallv_heads", "head_partitioned_attention", "ShardedDecoder",
]
