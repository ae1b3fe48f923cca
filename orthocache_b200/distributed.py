"""Sequence-parallel exchanges and attention through the C ABI over an NCCL
communicator (``orthocache_b200.comm.NcclComm``), and the one-kernel sharded
decode layer (``ShardedDecoder``).

The reference-named drop-ins live in their module twins and are re-exported
here: :mod:`orthocache_b200.alltoallv` (``alltoallv.py``: count sync,
offsets, pack, exchange, unpack) and :mod:`orthocache_b200.distributed_attention`
(``distributed_attention.py``, ``benchmarks/phase_e_stratified.py``).  This
module adds what the reference has no entry point for: the stratified
exchange and the per-peer AllToAllv by KV head as single C-ABI calls
(``oc_exchange_stratified``, ``oc_alltoallv_heads``), attention partitioned
by KV head, and the sharded decode layer whose partials cross NVLink inside
the kernel.
"""
from __future__ import annotations

import torch
import torch.distributed as dist  # noqa: F401

from . import _lib
from . import _core
from .alltoallv import (  # noqa: F401
    BLOCK_SIZE, _world, _all_gather_cat, stream_compact, count_sync, compute_offsets, pack_active_blocks,
    alltoallv_exchange, global_block_index, unpack_received_blocks, alltoallv_kv_exchange,
)
from .distributed_attention import (  # noqa: F401
    _attend_gathered, distributed_orthocache_attention, stratified_buckets, stratified_bucket,
    stratified_allgather_attention, sequence_parallel_attention, ici_data_volume,
)


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


__all__ = [
    "stream_compact", "count_sync", "compute_offsets", "pack_active_blocks", "alltoallv_exchange",
    "global_block_index", "unpack_received_blocks", "alltoallv_kv_exchange",
    "distributed_orthocache_attention", "stratified_buckets", "stratified_bucket",
    "stratified_allgather_attention", "sequence_parallel_attention", "ici_data_volume",
    "stratified_exchange", "alltoallv_heads", "head_partitioned_attention", "ShardedDecoder",
]
