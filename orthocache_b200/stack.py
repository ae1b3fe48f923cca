"""A decode stack of OrthoCache attention layers over sequence-sharded KV
caches (the structure of the reference's 60-layer configuration: sliding-
window layers interleaved with global eviction layers).

* sliding layers attend densely to the last ``window`` tokens of the whole
  sequence (no eviction); with the sequence sharded across ranks those
  tokens live on the last rank, every other rank contributes an empty
  partial;
* global layers run the OrthoCache path on every shard: the fused scorer's
  two-gate keep mask (``compute_multiband_mask``, spectral_energy.py:199-234),
  the union compaction (compaction.py:28-100) and indirect attention over
  the retained blocks (indirect_attention.py:127-170); across ranks the
  shards' (m, l, o) partials are all-gathered and merged in log-sum-exp form
  (distributed_attention.py:95-128 applied across shards).

Every device computation is a call into ``liborthocache_b200.so``; buffers
are allocated once, so a step can be captured in a CUDA graph (N = 1).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib

BLOCK = 512


class DecodeStack:
    """Layers ``kinds`` ("sliding" / "global") of one rank's shard.

    q: (B, 1, Hq, D); k, v: (B, shard_len, Hkv, D) bfloat16 per layer.
    ``group``: a torch.distributed process group (NCCL) when the sequence is
    sharded over several ranks (rank r holds tokens r*shard_len ..
    (r+1)*shard_len - 1); None for one shard.
    """

    def __init__(self, kinds, batch, q_heads, kv_heads, head_dim, shard_len, window=1024, zeta_max=5.0,
                 group=None, device=None):
        _lib.require_cuda()
        if shard_len % BLOCK or window % BLOCK or window > shard_len:
            raise ValueError("shard_len and window must be multiples of 512 with window <= shard_len")
        self.kinds = list(kinds)
        for k in self.kinds:
            if k not in ("sliding", "global"):
                raise ValueError(f"unknown layer kind {k!r}")
        self.B, self.Hq, self.Hkv, self.D, self.S = batch, q_heads, kv_heads, head_dim, shard_len
        self.nb = shard_len // BLOCK
        self.zeta_max = float(zeta_max)
        self.group = group
        self.P = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.device = dev
        B, nb = batch, self.nb
        self.keep = torch.empty((B, nb, kv_heads), dtype=torch.uint8, device=dev)
        self.perm = torch.empty((B, nb), dtype=torch.int32, device=dev)
        self.count = torch.empty((B,), dtype=torch.int32, device=dev)
        # sliding window: the last window / 512 blocks of the sequence, on the last rank
        wb = window // BLOCK
        self.win_idx = torch.arange(nb - wb, nb, dtype=torch.int32, device=dev).repeat(B, 1).contiguous()
        on_last = self.rank == self.P - 1
        self.win_count = torch.full((B,), wb if on_last else 0, dtype=torch.int32, device=dev)
        self.wb = wb
        rows = B * 1 * q_heads
        self.rows = rows
        self.out = torch.empty((B, 1, q_heads, head_dim), dtype=torch.bfloat16, device=dev)
        self.ws_bytes = _lib.query("oc_indirect_attention_workspace_bytes", B, 1, q_heads, kv_heads, head_dim,
                                   BLOCK, nb)
        self.ws = torch.empty((max(self.ws_bytes, 1),), dtype=torch.uint8, device=dev)
        if self.P > 1:
            self.send = torch.empty((rows * (head_dim + 2),), dtype=torch.float32, device=dev)
            self.recv = torch.empty((self.P * rows * (head_dim + 2),), dtype=torch.float32, device=dev)

    def _attend(self, q, k, v, idx, count, max_blocks):
        st = _lib.stream_ptr(self.device)
        B, Hq, Hkv, D = self.B, self.Hq, self.Hkv, self.D
        if self.P == 1:
            _lib.call("oc_indirect_attention", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), 1, _lib.ptr(idx),
                      idx.shape[1], 0, _lib.ptr(count), 1, 0, B, 1, Hq, Hkv, D, self.S, BLOCK, max_blocks,
                      _lib.ptr(self.out), 1, _lib.ptr(self.ws), self.ws_bytes, st)
            return self.out
        r = self.rows
        _lib.call("oc_partial_attention", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), 1, _lib.ptr(idx), idx.shape[1], 0,
                  _lib.ptr(count), 1, 0, B, 1, Hq, Hkv, D, self.S, BLOCK, max_blocks, _lib.ptr(self.send),
                  _lib.ptr(self.send[r:]), _lib.ptr(self.send[2 * r:]), _lib.ptr(self.ws), self.ws_bytes, st)
        dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
        _lib.call("oc_merge_partials_packed", _lib.ptr(self.recv), self.P, r, D, _lib.ptr(self.out), 1, st)
        return self.out

    def layer(self, i, q, k, v, tau):
        """Layer i: returns out (B, 1, Hq, D) bfloat16 (a buffer reused by the
        next layer)."""
        if self.kinds[i] == "sliding":
            return self._attend(q, k, v, self.win_idx, self.win_count, self.wb)
        st = _lib.stream_ptr(self.device)
        _lib.call("oc_score_blocks", _lib.ptr(k), _lib.ptr(q), 1, self.B, self.S, self.Hkv, self.D, 1, self.Hq,
                  1, 64, 64, 256, 256, 512, float(tau), self.zeta_max, None, None, None, None, None, None, None,
                  _lib.ptr(self.keep), 0, st)
        _lib.call("oc_stream_compact", _lib.ptr(self.keep), self.B, self.nb, self.Hkv, _lib.ptr(self.perm),
                  _lib.ptr(self.count), st)
        return self._attend(q, k, v, self.perm, self.count, self.nb)

    def step(self, qs, ks, vs, taus, outs=None):
        """All layers once (one decode step); outs: optional list of tensors
        receiving each layer's output."""
        for i in range(len(self.kinds)):
            o = self.layer(i, qs[i], ks[i], vs[i], taus[i])
            if outs is not None:
                outs[i].copy_(o)
        return self.out
