"""Shared host logic of the drop-in modules: mask compaction, the attention
call and lazily-synchronised metadata.  Every device computation is a call
into ``liborthocache_b200.so``."""
from __future__ import annotations

import torch

from . import _lib


class Meta(dict):
    """Metadata dict whose device scalars synchronise only when read.

    Values that are 0-d / 1-element tensors are returned as Python numbers;
    callables are evaluated on access.  ``raw(key)`` returns the stored object.
    """

    def __getitem__(self, key):
        v = dict.__getitem__(self, key)
        if callable(v) and not isinstance(v, torch.Tensor):
            v = v()
        if isinstance(v, torch.Tensor) and v.numel() == 1:
            v = v.item()
        return v

    def get(self, key, default=None):
        return self[key] if key in self else default

    def raw(self, key):
        return dict.__getitem__(self, key)

    def items(self):
        return [(k, self[k]) for k in self.keys()]

    def values(self):
        return [self[k] for k in self.keys()]


def compact(mask, batched=False):
    """Union-over-heads stream compaction on the device.

    mask: (nb,) or (nb, H) [batched: (B, nb) or (B, nb, H)], bool/uint8.
    Returns perm (B, nb) int32 and count (B,) int32 (device tensors).
    """
    m = _lib.as_device(mask)
    if not batched:
        m = m.unsqueeze(0)
    if m.dim() == 2:
        m = m.unsqueeze(-1)
    if m.dim() != 3:
        raise ValueError(f"block mask must be (nb,) or (nb, H) (batched: (B, nb[, H])), got {tuple(mask.shape)}")
    m = m.to(torch.uint8).contiguous()
    B, nb, H = m.shape
    perm = torch.empty((B, nb), dtype=torch.int32, device=m.device)
    count = torch.empty((B,), dtype=torch.int32, device=m.device)
    _lib.call("oc_stream_compact", _lib.ptr(m), B, nb, H, _lib.ptr(perm), _lib.ptr(count),
              _lib.stream_ptr(m.device))
    return perm, count


def compact_per_head(mask):
    """Per-(batch, head) compaction of a (B, nb, H) mask: perm (B, H, nb), count (B, H)."""
    m = _lib.as_device(mask).to(torch.uint8)
    B, nb, H = m.shape
    mt = m.permute(0, 2, 1).contiguous().reshape(B * H, nb, 1)
    perm = torch.empty((B * H, nb), dtype=torch.int32, device=m.device)
    count = torch.empty((B * H,), dtype=torch.int32, device=m.device)
    _lib.call("oc_stream_compact", _lib.ptr(mt), B * H, nb, 1, _lib.ptr(perm), _lib.ptr(count),
              _lib.stream_ptr(m.device))
    return perm.reshape(B, H, nb), count.reshape(B, H)


def batched_qkv(q, k, v, dtype=None):
    """Bring q (Sq,Hq,D)|(B,Sq,Hq,D) and k, v (S,H,D)|(B,S,H,D) to 4-D device tensors."""
    k = _lib.as_device(k)
    dt = dtype or k.dtype
    if dt not in (torch.float32, torch.bfloat16):
        dt = torch.float32
    k = k.to(dt)
    q = _lib.as_device(q, device=k.device, dtype=dt)
    v = _lib.as_device(v, device=k.device, dtype=dt)
    batched = k.dim() == 4
    if not batched:
        q, k, v = q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0)
    if q.dim() != 4 or k.shape != v.shape or q.shape[0] != k.shape[0] or q.shape[3] != k.shape[3]:
        raise ValueError(f"incompatible shapes q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)}")
    return q.contiguous(), k.contiguous(), v.contiguous(), batched


PREFILL_MIN_Q = 64


def prefill_applies(q, block_size):
    """Long query chunks (chunked prefill) go to the tensor-core kernel
    ``oc_prefill_attention``: bfloat16, head_dim 128, blocks of a multiple of
    128 tokens and at least ``PREFILL_MIN_Q`` query positions (its row tiles
    are 128 positions of one query head, so shorter chunks would be mostly
    padding and stay on the split-KV decode kernel)."""
    return (q.dtype == torch.bfloat16 and q.shape[-1] == 128 and block_size % 128 == 0
            and q.shape[1] >= PREFILL_MIN_Q)


def attend(q, k, v, idx, count, block_size, max_blocks=None, idx_stride=None, idx_head_stride=0,
           count_stride=1, count_head_stride=0, out_dtype=None):
    """Indirect block attention on 4-D tensors: ``oc_prefill_attention`` for
    long bfloat16 query chunks (``prefill_applies``), ``oc_indirect_attention``
    (split-KV) otherwise.

    q (B, Sq, Hq, D); k, v (B, S, Hkv, D); idx int32 index lists, count int32.
    Returns (B, Sq, Hq, D) in ``out_dtype`` (default q.dtype).
    """
    B, Sq, Hq, D = q.shape
    S, Hkv = k.shape[1], k.shape[2]
    nb = S // block_size
    if max_blocks is None:
        max_blocks = nb
    if idx_stride is None:
        idx_stride = idx.shape[-1] if idx.dim() >= 1 else 0
    out_dtype = out_dtype or q.dtype
    out = torch.empty((B, Sq, Hq, D), dtype=out_dtype, device=q.device)
    if prefill_applies(q, block_size):
        _lib.call("oc_prefill_attention", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.dtype_code(q),
                  _lib.ptr(idx), int(idx_stride), int(idx_head_stride), _lib.ptr(count), int(count_stride),
                  int(count_head_stride), B, Sq, Hq, Hkv, D, S, block_size, max_blocks,
                  _lib.ptr(out), _lib.dtype_code(out), _lib.stream_ptr(q.device))
        return out
    ws_bytes = _lib.query("oc_indirect_attention_workspace_bytes", B, Sq, Hq, Hkv, D, block_size, max_blocks)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    _lib.call("oc_indirect_attention", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.dtype_code(q),
              _lib.ptr(idx), int(idx_stride), int(idx_head_stride), _lib.ptr(count), int(count_stride),
              int(count_head_stride), B, Sq, Hq, Hkv, D, S, block_size, max_blocks,
              _lib.ptr(out), _lib.dtype_code(out), _lib.ptr(ws), ws_bytes, _lib.stream_ptr(q.device))
    return out


def partial_attend(q, k, v, idx, count, block_size, max_blocks=None, idx_stride=None):
    """(m, l, o) of one shard for the log-sum-exp merge (``oc_partial_attention``)."""
    B, Sq, Hq, D = q.shape
    S, Hkv = k.shape[1], k.shape[2]
    nb = S // block_size
    if max_blocks is None:
        max_blocks = nb
    if idx_stride is None:
        idx_stride = idx.shape[-1]
    rows = B * Sq * Hq
    f32 = dict(dtype=torch.float32, device=q.device)
    m = torch.empty((rows,), **f32)
    l = torch.empty((rows,), **f32)
    o = torch.empty((rows, D), **f32)
    ws_bytes = _lib.query("oc_indirect_attention_workspace_bytes", B, Sq, Hq, Hkv, D, block_size, max_blocks)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    _lib.call("oc_partial_attention", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.dtype_code(q),
              _lib.ptr(idx), int(idx_stride), 0, _lib.ptr(count), 1, 0, B, Sq, Hq, Hkv, D, S, block_size,
              max_blocks, _lib.ptr(m), _lib.ptr(l), _lib.ptr(o), _lib.ptr(ws), ws_bytes,
              _lib.stream_ptr(q.device))
    return m, l, o


def merge_partials(m, l, o, out_shape, out_dtype):
    """Combine P stacked (m, l, o) parts: m, l (P, rows), o (P, rows, D)."""
    P, rows = m.shape
    D = o.shape[-1]
    out = torch.empty(out_shape, dtype=out_dtype, device=m.device)
    _lib.call("oc_merge_partials", _lib.ptr(m.contiguous()), _lib.ptr(l.contiguous()), _lib.ptr(o.contiguous()),
              P, rows, D, _lib.ptr(out), _lib.dtype_code(out), _lib.stream_ptr(m.device))
    return out


def gather_blocks(src, perm, count, nb_dst, block_size, zero_tail=True, perm_stride=None):
    """dst[b, i] = src[b, perm[b, i]] for i < count[b] (``oc_gather_blocks``).

    src: (B, S, H, D) viewed as blocks of ``block_size`` tokens; returns
    (B, nb_dst * block_size, H, D).
    """
    B, S, H, D = src.shape
    nb_src = S // block_size
    dst = torch.empty((B, nb_dst * block_size, H, D), dtype=src.dtype, device=src.device)
    _lib.call("oc_gather_blocks", _lib.ptr(src), _lib.dtype_code(src), B, nb_src, block_size * H * D,
              _lib.ptr(perm), int(perm_stride if perm_stride is not None else perm.shape[-1]),
              _lib.ptr(count), _lib.ptr(dst), nb_dst, 1 if zero_tail else 0, _lib.stream_ptr(src.device))
    return dst


def count_tensor(n, device, batch=1):
    if isinstance(n, torch.Tensor):
        return n.to(device=device, dtype=torch.int32).reshape(-1).expand(batch).contiguous() \
            if n.numel() == 1 else n.to(device=device, dtype=torch.int32).contiguous()
    return torch.full((batch,), int(n), dtype=torch.int32, device=device)


def fill_empty_heads(out, v, count, count_stride, count_head_stride):
    """Rows of heads whose list is empty get mean(V) (reference -1e9 predication)."""
    B, Sq, Hq, D = out.shape
    S, Hkv = v.shape[1], v.shape[2]
    _lib.call("oc_empty_heads_mean", _lib.ptr(v), _lib.dtype_code(v), _lib.ptr(count), int(count_stride),
              int(count_head_stride), B, Sq, Hq, Hkv, D, S, _lib.ptr(out), _lib.dtype_code(out),
              _lib.stream_ptr(v.device))
    return out
