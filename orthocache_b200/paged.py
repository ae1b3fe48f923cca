"""Paged KV cache with write-time spectral metadata.

The reference attends through block indices only (``indirect_attention.py:
155-159``), so its index table doubles as a page table: keys and values live
in a pool of fixed-size pages shared by every sequence, and a per-sequence
block table maps logical block j to a pool page.  The query-independent part
of the scoring (DC coefficients, E_AC, ζ — ``docs/mathematical_framework.md:
242-250``) is computed once per page when the page is written, so a decode
step reads the pool's pages only for the retained blocks:

    cache = PagedKVCache(num_pages, kv_heads, head_dim)
    cache.write(pages, k_blocks, v_blocks)             # keys, values and metadata of the pages
    out, keep, perm, count = cache.attend(q, block_table, num_blocks, tau, zeta_max)

Every step is a call into ``liborthocache_b200.so``: ``oc_block_metadata``
(write), ``oc_score_from_metadata_paged`` (gates of the logical blocks),
``oc_stream_compact`` (union compaction), ``oc_indirect_attention_paged`` or,
for long bfloat16 query chunks, ``oc_prefill_attention_paged``.
"""
from __future__ import annotations

import torch

from . import _core, _lib

PAGE = 512


class PagedKVCache:
    """A pool of ``num_pages`` pages of 512 tokens, (kv_heads, head_dim) each."""

    def __init__(self, num_pages, kv_heads, head_dim, dtype=torch.bfloat16, device=None):
        _lib.require_cuda()
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.num_pages, self.kv_heads, self.head_dim = int(num_pages), int(kv_heads), int(head_dim)
        self.k = torch.zeros((num_pages * PAGE, kv_heads, head_dim), dtype=dtype, device=dev)
        self.v = torch.zeros_like(self.k)
        f32 = dict(dtype=torch.float32, device=dev)
        self.dc = torch.zeros((num_pages, kv_heads, head_dim), **f32)
        self.e_ac = torch.zeros((num_pages, kv_heads), **f32)
        self.zeta = torch.full((num_pages, kv_heads), float("inf"), **f32)  # unwritten pages fail the ζ gate

    @property
    def device(self):
        return self.k.device

    def write(self, pages, k_blocks, v_blocks):
        """Store blocks (n * 512, kv_heads, head_dim) into the given n pages and
        compute their metadata (one scorer pass over the new keys)."""
        pages = torch.as_tensor(pages, dtype=torch.long, device=self.device).reshape(-1)
        n = pages.numel()
        kb = _lib.as_device(k_blocks, device=self.device, dtype=self.k.dtype).reshape(n, PAGE, self.kv_heads,
                                                                                     self.head_dim)
        vb = _lib.as_device(v_blocks, device=self.device, dtype=self.v.dtype).reshape(n, PAGE, self.kv_heads,
                                                                                     self.head_dim)
        kc = kb.reshape(n * PAGE, self.kv_heads, self.head_dim).contiguous()
        dc = torch.empty((n, self.kv_heads, self.head_dim), dtype=torch.float32, device=self.device)
        e_ac = torch.empty((n, self.kv_heads), dtype=torch.float32, device=self.device)
        zeta = torch.empty_like(e_ac)
        _lib.call("oc_block_metadata", _lib.ptr(kc), _lib.dtype_code(kc), 1, n * PAGE, self.kv_heads,
                  self.head_dim, _lib.ptr(dc), _lib.ptr(e_ac), _lib.ptr(zeta), _lib.stream_ptr(self.device))
        self.k.view(self.num_pages, PAGE, self.kv_heads, self.head_dim).index_copy_(0, pages, kb)
        self.v.view(self.num_pages, PAGE, self.kv_heads, self.head_dim).index_copy_(0, pages, vb)
        self.dc.index_copy_(0, pages, dc)
        self.e_ac.index_copy_(0, pages, e_ac)
        self.zeta.index_copy_(0, pages, zeta)

    def gates(self, q, block_table, num_blocks, tau, zeta_max):
        """Two-gate keep mask (B, num_blocks, kv_heads) of the logical blocks
        and the bound maxima, from the pages' metadata."""
        q4 = _lib.as_device(q, device=self.device)
        if q4.dim() == 3:
            q4 = q4.unsqueeze(0)
        q4 = q4.contiguous()
        table = _lib.as_device(block_table, device=self.device, dtype=torch.int32)
        if table.dim() == 1:
            table = table.unsqueeze(0)
        table = table.contiguous()
        B, Sq, Hq, D = q4.shape
        keep = torch.empty((B, num_blocks, self.kv_heads), dtype=torch.uint8, device=self.device)
        bmax = torch.empty((B, num_blocks, self.kv_heads), dtype=torch.float32, device=self.device)
        _lib.call("oc_score_from_metadata_paged", _lib.ptr(self.dc), _lib.ptr(self.e_ac), _lib.ptr(self.zeta),
                  self.num_pages, _lib.ptr(table), table.shape[1], _lib.ptr(q4), _lib.dtype_code(q4), B,
                  int(num_blocks), self.kv_heads, D, Sq, Hq, float(tau), float(zeta_max), _lib.ptr(bmax), None,
                  _lib.ptr(keep), _lib.stream_ptr(self.device))
        return keep, bmax, q4, table

    def attend(self, q, block_table, num_blocks, tau, zeta_max):
        """Decode / prefill step over the pool: gates from the metadata, union
        compaction, attention over the retained pages.  Returns (out (B, Sq,
        Hq, D), keep, perm, count)."""
        keep, _, q4, table = self.gates(q, block_table, num_blocks, tau, zeta_max)
        perm, count = _core.compact(keep, batched=True)
        B, Sq, Hq, D = q4.shape
        nb = int(num_blocks)
        out = torch.empty((B, Sq, Hq, D), dtype=q4.dtype, device=self.device)
        if _core.prefill_applies(q4, PAGE) and q4.dtype == self.k.dtype:
            ws_bytes = _lib.query("oc_prefill_attention_paged_workspace_bytes", B, nb)
            ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=self.device)
            name = "oc_prefill_attention_paged"
        else:
            ws_bytes = _lib.query("oc_indirect_attention_paged_workspace_bytes", B, Sq, Hq, self.kv_heads, D, PAGE,
                                  nb)
            ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=self.device)
            name = "oc_indirect_attention_paged"
        qq = q4.to(self.k.dtype)
        _lib.call(name, _lib.ptr(qq), _lib.ptr(self.k), _lib.ptr(self.v), _lib.dtype_code(self.k), _lib.ptr(table),
                  table.shape[1], _lib.ptr(perm), nb, _lib.ptr(count), 1, B, Sq, Hq, self.kv_heads, D,
                  self.num_pages, PAGE, nb, _lib.ptr(out), _lib.dtype_code(out), _lib.ptr(ws), ws_bytes,
                  _lib.stream_ptr(self.device))
        return out, keep, perm, count
