"""Write-time spectral metadata of a KV cache.

The reference's design notes make ζ query-independent on purpose: "It is a
structural property of the key block, computed once when the block is written
to the KV cache and stored as a static scalar metadata entry"
(``docs/mathematical_framework.md:244-250``).  The query-aware bound needs only
two more per-block quantities that do not depend on the query either: the DC
coefficient of each channel (the block mean times sqrt(512)) and the AC energy
E_AC (``spectral_energy.py:150-177``).  This module keeps the three, per
(batch, block, KV head), in device memory:

    cache = SpectralMetadataCache.from_keys(keys)        # one scorer pass
    cache.update_blocks(keys, first_block=j, num_blocks=1)   # block j rewritten
    keep, bound_max = cache.multiband_mask(q, tau, zeta_max)  # reads 0.5 MB, not |K|
    out, keep, perm, count = cache.decode_step(q, keys, values, tau)  # gates + attention, one launch

``multiband_mask`` gives the same mask as ``compute_multiband_mask`` on the
same keys (up to float32 summation order in the bound, as the fused scorer).
At 64K tokens, 8 KV heads and head_dim 128 the cache is 128 x 8 x (128 + 2)
floats = 0.53 MB against 134 MB of keys.
"""
from __future__ import annotations

import torch

from . import _lib

BLOCK = 512


class SpectralMetadataCache:
    """dc (B, nb, H, D), e_ac (B, nb, H), zeta (B, nb, H) float32 on the device."""

    def __init__(self, batch, num_blocks, kv_heads, head_dim, device=None):
        _lib.require_cuda()
        device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.batch, self.num_blocks, self.kv_heads, self.head_dim = batch, num_blocks, kv_heads, head_dim
        self.dc = torch.zeros((batch, num_blocks, kv_heads, head_dim), dtype=torch.float32, device=device)
        self.e_ac = torch.zeros((batch, num_blocks, kv_heads), dtype=torch.float32, device=device)
        self.zeta = torch.zeros((batch, num_blocks, kv_heads), dtype=torch.float32, device=device)

    @classmethod
    def from_keys(cls, keys):
        """Metadata of every block of keys (S, H, D) or (B, S, H, D)."""
        k = _batched(keys)
        B, S, H, D = k.shape
        if S % BLOCK:
            raise ValueError(f"seq_len {S} is not a multiple of 512")
        cache = cls(B, S // BLOCK, H, D, device=k.device)
        cache.update_blocks(keys, 0, S // BLOCK)
        return cache

    def update_blocks(self, keys, first_block, num_blocks):
        """Recompute the metadata of blocks first_block .. first_block +
        num_blocks - 1 from the full key tensor (only those blocks' keys are
        read): the call to make after writing or overwriting them."""
        k = _batched(keys)
        B, S, H, D = k.shape
        if (B, H, D) != (self.batch, self.kv_heads, self.head_dim):
            raise ValueError(f"keys {tuple(k.shape)} do not match the cache ({self.batch}, *, {self.kv_heads}, "
                             f"{self.head_dim})")
        if first_block < 0 or num_blocks < 0 or first_block + num_blocks > min(self.num_blocks, S // BLOCK):
            raise ValueError(f"blocks [{first_block}, {first_block + num_blocks}) outside the cache")
        if num_blocks == 0:
            return
        dt = _lib.dtype_code(k)
        sl = slice(first_block, first_block + num_blocks)
        whole = first_block == 0 and num_blocks == self.num_blocks and S == self.num_blocks * BLOCK
        for b in range(B) if not whole else [None]:
            kb = k if b is None else k[b:b + 1]
            kb = kb[:, first_block * BLOCK:(first_block + num_blocks) * BLOCK].contiguous()
            rows = kb.shape[0]
            dc = torch.empty((rows, num_blocks, H, D), dtype=torch.float32, device=k.device)
            e_ac = torch.empty((rows, num_blocks, H), dtype=torch.float32, device=k.device)
            zeta = torch.empty((rows, num_blocks, H), dtype=torch.float32, device=k.device)
            _lib.call("oc_block_metadata", _lib.ptr(kb), dt, rows, num_blocks * BLOCK, H, D, _lib.ptr(dc),
                      _lib.ptr(e_ac), _lib.ptr(zeta), _lib.stream_ptr(k.device))
            bs = slice(None) if b is None else slice(b, b + 1)
            self.dc[bs, sl] = dc
            self.e_ac[bs, sl] = e_ac
            self.zeta[bs, sl] = zeta

    def multiband_mask(self, q, tau, zeta_max=5.0, want_bounds=False):
        """Two-gate keep mask (``spectral_energy.py:199-234``) from the cached
        metadata.  q (Sq, Hq, D) or (B, Sq, Hq, D).  Returns keep (B, nb, H)
        bool and bound_max (B, nb, H) float32 (the batch dimension dropped for
        a 3-D q), plus bounds (B, Sq, nb, Hq) when want_bounds."""
        qq = _lib.as_device(q, device=self.dc.device)
        batched = qq.dim() == 4
        if not batched:
            qq = qq.unsqueeze(0)
        if qq.dtype not in (torch.float32, torch.bfloat16):
            qq = qq.float()
        qq = qq.contiguous()
        B, Sq, Hq, D = qq.shape
        if B != self.batch or D != self.head_dim or Hq % self.kv_heads:
            raise ValueError(f"q {tuple(qq.shape)} does not match the cache")
        nb, H = self.num_blocks, self.kv_heads
        keep = torch.empty((B, nb, H), dtype=torch.uint8, device=qq.device)
        bmax = torch.empty((B, nb, H), dtype=torch.float32, device=qq.device)
        bounds = torch.empty((B, Sq, nb, Hq), dtype=torch.float32, device=qq.device) if want_bounds else None
        _lib.call("oc_score_from_metadata", _lib.ptr(self.dc), _lib.ptr(self.e_ac), _lib.ptr(self.zeta),
                  _lib.ptr(qq), _lib.dtype_code(qq), B, nb, H, D, Sq, Hq, float(tau), float(zeta_max),
                  _lib.ptr(bmax), _lib.ptr(bounds), _lib.ptr(keep), _lib.stream_ptr(qq.device))
        keep = keep.bool()
        if not batched:
            keep, bmax = keep[0], bmax[0]
            bounds = bounds[0] if bounds is not None else None
        return (keep, bmax, bounds) if want_bounds else (keep, bmax)

    def decode_step(self, q, keys, values, tau, zeta_max=5.0, workspace=None):
        """One decode step over the retained blocks with the gates from this
        cache (``oc_decode_step_from_metadata``: one fused launch for bf16,
        head_dim 128, <= 8 query rows per KV head; separate kernels
        otherwise).  q (B, Sq, Hq, D); keys, values (B, S, H, D) of the same
        dtype, S = num_blocks * 512.  ``workspace``: a uint8 device tensor
        kept by the caller across steps (zero-filled once; allocated here when
        None).  Returns out (B, Sq, Hq, D) bfloat16, keep (B, nb, H) bool,
        perm (B, nb) and count (B) int32."""
        k, v = _batched(keys), _batched(values)
        qq = _lib.as_device(q, device=k.device)
        if qq.dim() != 4:
            raise ValueError(f"q must be (B, Sq, Hq, D), got {tuple(qq.shape)}")
        qq = qq.to(k.dtype).contiguous()
        B, Sq, Hq, D = qq.shape
        _, S, H, _ = k.shape
        if (B, H, D) != (self.batch, self.kv_heads, self.head_dim) or S != self.num_blocks * BLOCK or \
                v.shape != k.shape or Hq % H:
            raise ValueError(f"q {tuple(qq.shape)}, keys {tuple(k.shape)}, values {tuple(v.shape)} do not match "
                             f"the cache")
        nb = self.num_blocks
        need = _lib.query("oc_decode_step_workspace_bytes", B, Sq, Hq, H, D, S)
        if workspace is None:
            workspace = torch.zeros((need,), dtype=torch.uint8, device=k.device)
        elif workspace.numel() < need:
            raise ValueError(f"workspace of {workspace.numel()} bytes, need {need}")
        keep = torch.empty((B, nb, H), dtype=torch.uint8, device=k.device)
        perm = torch.empty((B, nb), dtype=torch.int32, device=k.device)
        count = torch.empty((B,), dtype=torch.int32, device=k.device)
        out = torch.empty((B, Sq, Hq, D), dtype=torch.bfloat16, device=k.device)
        _lib.call("oc_decode_step_from_metadata", _lib.ptr(qq), _lib.ptr(k), _lib.ptr(v), _lib.dtype_code(k),
                  _lib.ptr(self.dc), _lib.ptr(self.e_ac), _lib.ptr(self.zeta), B, Sq, Hq, H, D, S, float(tau),
                  float(zeta_max), _lib.ptr(keep), _lib.ptr(perm), _lib.ptr(count), _lib.ptr(out), 1,
                  _lib.ptr(workspace), workspace.numel(), _lib.stream_ptr(k.device))
        return out, keep.bool(), perm, count


def _batched(keys):
    k = _lib.as_device(keys)
    if k.dim() == 3:
        k = k.unsqueeze(0)
    if k.dim() != 4:
        raise ValueError(f"keys must be (S, H, D) or (B, S, H, D), got {tuple(k.shape)}")
    if k.dtype not in (torch.float32, torch.bfloat16):
        k = k.float()
    return k.contiguous()
