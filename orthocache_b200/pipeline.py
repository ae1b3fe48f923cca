"""End-to-end entry point (reference: src/orthocache/pipeline.py).

``orthocache_forward`` runs the reference's flow — ζ, optional auto-τ, the
two-gate mask, then compact or sparse attention — with one pass of the fused
scorer over the keys (the reference transforms the keys up to four times).
"""
from __future__ import annotations

import math
import time

import torch

from . import _core, _lib
from .spectral_energy import score_blocks

_MODES = ("dense", "sparse", "compact")


def _sync():
    torch.cuda.synchronize()


def _dense_attention(q, keys, values, head_dim=None):
    """Plain softmax attention over every key (``pipeline.py:160-165``)."""
    qq, k, v, batched = _core.batched_qkv(q, keys, values)
    B, S = k.shape[0], k.shape[1]
    bs = 512 if S % 512 == 0 else 64
    if S % bs:
        raise ValueError(f"dense attention needs seq_len divisible by 64, got {S}")
    nb = S // bs
    idx = torch.arange(nb, dtype=torch.int32, device=k.device)
    cnt = torch.full((1,), nb, dtype=torch.int32, device=k.device)
    out = _core.attend(qq, k, v, idx, cnt, bs, idx_stride=0, count_stride=0)
    return out if batched else out[0]


def _compute_auto_tau(q, keys, block_size=512):
    """mean - std (population) of the per-(block, head) max bound (``pipeline.py:168-176``).

    Returned as a 0-d float32 device tensor."""
    bm = score_blocks(keys, q, block_size=block_size, want=("bound_max",))["bound_max"]
    return bm.mean() - bm.std(unbiased=False)


def orthocache_forward(q, keys, values, block_size: int = 512, zeta_max: float = 5.0,
                       tau: float | None = None, mode: str = "compact"):
    """Full pipeline: spectral analysis -> two-gate eviction -> attention (``pipeline.py:33-157``).

    Returns (output (Sq, H, D) in q's dtype, metadata dict with the reference's keys).
    """
    if mode not in _MODES:
        raise ValueError(f"Unknown mode: {mode!r}. Use 'dense', 'sparse', or 'compact'.")
    qq, k, v, batched = _core.batched_qkv(q, keys, values)
    B, S, H, D = k.shape
    Sq = qq.shape[1]
    num_blocks = S // block_size
    metadata = {
        "mode": mode, "seq_len_q": Sq, "seq_len_k": S, "num_blocks": num_blocks,
        "num_heads": H, "head_dim": D, "block_size": block_size, "zeta_max": zeta_max,
    }
    if mode == "dense":
        t0 = time.perf_counter()
        out = _dense_attention(qq, k, v, D)
        _sync()
        metadata["latency_ms"] = (time.perf_counter() - t0) * 1000
        metadata["eviction_rate"] = 0.0
        return (out if batched else out[0]), metadata

    t_spec = time.perf_counter()
    sc = score_blocks(k, qq, block_size=block_size, want=("zeta", "bound_max"))
    zeta, bmax = sc["zeta"], sc["bound_max"]
    if tau is None:
        tau_dev = (bmax.mean() - bmax.std(unbiased=False)).reshape(1).float()
        tau = float(tau_dev.item())
        metadata["tau_auto"] = True
    else:
        tau_dev = None
        metadata["tau_auto"] = False
    metadata["tau"] = tau
    keep = torch.empty(bmax.shape, dtype=torch.uint8, device=k.device)
    _lib.call("oc_apply_gates", _lib.ptr(bmax), _lib.ptr(zeta), bmax.numel(), _lib.ptr(tau_dev),
              float(tau), float(zeta_max), _lib.ptr(keep), _lib.stream_ptr(k.device))
    _sync()
    metadata["spectral_ms"] = (time.perf_counter() - t_spec) * 1000

    z = zeta.mean(dim=-1)  # mean over heads, per block (pipeline.py:123)
    metadata["zeta_mean"] = float(z.mean())
    metadata["zeta_std"] = float(z.std(unbiased=False))
    metadata["zeta_min"] = float(z.min())
    metadata["zeta_max_observed"] = float(z.max())

    t_attn = time.perf_counter()
    if mode == "compact":
        perm, count = _core.compact(keep, batched=True)
        out = _core.attend(qq, k, v, perm, count, block_size)
        retained = int(count.sum().item()) if batched else int(count[0].item())
        metadata["compact_num_active"] = retained
    else:  # sparse: per-head masks
        perm, count = _core.compact_per_head(keep)
        out = _core.attend(qq, k, v, perm, count, block_size, idx_stride=H * num_blocks,
                           idx_head_stride=num_blocks, count_stride=H, count_head_stride=1)
        _core.fill_empty_heads(out, v, count, H, 1)
        un, uc = _core.compact(keep, batched=True)
        retained = int(uc.sum().item()) if batched else int(uc[0].item())
    _sync()
    metadata["blocks_retained"] = retained
    metadata["blocks_evicted"] = num_blocks * B - retained
    metadata["eviction_rate"] = 1.0 - retained / (num_blocks * B) if num_blocks else 0.0
    t_end = time.perf_counter()
    metadata["attention_ms"] = (t_end - t_attn) * 1000
    metadata["total_ms"] = (t_end - t_spec) * 1000
    return (out if batched else out[0]), metadata
