"""End-to-end entry point (reference: src/orthocache/pipeline.py).

``orthocache_forward`` runs the reference's flow — ζ, optional auto-τ, the
two-gate mask, then compact or sparse attention — with one pass of the fused
scorer over the keys (the reference transforms the keys up to four times).
"""
from __future__ import annotations

import torch

from . import _core, _lib
from .spectral_energy import score_blocks

_MODES = ("dense", "sparse", "compact")


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


def _elapsed(e0, e1):
    """Milliseconds between two recorded CUDA events, read when asked for."""
    def read():
        e1.synchronize()
        return e0.elapsed_time(e1)
    return read


def orthocache_forward(q, keys, values, block_size: int = 512, zeta_max: float = 5.0,
                       tau: float | None = None, mode: str = "compact"):
    """Full pipeline: spectral analysis -> two-gate eviction -> attention (``pipeline.py:33-157``).

    Returns (output (Sq, H, D) in q's dtype, metadata dict with the reference's keys).
    Nothing here waits for the GPU: τ (auto: mean - std of the bounds, on the
    device), the ζ statistics, the retained counts and the timings (CUDA
    events) are device values that the metadata dict (``_core.Meta``) reads
    only when a key is accessed.
    """
    if mode not in _MODES:
        raise ValueError(f"Unknown mode: {mode!r}. Use 'dense', 'sparse', or 'compact'.")
    qq, k, v, batched = _core.batched_qkv(q, keys, values)
    B, S, H, D = k.shape
    Sq = qq.shape[1]
    num_blocks = S // block_size
    metadata = _core.Meta({
        "mode": mode, "seq_len_q": Sq, "seq_len_k": S, "num_blocks": num_blocks,
        "num_heads": H, "head_dim": D, "block_size": block_size, "zeta_max": zeta_max,
    })
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record()
    if mode == "dense":
        out = _dense_attention(qq, k, v, D)
        ev[1].record()
        metadata["latency_ms"] = _elapsed(ev[0], ev[1])
        metadata["eviction_rate"] = 0.0
        return (out if batched else out[0]), metadata

    sc = score_blocks(k, qq, block_size=block_size, want=("zeta", "bound_max"))
    zeta, bmax = sc["zeta"], sc["bound_max"]
    if tau is None:
        tau_dev = (bmax.mean() - bmax.std(unbiased=False)).reshape(1).float()
        metadata["tau"] = tau_dev.reshape(())
        metadata["tau_auto"] = True
        tau_host = 0.0  # unused: the gates read tau_dev
    else:
        tau_dev = None
        tau_host = float(tau)
        metadata["tau"] = tau_host
        metadata["tau_auto"] = False
    keep = torch.empty(bmax.shape, dtype=torch.uint8, device=k.device)
    _lib.call("oc_apply_gates", _lib.ptr(bmax), _lib.ptr(zeta), bmax.numel(), _lib.ptr(tau_dev),
              tau_host, float(zeta_max), _lib.ptr(keep), _lib.stream_ptr(k.device))
    ev[1].record()
    metadata["spectral_ms"] = _elapsed(ev[0], ev[1])

    z = zeta.mean(dim=-1)  # mean over heads, per block (pipeline.py:123)
    metadata["zeta_mean"] = z.mean()
    metadata["zeta_std"] = z.std(unbiased=False)
    metadata["zeta_min"] = z.min()
    metadata["zeta_max_observed"] = z.max()

    if mode == "compact":
        perm, count = _core.compact(keep, batched=True)
        out = _core.attend(qq, k, v, perm, count, block_size)
        retained = count.sum()
        metadata["compact_num_active"] = retained
    else:  # sparse: per-head masks
        perm, count = _core.compact_per_head(keep)
        out = _core.attend(qq, k, v, perm, count, block_size, idx_stride=H * num_blocks,
                           idx_head_stride=num_blocks, count_stride=H, count_head_stride=1)
        _core.fill_empty_heads(out, v, count, H, 1)
        un, uc = _core.compact(keep, batched=True)
        retained = uc.sum()
    ev[2].record()
    total = num_blocks * B
    metadata["blocks_retained"] = retained
    metadata["blocks_evicted"] = lambda: total - int(retained.item())
    metadata["eviction_rate"] = lambda: (1.0 - int(retained.item()) / total) if total else 0.0
    metadata["attention_ms"] = _elapsed(ev[1], ev[2])
    metadata["total_ms"] = _elapsed(ev[0], ev[2])
    return (out if batched else out[0]), metadata
