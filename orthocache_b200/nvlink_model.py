"""Interconnect byte model of a sharded decode step, for NVLink / NVSwitch.

Two parts:

* the reference's analytical model (``ici_bandwidth_model.py:39-99`` and
  ``:107-160``), restated with the same names, arguments and results:
  per decode step and device, the dense all-gather shard
  ``L * S * d_k * H_kv / P**2 * dtype_bytes`` and its sparse counterpart
  ``dense * (1 - sparsity)``;
* what the three exchanges built here actually move per GPU and decode step
  (``exchange_bytes``), and the time that takes at a per-direction link
  bandwidth (``exchange_time_us``; default the peer-copy rate measured on
  this pool's NVSwitch boxes, 770 GB/s per direction per GPU):

  - ``"partials"``: the one-kernel LSE merge (``oc_decode_step_sharded``).
    Every rank stores its (m, l, o) rows of every group into every other
    rank's region, one 8-byte word per value (float + call number):
    ``L * (P - 1) * B * Sq * Hq * (D + 2) * 8`` bytes sent per GPU, independent
    of the context length;
  - ``"stratified"``: the reference's stratified all-gather of the retained
    blocks (``phase_e_stratified.py``): each rank receives every other rank's
    ``bucket`` padded blocks of K and V, ``L * (P - 1) * bucket * 512 * H_kv *
    d_k * 2 * dtype_bytes``;
  - ``"alltoallv_heads"``: the AllToAllv by KV head: each rank receives its
    ``H_kv / P`` heads of every other rank's retained blocks,
    ``L * (P - 1) * kept * 512 * (H_kv / P) * d_k * 2 * dtype_bytes``.
"""
from __future__ import annotations

BLOCK = 512
_BYTES_PER_GB = 1e9
_BYTES_PER_MB = 1e6
_DEFAULT_SPARSITY_LEVELS = [0.0, 0.1, 0.3, 0.5, 0.688, 0.75, 0.9]
MEASURED_PEER_GBS = 770.0  # peer copy, GB/s per direction per GPU (NVLink 5 through NVSwitch)


def ici_bytes_per_step(num_layers: int, seq_len: int, head_dim: int, num_kv_heads: int, num_devices: int,
                       sparsity: float, dtype_bytes: int = 2) -> dict:
    """Per-device interconnect bytes of one decode step without and with
    eviction (``ici_bandwidth_model.py:39-99``): dense = L S d_k H_kv / P^2
    dtype_bytes, truncated to an integer; sparse = int(dense (1 - sparsity))."""
    if not 0.0 <= sparsity <= 1.0:
        raise ValueError(f"sparsity must be in [0, 1], got {sparsity}")
    dense = int(num_layers * seq_len * head_dim * num_kv_heads * dtype_bytes / (num_devices * num_devices))
    sparse = int(dense * (1.0 - sparsity))
    saved = dense - sparse
    return {
        "dense_bytes": dense,
        "sparse_bytes": sparse,
        "savings_bytes": saved,
        "savings_pct": round(saved / dense * 100.0, 2) if dense > 0 else 0.0,
        "savings_gb_per_1000_steps": round(saved * 1000 / _BYTES_PER_GB, 3),
    }


def ici_bandwidth_table(num_layers: int, seq_len: int, head_dim: int, num_kv_heads: int, num_devices: int,
                        dtype_bytes: int = 2, sparsity_levels=None) -> list:
    """``ici_bytes_per_step`` over sparsity levels, in decimal MB
    (``ici_bandwidth_model.py:107-160``)."""
    levels = list(_DEFAULT_SPARSITY_LEVELS) if sparsity_levels is None else list(sparsity_levels)
    rows = []
    for s in levels:
        r = ici_bytes_per_step(num_layers, seq_len, head_dim, num_kv_heads, num_devices, s, dtype_bytes)
        rows.append({"sparsity": s,
                     "dense_mb": round(r["dense_bytes"] / _BYTES_PER_MB, 2),
                     "sparse_mb": round(r["sparse_bytes"] / _BYTES_PER_MB, 2),
                     "savings_mb": round(r["savings_bytes"] / _BYTES_PER_MB, 2),
                     "savings_pct": r["savings_pct"]})
    return rows


def exchange_bytes(variant: str, num_layers: int, num_devices: int, head_dim: int, num_kv_heads: int,
                   num_q_heads: int = None, batch: int = 1, q_len: int = 1, kept_blocks: int = 0,
                   bucket_blocks: int = None, dtype_bytes: int = 2) -> int:
    """Bytes one GPU sends (= receives, the exchanges are symmetric) per
    decode step over all layers, for ``variant`` in ("partials",
    "stratified", "alltoallv_heads").  kept_blocks: retained blocks per shard
    and batch row; bucket_blocks: the stratified bucket (default kept_blocks)."""
    P, L = num_devices, num_layers
    if P < 1 or L < 0:
        raise ValueError("num_devices >= 1 and num_layers >= 0")
    if variant == "partials":
        hq = num_kv_heads if num_q_heads is None else num_q_heads
        return L * (P - 1) * batch * q_len * hq * (head_dim + 2) * 8
    blk = BLOCK * head_dim * 2 * dtype_bytes  # K and V of one block and KV head
    if variant == "stratified":
        bucket = kept_blocks if bucket_blocks is None else bucket_blocks
        return L * (P - 1) * batch * bucket * num_kv_heads * blk
    if variant == "alltoallv_heads":
        if num_kv_heads % P:
            raise ValueError(f"{num_kv_heads} KV heads do not split over {P} devices")
        return L * (P - 1) * batch * kept_blocks * (num_kv_heads // P) * blk
    raise ValueError(f"unknown exchange variant {variant!r}")


def exchange_time_us(nbytes: int, link_gbs: float = MEASURED_PEER_GBS) -> float:
    """Transfer time of nbytes at link_gbs GB/s per direction (no latency term)."""
    return nbytes / (link_gbs * 1e3)
