"""CPU oracle for the OrthoCache eviction + attention hot path.

TEST INFRASTRUCTURE ONLY.  This module is the checker: the parity tests,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of ``bench.py`` may
import it.  The product (``orthocache_b200``) never imports, links or calls
anything under ``oracle/``.

It restates, in vectorised NumPy, the algorithm of the reference package
``orthocache`` (v0.3.0, ``src/orthocache``) for the functions on the hot path.
Each function cites the reference lines it follows.  Arithmetic conventions:

* The FWHT runs in float32 with the reference's stage order (h = 1, 2, ..., 256;
  ``a + b`` then ``a - b``) and its final float32 division by
  ``22.627416997969522`` (``fwht.py:25-61``).  Every coefficient is therefore
  the IEEE-float32 value the reference's own butterfly produces.
* Reductions (band energies, dot products, softmax sums) are accumulated in
  float64 and rounded once to float32.  The reference accumulates in float32
  in an XLA-chosen order; both are within a few ulp of the exact sum, and the
  parity tolerances account for that.
* GQA extension (the reference is MHA only): query head ``hq`` reads KV head
  ``hq // G`` with ``G = Hq // Hkv``; for the logit-bound gate the ``G`` query
  heads of a group are extra query rows, so the max of
  ``spectral_energy.py:195`` runs over ``Sq * G`` rows.  With ``G == 1`` every
  function reduces to the reference exactly.

Pinning: ``tests/test_oracle_pins.py`` checks this module against the golden
vectors in ``tests/golden/`` (made by ``tests/golden/make_golden.py`` from the
reference's own float64 ``reference.py``) and against the known answers of the
reference's tests.
"""
from __future__ import annotations

import math

import numpy as np

BLOCK = 512
FWHT_NORM = np.float32(22.627416997969522)  # fwht.py:61
BAND_LOW = (1, 64)      # spectral_energy.py:16
BAND_MID = (64, 256)    # spectral_energy.py:17
BAND_HIGH = (256, 512)  # spectral_energy.py:18
ZETA_EPS = np.float32(1e-6)  # spectral_energy.py:138


# --------------------------------------------------------------------------
# a1  fwht_512  (fwht.py:4-65)
# --------------------------------------------------------------------------
def fwht_512(x: np.ndarray) -> np.ndarray:
    """512-row FWHT along axis 0, natural (Hadamard) order, float32.

    Follows ``fwht.py:16-64``: stage s pairs rows that differ in bit s
    (h = 2**s), writes ``a + b`` to the lower and ``a - b`` to the upper row,
    for s = 0..8 in that order, then divides by ``22.627416997969522``.
    """
    x = np.asarray(x, dtype=np.float32)
    one_d = x.ndim == 1
    if one_d:
        x = x[:, None]
    if x.shape[0] != BLOCK:
        raise ValueError(f"fwht_512 needs 512 rows, got {x.shape[0]}")
    d = x.shape[1]
    y = x.copy()
    h = 1
    while h < BLOCK:
        y = y.reshape(BLOCK // (2 * h), 2, h, d)
        a = y[:, 0]
        b = y[:, 1]
        y = np.stack([a + b, a - b], axis=1).reshape(BLOCK, d)
        h *= 2
    y = y / FWHT_NORM
    return y[:, 0] if one_d else y


# --------------------------------------------------------------------------
# a2 / a3 / a4  spectral bands and zeta  (spectral_energy.py:38-138)
# --------------------------------------------------------------------------
def spectral_coefficients(keys: np.ndarray, block_size: int = BLOCK) -> np.ndarray:
    """WHT coefficients per block: (nb, 512, H, D) float32.

    ``_run_fwht_on_blocks`` (``spectral_energy.py:38-66``): reshape the keys to
    (nb, 512, H, D) and run ``fwht_512`` along the token axis of each block.
    """
    if block_size != BLOCK:
        raise ValueError("the spectral scorer is defined for block_size=512 only")
    keys = np.asarray(keys, dtype=np.float32)
    s, h, d = keys.shape
    if s % BLOCK:
        raise ValueError("seq_len must be a multiple of 512")
    nb = s // BLOCK
    blocks = keys.reshape(nb, BLOCK, h, d).transpose(1, 0, 2, 3).reshape(BLOCK, -1)
    spec = fwht_512(blocks).reshape(BLOCK, nb, h, d).transpose(1, 0, 2, 3)
    return np.ascontiguousarray(spec)


def _band_energy(spec: np.ndarray, band) -> np.ndarray:
    lo, hi = band
    part = spec[:, lo:hi].astype(np.float64)
    return np.einsum("bkhd,bkhd->bh", part, part).astype(np.float32)


def spectral_bands(keys, block_size=BLOCK, band_low=BAND_LOW, band_mid=BAND_MID,
                   band_high=BAND_HIGH):
    """(dc, low, mid, high) as ``compute_spectral_bands`` (``spectral_energy.py:69-106``).

    dc: (nb, H, D) = coefficient 0; each band energy: (nb, H) = sum over the
    band's coefficient indices and over D of coef**2 (``:102-104``).
    """
    spec = spectral_coefficients(keys, block_size)
    dc = spec[:, 0].copy()
    return (dc, _band_energy(spec, band_low), _band_energy(spec, band_mid),
            _band_energy(spec, band_high))


def zeta_from_energies(low: np.ndarray, high: np.ndarray) -> np.ndarray:
    """``high / (low + 1e-6)`` in float32 (``spectral_energy.py:138``)."""
    return (np.asarray(high, np.float32) / (np.asarray(low, np.float32) + ZETA_EPS)).astype(np.float32)


def spectral_decay_ratio(keys, block_size=BLOCK, band_low=BAND_LOW, band_high=BAND_HIGH):
    """ζ per (block, head) (``spectral_energy.py:109-138``); mid band = [low_hi, high_lo)."""
    _, low, _, high = spectral_bands(keys, block_size, band_low,
                                     (band_low[1], band_high[0]), band_high)
    return zeta_from_energies(low, high)


# --------------------------------------------------------------------------
# a5 / a6 / a7  query-aware bound and the two-gate mask
# (spectral_energy.py:141-234)
# --------------------------------------------------------------------------
def _group(hq: int, hkv: int) -> int:
    if hq % hkv:
        raise ValueError(f"query heads ({hq}) must be a multiple of kv heads ({hkv})")
    return hq // hkv


def query_aware_bounds(q, keys, block_size=BLOCK):
    """Per-query-head logit upper bound, shape (Sq, nb, Hq).

    ``compute_query_aware_bounds`` (``spectral_energy.py:141-177``):
    mean = DC / sqrt(512); alignment = q . mean / sqrt(d);
    residual = ||q|| * sqrt(E_AC) / sqrt(d) with E_AC = sum of coef**2 over
    indices 1..511; bound = alignment + residual.  Query head ``hq`` uses KV
    head ``hq // G`` (GQA extension; identity for MHA).
    """
    q = np.asarray(q, np.float32)
    spec = spectral_coefficients(keys, block_size)
    nb, _, hkv, d = spec.shape
    sq, hq, _ = q.shape
    g = _group(hq, hkv)
    dc = spec[:, 0].astype(np.float64)                      # (nb, Hkv, D)
    ac = spec[:, 1:].astype(np.float64)
    e_ac = np.einsum("bkhd,bkhd->bh", ac, ac)               # (nb, Hkv)
    mean = dc / math.sqrt(BLOCK)
    q64 = q.astype(np.float64).reshape(sq, hkv, g, d)
    align = np.einsum("qhgd,bhd->qbhg", q64, mean) / math.sqrt(d)
    qn = np.sqrt(np.einsum("qhgd,qhgd->qhg", q64, q64))      # (Sq, Hkv, G)
    resid = qn[:, None, :, :] * np.sqrt(e_ac)[None, :, :, None] / math.sqrt(d)
    return (align + resid).reshape(sq, nb, hq).astype(np.float32)


def block_metadata(keys, block_size=BLOCK):
    """Query-independent metadata of every block, computed once when a block
    is written (the hoisting of ``docs/mathematical_framework.md:244-250``):
    dc (nb, H, D) = WHT coefficient 0, e_ac (nb, H) = energy of coefficients
    1..511 (``spectral_energy.py:159-160``), zeta (nb, H)
    (``spectral_energy.py:109-138``).  float32."""
    spec = spectral_coefficients(keys, block_size)
    dc = spec[:, 0].astype(np.float64)
    ac = spec[:, 1:].astype(np.float64)
    e_ac = np.einsum("bkhd,bkhd->bh", ac, ac)
    return dc.astype(np.float32), e_ac.astype(np.float32), spectral_decay_ratio(keys, block_size)


def bounds_from_metadata(q, dc, e_ac):
    """``compute_query_aware_bounds`` (``spectral_energy.py:141-177``) from the
    cached dc and E_AC instead of the keys: (Sq, nb, Hq)."""
    q64 = np.asarray(q, np.float64)
    dc = np.asarray(dc, np.float64)
    e_ac = np.asarray(e_ac, np.float64)
    nb, hkv, d = dc.shape
    sq, hq, _ = q64.shape
    g = _group(hq, hkv)
    q64 = q64.reshape(sq, hkv, g, d)
    align = np.einsum("qhgd,bhd->qbhg", q64, dc / math.sqrt(BLOCK)) / math.sqrt(d)
    qn = np.sqrt(np.einsum("qhgd,qhgd->qhg", q64, q64))
    resid = qn[:, None, :, :] * np.sqrt(e_ac)[None, :, :, None] / math.sqrt(d)
    return (align + resid).reshape(sq, nb, hq).astype(np.float32)


def max_bounds(q, keys, block_size=BLOCK):
    """Max over the query axis (and the G heads of each group): (nb, Hkv).

    ``compute_query_aware_mask`` (``spectral_energy.py:194-195``).
    """
    b = query_aware_bounds(q, keys, block_size)
    sq, nb, hq = b.shape
    hkv = np.asarray(keys).shape[1]
    g = hq // hkv
    return b.reshape(sq, nb, hkv, g).max(axis=(0, 3))


def query_aware_mask(q, keys, tau, block_size=BLOCK):
    """``max_bounds >= tau`` (``spectral_energy.py:180-196``)."""
    return max_bounds(q, keys, block_size) >= np.float32(tau)


def multiband_mask(q, keys, tau, zeta_max, block_size=BLOCK):
    """Two-gate keep mask (``spectral_energy.py:199-234``): bound >= tau AND ζ <= zeta_max."""
    return query_aware_mask(q, keys, tau, block_size) & (
        spectral_decay_ratio(keys, block_size) <= np.float32(zeta_max))


def score_blocks(q, keys, tau, zeta_max, block_size=BLOCK, band_low=BAND_LOW,
                 band_mid=BAND_MID, band_high=BAND_HIGH):
    """Everything the fused scorer emits, from one FWHT of the keys.

    Returns a dict with dc (nb,H,D), e_low/e_mid/e_high/zeta/bound_max (nb,H)
    and keep (nb,H) bool.  ζ uses the low and high bands as
    ``compute_spectral_decay_ratio`` does; E_AC is the sum over indices
    1..511 as in ``compute_query_aware_bounds`` (``spectral_energy.py:159-160``).
    """
    dc, lo, mi, hi = spectral_bands(keys, block_size, band_low, band_mid, band_high)
    zeta = zeta_from_energies(lo, hi)
    bmax = max_bounds(q, keys, block_size)
    keep = (bmax >= np.float32(tau)) & (zeta <= np.float32(zeta_max))
    return dict(dc=dc, e_low=lo, e_mid=mi, e_high=hi, zeta=zeta, bound_max=bmax, keep=keep)


def near_threshold(zeta, bound_max, tau, zeta_max, rel=1e-5):
    """Blocks whose ζ or bound lies within ``rel`` (relative) of its threshold.

    The parity contract exempts exactly these (block, head) cells from the
    bit-exact mask comparison; callers report them.
    """
    zeta = np.asarray(zeta, np.float64)
    bm = np.asarray(bound_max, np.float64)
    zt = abs(float(zeta_max))
    tt = abs(float(tau))
    zn = np.abs(zeta - zeta_max) <= rel * np.maximum(np.maximum(np.abs(zeta), zt), 1e-30)
    tn = np.abs(bm - tau) <= rel * np.maximum(np.maximum(np.abs(bm), tt), 1e-30)
    return zn | tn


def block_energy(keys, block_size=BLOCK):
    """``compute_block_energy_jax`` (``spectral_energy.py:21-35``): sum of squares per (block, head)."""
    k = np.asarray(keys, np.float64)
    s, h, d = k.shape
    nb = s // block_size
    return np.einsum("bthd,bthd->bh", k.reshape(nb, block_size, h, d),
                     k.reshape(nb, block_size, h, d)).astype(np.float32)


# --------------------------------------------------------------------------
# a9 / a10  stream compaction (compaction.py:28-154; alltoallv.py:44-75)
# --------------------------------------------------------------------------
def stream_compact_mask(block_mask: np.ndarray):
    """(perm int32 (nb,), num_active int).

    Union over heads for a 2-D mask (``compaction.py:65``); a stable
    permutation with active blocks first in ascending order, then inactive
    blocks in ascending order (``compaction.py:76-82``,
    ``adaptive_attention.py:37-40``).
    """
    m = np.asarray(block_mask).astype(bool)
    if m.ndim == 2:
        m = m.any(axis=-1)
    idx = np.arange(m.shape[0], dtype=np.int32)
    perm = np.concatenate([idx[m], idx[~m]]).astype(np.int32)
    return perm, int(m.sum())


def stream_compact(keys, values, block_mask, block_size=BLOCK):
    """(compact_k, compact_v, perm, num_active) (``compaction.py:28-100``).

    Gathers blocks by ``perm``; positions >= num_active are zero (``:94-98``).
    """
    perm, n = stream_compact_mask(block_mask)
    s, h, d = keys.shape
    nb = s // block_size
    kb = np.asarray(keys).reshape(nb, block_size, h, d)[perm].copy()
    vb = np.asarray(values).reshape(nb, block_size, h, d)[perm].copy()
    kb[n:] = 0
    vb[n:] = 0
    return kb, vb, perm, n


def stream_decompact(compact, perm, num_active, num_blocks):
    """Scatter back, zero inactive (``compaction.py:103-154``)."""
    out = np.zeros((num_blocks,) + compact.shape[1:], compact.dtype)
    out[perm[:num_active]] = compact[:num_active]
    return out


# --------------------------------------------------------------------------
# a11 / a12  attention (indirect_attention.py:127-170,
# adaptive_attention.py:90-120, sparse_attention.py:5-64)
# --------------------------------------------------------------------------
def indirect_attention(q, keys, values, perm, num_active, block_size=BLOCK):
    """Attention of every query head over the blocks perm[:num_active].

    Numerics of ``_multihead_loop`` (``adaptive_attention.py:90-120``): fp32
    inputs, logits = q.k / sqrt(d), softmax over all retained tokens, o / l.
    The oracle evaluates the exact softmax in float64 (the online form is
    algebraically identical).  num_active == 0 gives zeros
    (``indirect_attention.py:150-151``).  Returns float32 (Sq, Hq, D).
    """
    q = np.asarray(q, np.float64)
    sq, hq, d = q.shape
    k = np.asarray(keys, np.float64)
    v = np.asarray(values, np.float64)
    s, hkv, _ = k.shape
    g = _group(hq, hkv)
    if num_active == 0:
        return np.zeros((sq, hq, d), np.float32)
    blocks = np.asarray(perm[:num_active], np.int64)
    tok = (blocks[:, None] * block_size + np.arange(block_size)[None, :]).reshape(-1)
    ks = k[tok].reshape(-1, hkv, 1, d)
    vs = v[tok].reshape(-1, hkv, 1, d)
    qg = q.reshape(sq, hkv, g, d)
    logits = np.einsum("qhgd,khxd->qkhg", qg, ks) / math.sqrt(d)
    logits -= logits.max(axis=1, keepdims=True)
    w = np.exp(logits)
    w /= w.sum(axis=1, keepdims=True)
    out = np.einsum("qkhg,khxd->qhgd", w, vs)
    return out.reshape(sq, hq, d).astype(np.float32)


def partial_attention(q, keys, values, perm, num_active, block_size=BLOCK):
    """Unnormalised attention state of one shard over blocks perm[:num_active]:
    (m, l, o) per query row in float64 with m the max logit (natural units),
    l = sum exp(s - m), o = sum exp(s - m) v — the running state of the
    online softmax of ``_multihead_loop`` (``adaptive_attention.py:90-120``)
    and of ``distributed_attention.py:95-128`` after the shard's last block.
    No retained block: m = -inf, l = 0, o = 0.  Shapes (Sq, Hq), (Sq, Hq),
    (Sq, Hq, D)."""
    q = np.asarray(q, np.float64)
    sq, hq, d = q.shape
    k = np.asarray(keys, np.float64)
    v = np.asarray(values, np.float64)
    s, hkv, _ = k.shape
    g = _group(hq, hkv)
    if num_active == 0:
        return np.full((sq, hq), -np.inf), np.zeros((sq, hq)), np.zeros((sq, hq, d))
    blocks = np.asarray(perm[:num_active], np.int64)
    tok = (blocks[:, None] * block_size + np.arange(block_size)[None, :]).reshape(-1)
    ks = k[tok].reshape(-1, hkv, 1, d)
    vs = v[tok].reshape(-1, hkv, 1, d)
    qg = q.reshape(sq, hkv, g, d)
    logits = np.einsum("qhgd,khxd->qkhg", qg, ks) / math.sqrt(d)
    m = logits.max(axis=1)
    w = np.exp(logits - m[:, None])
    l = w.sum(axis=1)
    o = np.einsum("qkhg,khxd->qhgd", w, vs)
    return m.reshape(sq, hq), l.reshape(sq, hq), o.reshape(sq, hq, d)


def merge_partials(parts):
    """Log-sum-exp merge of shard states [(m, l, o), ...] into o / l (zeros
    where no shard retained anything); float32 (Sq, Hq, D)."""
    m = np.max(np.stack([p[0] for p in parts]), axis=0)
    safe = np.where(np.isfinite(m), m, 0.0)
    l = sum(p[1] * np.where(np.isfinite(p[0]), np.exp(p[0] - safe), 0.0) for p in parts)
    o = sum(p[2] * np.where(np.isfinite(p[0]), np.exp(p[0] - safe), 0.0)[..., None] for p in parts)
    out = np.where(l[..., None] > 0, o / np.where(l > 0, l, 1.0)[..., None], 0.0)
    return out.astype(np.float32)


def block_sparse_attention(q, keys, values, block_mask, block_size=BLOCK):
    """Predicated attention with a per-(block, head) mask (``sparse_attention.py:5-64``).

    Evicted logits are replaced by -1e9 before a softmax over all tokens
    (``:49-57``).  ``block_mask`` is (nb, Hkv); query head hq uses kv head hq // G.
    """
    q = np.asarray(q, np.float64)
    sq, hq, d = q.shape
    k = np.asarray(keys, np.float64)
    v = np.asarray(values, np.float64)
    s, hkv, _ = k.shape
    g = _group(hq, hkv)
    m = np.asarray(block_mask, bool)
    qg = q.reshape(sq, hkv, g, d)
    logits = np.einsum("qhgd,khd->qkhg", qg, k) / math.sqrt(d)
    tok_mask = np.repeat(m, block_size, axis=0)              # (S, Hkv)
    logits = np.where(tok_mask[None, :, :, None], logits, -1e9)
    logits -= logits.max(axis=1, keepdims=True)
    w = np.exp(logits)
    w /= w.sum(axis=1, keepdims=True)
    out = np.einsum("qkhg,khd->qhgd", w, v)
    return out.reshape(sq, hq, d).astype(np.float32)


def dense_attention(q, keys, values):
    """Plain softmax attention (``pipeline.py:160-165``), float64 -> float32."""
    s = np.asarray(keys).shape[0]
    hkv = np.asarray(keys).shape[1]
    return block_sparse_attention(q, keys, values, np.ones((s // BLOCK if s % BLOCK == 0 else 1, hkv), bool),
                                  BLOCK if s % BLOCK == 0 else s)


def next_bucket(n: int) -> int:
    """``_next_bucket`` (``indirect_attention.py:20-26``)."""
    for b in (1, 2, 4, 8, 16, 32, 64, 128, 256, 512):
        if b >= n:
            return b
    return n


def auto_tau(q, keys, block_size=BLOCK) -> float:
    """mean - std of the per-(block, head) max bound (``pipeline.py:168-176``)."""
    mb = max_bounds(q, keys, block_size).astype(np.float64)
    return float(mb.mean() - mb.std())


# --------------------------------------------------------------------------
# a14 - a18  sequence-parallel exchange (alltoallv.py, distributed_attention.py,
# benchmarks/phase_e_stratified.py)
# --------------------------------------------------------------------------
def pack_active_blocks(kv_shard, perm, num_active, max_blocks, block_size=BLOCK):
    """Active blocks to the front of a zeroed buffer (``alltoallv.py:150-212``)."""
    kv = np.asarray(kv_shard)
    s, h, d = kv.shape
    out = np.zeros((max_blocks * block_size, h, d), kv.dtype)
    kb = kv.reshape(-1, block_size, h, d)
    for i in range(num_active):
        out[i * block_size:(i + 1) * block_size] = kb[perm[i]]
    return out


def compute_offsets(all_counts):
    """Exclusive prefix sum and total (``alltoallv.py:113-145``)."""
    c = np.asarray(all_counts, np.int64)
    pre = np.cumsum(c)
    off = np.concatenate([[0], pre[:-1]]).astype(np.int32)
    return off, int(pre[-1]) if len(pre) else 0


def global_block_index(all_counts, slots_per_device):
    """Indirection over the gathered buffer (``distributed_attention.py:182-191``).

    Slot j of the gathered buffer belongs to device j // slots and is valid iff
    j % slots < counts[device]; valid slots first, ascending, then the rest.
    """
    c = np.asarray(all_counts, np.int64)
    p = len(c)
    j = np.arange(p * slots_per_device)
    dev = j // slots_per_device
    valid = (j % slots_per_device) < c[dev]
    order = np.concatenate([j[valid], j[~valid]]).astype(np.int32)
    return order, int(valid.sum())


def stratified_buckets(nb_per_dev: int):
    """The four capacity buckets of ``build_stratified`` (``phase_e_stratified.py:182-197``)."""
    cand = [max(1, nb_per_dev // 4), max(1, nb_per_dev // 2),
            max(1, (nb_per_dev * 3) // 4), nb_per_dev]
    out = []
    for b in cand:
        if b not in out:
            out.append(b)
    while len(out) < 4:
        out.append(out[-1])
    return tuple(out)


def stratified_bucket(gmax: int, buckets) -> int:
    """Bucket choice from the global max count (``phase_e_stratified.py:262-265``)."""
    b1, b2, b3, b4 = buckets
    if gmax <= b1:
        return b1
    if gmax <= b2:
        return b2
    if gmax <= b3:
        return b3
    return b4


def unpack_received(kv_received, all_counts, num_devices, max_blocks, block_size=BLOCK):
    """Valid tokens of each device's chunk to the front (``alltoallv.py:264-335``)."""
    kv = np.asarray(kv_received)
    shard = max_blocks * block_size
    t = np.arange(num_devices * shard)
    sid = t // shard
    valid = (t - sid * shard) < (np.asarray(all_counts)[sid] * block_size)
    order = np.concatenate([t[valid], t[~valid]])
    out = kv[order].copy()
    out[int(valid.sum()):] = 0
    off, _ = compute_offsets(all_counts)
    return out, (off * block_size).astype(np.int32)
