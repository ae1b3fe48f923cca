"""Seeded synthetic KV-cache workloads with the shapes and spectra of the
benchmark configurations (no dataset or model weights are available).

Key blocks are one of three kinds, chosen per 512-token block (shared by all
heads) from ``numpy.random.default_rng(seed)``:

* smooth: block mean N(0,1) per (head, channel) + sum of 3 cosines along the
  token axis with per-channel amplitudes N(0,1), periods U[256, 2048] tokens
  and random phase, + N(0, 0.05) noise;
* noise: block mean + iid N(0,1);
* mid: block mean + 0.5 * a random +-1 combination (per channel) of 4
  natural-order Walsh rows drawn from indices 64..191.

Values are N(0,1); queries N(0, 1/sqrt(D)) in standard deviation.  Tensors are
generated with a torch generator on the target device, block-chunk by
block-chunk, so a 64K-token cache is made on the GPU in milliseconds.

With natural-order bands, smooth blocks have ζ in the tens (their energy sits
at coefficients 128, 256, 384, ...) and noise blocks ζ ≈ 4, so with the
default ζ_max = 5 the ζ gate evicts the smooth blocks; ``calibrate_tau``
then sets τ so that the union keep count hits the target eviction exactly.
"""
from __future__ import annotations

import math

import numpy as np
import torch

KIND_SMOOTH, KIND_NOISE, KIND_MID = 0, 1, 2
BLOCK = 512


def block_kinds(nb, smooth_frac, mid_frac=0.0, seed=0):
    """Per-block kinds: round(smooth_frac*nb) smooth, round(mid_frac*nb) mid, rest noise."""
    rng = np.random.default_rng(seed)
    n_s = int(round(smooth_frac * nb))
    n_m = int(round(mid_frac * nb))
    kinds = np.full(nb, KIND_NOISE, np.int64)
    order = rng.permutation(nb)
    kinds[order[:n_s]] = KIND_SMOOTH
    kinds[order[n_s:n_s + n_m]] = KIND_MID
    return kinds


def _walsh_rows(rows, device):
    """Natural-order Walsh rows W_j[t] = (-1)^popcount(j & t), t < 512."""
    t = torch.arange(BLOCK, device=device)
    j = torch.as_tensor(rows, device=device).reshape(-1, 1)
    x = j & t
    par = torch.zeros_like(x)
    for bit in range(9):
        par ^= (x >> bit) & 1
    return (1 - 2 * par).float()


def make_keys(nb, H, D, kinds, seed=0, device="cuda", dtype=torch.bfloat16, chunk=16):
    """Keys (nb*512, H, D) following ``kinds`` (length nb)."""
    g = torch.Generator(device=device)
    g.manual_seed(int(seed) * 7919 + 17)
    out = torch.empty((nb * BLOCK, H, D), dtype=dtype, device=device)
    kinds_t = torch.as_tensor(np.asarray(kinds), device=device)
    t = torch.arange(BLOCK, device=device, dtype=torch.float32)
    two_pi = 2.0 * math.pi
    for b0 in range(0, nb, chunk):
        n = min(chunk, nb - b0)
        kd = kinds_t[b0:b0 + n]
        mean = torch.randn((n, 1, H, D), generator=g, device=device)
        noise = torch.randn((n, BLOCK, H, D), generator=g, device=device)
        amp = torch.randn((n, H, 3, D), generator=g, device=device)
        per = 256.0 + 1792.0 * torch.rand((n, H, 3), generator=g, device=device)
        ph = two_pi * torch.rand((n, H, 3), generator=g, device=device)
        cos = torch.cos(two_pi * t.view(1, 1, 1, BLOCK) / per[..., None] + ph[..., None])  # (n,H,3,512)
        smooth = torch.einsum("nhct,nhcd->nthd", cos, amp) + 0.05 * noise
        rows = torch.randint(64, 192, (n, 4), generator=g, device=device)
        sign = torch.randint(0, 2, (n, 4, H, D), generator=g, device=device).float() * 2 - 1
        w = _walsh_rows(rows.reshape(-1), device).reshape(n, 4, BLOCK)
        mid = 0.5 * torch.einsum("nrt,nrhd->nthd", w, sign)
        sel = kd.view(n, 1, 1, 1)
        blk = torch.where(sel == KIND_SMOOTH, smooth, torch.where(sel == KIND_MID, mid, noise)) + mean
        out[b0 * BLOCK:(b0 + n) * BLOCK] = blk.reshape(n * BLOCK, H, D).to(dtype)
    return out


def make_values(S, H, D, seed=0, device="cuda", dtype=torch.bfloat16):
    g = torch.Generator(device=device)
    g.manual_seed(int(seed) * 7919 + 29)
    return torch.randn((S, H, D), generator=g, device=device).to(dtype)


def make_queries(Sq, Hq, D, seed=0, device="cuda", dtype=torch.bfloat16):
    g = torch.Generator(device=device)
    g.manual_seed(int(seed) * 7919 + 41)
    return (torch.randn((Sq, Hq, D), generator=g, device=device) * D ** -0.5).to(dtype)


def calibrate_tau(zeta, bound_max, zeta_max, evict):
    """τ that makes the union keep mask retain round((1 - evict) * nb) blocks.

    zeta, bound_max: (nb, H) scores.  A block survives both gates iff some head
    h has ζ[b,h] <= zeta_max and bound[b,h] >= τ, i.e. iff τ <= s_b with
    s_b = max over the ζ-passing heads of the bound.  τ is placed halfway
    between the k-th and (k+1)-th largest s_b (k = blocks to keep), or 1 %
    below the k-th when fewer than k+1 blocks pass the ζ gate; so no block
    sits near the threshold.  Returns (tau, kept_count).
    """
    z = torch.as_tensor(zeta).double().cpu()
    bm = torch.as_tensor(bound_max).double().cpu()
    nb = z.shape[0]
    k = int(round((1.0 - evict) * nb))
    s = torch.where(z <= zeta_max, bm, torch.full_like(bm, -math.inf)).max(dim=1).values
    srt = torch.sort(s, descending=True).values
    if k <= 0:
        top = float(srt[0])
        return (top + max(1.0, abs(top)) if math.isfinite(top) else 0.0), 0
    kth = float(srt[k - 1])
    if not math.isfinite(kth):
        finite = srt[torch.isfinite(srt)]
        kth = float(finite[-1]) if len(finite) else 0.0
        return kth - max(0.01 * abs(kth), 1e-2), int(len(finite))
    nxt = float(srt[k]) if k < nb else -math.inf
    if math.isfinite(nxt):
        return 0.5 * (kth + nxt), k
    return kth - max(0.01 * abs(kth), 1e-2), k
