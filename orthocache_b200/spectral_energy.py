"""Spectral scoring drop-ins (reference: src/orthocache/spectral_energy.py).

Every function here is one launch of the fused block scorer
(``oc_score_blocks``): the keys are read once, and the WHT band energies, ζ,
the query-aware bound and the two-gate mask come out of the same pass.  The
reference recomputes the FWHT of all keys once per function (four times per
``orthocache_forward`` call, ``pipeline.py:100-113``).

Shapes follow the reference: keys (S, H, D), queries (Sq, Hq, D); a leading
batch dimension (B, S, H, D) / (B, Sq, Hq, D) is also accepted and carried
through every output.  GQA extension: ``Hq`` may be a multiple of the keys'
``H``; query head ``hq`` then reads KV head ``hq // (Hq // H)``.
"""
from __future__ import annotations

import math

import torch

from . import _lib

BAND_DC = 0
BAND_LOW = (1, 64)      # spectral_energy.py:16
BAND_MID = (64, 256)    # spectral_energy.py:17
BAND_HIGH = (256, 512)  # spectral_energy.py:18
BLOCK = 512


def _check_block(block_size):
    if block_size != BLOCK:
        raise ValueError(f"the spectral scorer is a 512-point transform; block_size={block_size}")


def _as_batched(x, name):
    x = _lib.as_device(x)
    if x.dim() == 3:
        return x.unsqueeze(0), False
    if x.dim() == 4:
        return x, True
    raise ValueError(f"{name} must be (S, H, D) or (B, S, H, D), got {tuple(x.shape)}")


LONG_CHUNK_ROWS = 32  # query rows per KV head above which the bounds run as a GEMM


def score_blocks(keys, q=None, tau=-math.inf, zeta_max=math.inf, block_size=BLOCK,
                 band_low=BAND_LOW, band_mid=BAND_MID, band_high=BAND_HIGH,
                 want=("keep",), mode=0):
    """Run the fused scorer once and return the requested outputs as a dict.

    ``want`` names any of: dc, e_low, e_mid, e_high, zeta, bound_max, bounds,
    keep.  Shapes (batch dim dropped for 3-D inputs): dc (nb, H, D); e_*,
    zeta, bound_max (nb, H) float32; bounds (Sq, nb, Hq) float32; keep
    (nb, H) bool.  ``mode``: 0 automatic, 1 partial-transform scorer, 2 full
    9-stage butterfly scorer.
    """
    _check_block(block_size)
    k, batched = _as_batched(keys, "keys")
    B, S, H, D = k.shape
    if S % BLOCK:
        raise ValueError(f"seq_len {S} is not a multiple of 512")
    nb = S // BLOCK
    qq = None
    Sq = Hq = 0
    if q is not None:
        qq = _lib.as_device(q, device=k.device, dtype=k.dtype)
        if qq.dim() == 3:
            qq = qq.unsqueeze(0)
        if qq.dim() != 4 or qq.shape[0] != B or qq.shape[3] != D:
            raise ValueError(f"q shape {tuple(qq.shape)} does not match keys {tuple(k.shape)}")
        Sq, Hq = qq.shape[1], qq.shape[2]
    dev = k.device
    f32 = dict(dtype=torch.float32, device=dev)
    out = {}
    if "dc" in want:
        out["dc"] = torch.empty((B, nb, H, D), **f32)
    for name in ("e_low", "e_mid", "e_high", "zeta", "bound_max"):
        if name in want:
            out[name] = torch.empty((B, nb, H), **f32)
    if "bounds" in want:
        if qq is None:
            raise ValueError("bounds need q")
        out["bounds"] = torch.empty((B, Sq, nb, Hq), **f32)
    keep = torch.empty((B, nb, H), dtype=torch.uint8, device=dev) if "keep" in want else None
    if B * nb * H == 0:
        if keep is not None:
            out["keep"] = keep.bool()
        return out if batched else {n: t[0] for n, t in out.items()}
    if (qq is not None and Sq * (Hq // H) > LONG_CHUNK_ROWS and int(mode) == 0
            and (tuple(band_low), tuple(band_mid), tuple(band_high)) == (BAND_LOW, BAND_MID, BAND_HIGH)
            and set(want) <= {"dc", "zeta", "bound_max", "bounds", "keep"}):
        # Long query chunks: the query-independent block metadata in one pass
        # over the keys, then the bounds of all rows as a tiled GEMM.
        dc = out.get("dc", torch.empty((B, nb, H, D), **f32))
        zeta = out.get("zeta", torch.empty((B, nb, H), **f32))
        bmax = out.get("bound_max", torch.empty((B, nb, H), **f32))
        e_ac = torch.empty((B, nb, H), **f32)
        _lib.call("oc_block_metadata", _lib.ptr(k), _lib.dtype_code(k), B, S, H, D, _lib.ptr(dc), _lib.ptr(e_ac),
                  _lib.ptr(zeta), _lib.stream_ptr(dev))
        _lib.call("oc_score_from_metadata", _lib.ptr(dc), _lib.ptr(e_ac), _lib.ptr(zeta), _lib.ptr(qq),
                  _lib.dtype_code(qq), B, nb, H, D, Sq, Hq, float(tau), float(zeta_max), _lib.ptr(bmax),
                  _lib.ptr(out.get("bounds")), _lib.ptr(keep), _lib.stream_ptr(dev))
    else:
        _lib.call("oc_score_blocks", _lib.ptr(k), _lib.ptr(qq), _lib.dtype_code(k),
                  B, S, H, D, Sq, Hq,
                  int(band_low[0]), int(band_low[1]), int(band_mid[0]), int(band_mid[1]),
                  int(band_high[0]), int(band_high[1]),
                  float(tau), float(zeta_max),
                  _lib.ptr(out.get("dc")), _lib.ptr(out.get("e_low")), _lib.ptr(out.get("e_mid")),
                  _lib.ptr(out.get("e_high")), _lib.ptr(out.get("zeta")), _lib.ptr(out.get("bound_max")),
                  _lib.ptr(out.get("bounds")), _lib.ptr(keep), int(mode), _lib.stream_ptr(dev))
    if keep is not None:
        out["keep"] = keep.bool()
    if not batched:
        out = {n: t[0] for n, t in out.items()}
    return out


def compute_spectral_bands(keys, block_size: int = BLOCK, band_low: tuple = BAND_LOW,
                           band_mid: tuple = BAND_MID, band_high: tuple = BAND_HIGH):
    """(dc, low, mid, high) per block (``spectral_energy.py:69-106``).

    dc: (nb, H, D) WHT coefficient 0; low/mid/high: (nb, H) sum over the band's
    coefficients and over D of coef**2.
    """
    r = score_blocks(keys, None, block_size=block_size, band_low=band_low, band_mid=band_mid,
                     band_high=band_high, want=("dc", "e_low", "e_mid", "e_high"))
    return r["dc"], r["e_low"], r["e_mid"], r["e_high"]


def compute_spectral_decay_ratio(keys, block_size: int = BLOCK, band_low: tuple = BAND_LOW,
                                 band_high: tuple = BAND_HIGH):
    """ζ = E_high / (E_low + 1e-6) per (block, head) (``spectral_energy.py:109-138``)."""
    return score_blocks(keys, None, block_size=block_size, band_low=band_low,
                        band_mid=(band_low[1], band_high[0]), band_high=band_high,
                        want=("zeta",))["zeta"]


def compute_query_aware_bounds(q, keys, block_size: int = BLOCK):
    """Logit upper bound per (query, block, query head) (``spectral_energy.py:141-177``).

    Returns (Sq, nb, Hq): q·mean/√D + ‖q‖·√E_AC/√D with mean = DC/√512.
    """
    return score_blocks(keys, q, block_size=block_size, want=("bounds",))["bounds"]


def compute_query_aware_mask(q, keys, tau: float, block_size: int = BLOCK):
    """Single-gate mask: max over query rows of the bound >= tau (``spectral_energy.py:180-196``)."""
    return score_blocks(keys, q, tau=tau, zeta_max=math.inf, block_size=block_size,
                        want=("keep",))["keep"]


def compute_multiband_mask(q, keys, tau: float, zeta_max: float, block_size: int = BLOCK):
    """Two-gate keep mask: bound >= tau AND ζ <= zeta_max (``spectral_energy.py:199-234``)."""
    return score_blocks(keys, q, tau=tau, zeta_max=zeta_max, block_size=block_size,
                        want=("keep",))["keep"]


def compute_block_energy_jax(keys, block_size: int = BLOCK):
    """Sum of squared keys per (block, head) (``spectral_energy.py:21-35``)."""
    k, batched = _as_batched(keys, "keys")
    B, S, H, D = k.shape
    if S % block_size:
        raise ValueError(f"seq_len {S} is not a multiple of block_size {block_size}")
    out = torch.empty((B, S // block_size, H), dtype=torch.float32, device=k.device)
    _lib.call("oc_block_energy", _lib.ptr(k), _lib.dtype_code(k), B, S, H, D, block_size,
              _lib.ptr(out), _lib.stream_ptr(k.device))
    return out if batched else out[0]


def generate_threshold_mask(energies, epsilon: float):
    """``energies >= epsilon`` (``spectral_energy.py:237-239``)."""
    e = _lib.as_device(energies, dtype=torch.float32)
    keep = torch.empty(e.shape, dtype=torch.uint8, device=e.device)
    _lib.call("oc_apply_gates", _lib.ptr(e), None, e.numel(), None, float(epsilon), math.inf,
              _lib.ptr(keep), _lib.stream_ptr(e.device))
    return keep.bool()
