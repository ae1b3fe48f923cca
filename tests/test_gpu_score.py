"""Parity of the FWHT and the fused block scorer (CUDA, through the C ABI)
against the CPU oracle and the reference's golden vectors."""
import math
import os
import sys

import numpy as np
import pytest
import torch

from oracle import oc_oracle as O
from gpu_util import dev, host, bf16_round, assert_mask_parity

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_golden import inputs  # noqa: E402

GOLD = np.load(os.path.join(HERE, "golden", "reference_golden.npz"))
X = inputs()


def oc():
    import orthocache_b200 as m
    return m


def test_fwht_bit_exact_vs_oracle():
    x = X["fwht2d_x"]
    y = host(oc().fwht_512(dev(x)))
    assert np.array_equal(y, O.fwht_512(x)), "FWHT must be bit-identical to the float32 butterfly"
    np.testing.assert_allclose(y, GOLD["fwht2d"], rtol=1e-5, atol=1e-5)


def test_fwht_1d_and_ragged_columns():
    y = host(oc().fwht_512(dev(X["fwht1d_x"])))
    assert np.array_equal(y, O.fwht_512(X["fwht1d_x"]))
    rs = np.random.RandomState(1)
    for n in (1, 31, 33, 1000):
        x = rs.randn(512, n).astype(np.float32)
        assert np.array_equal(host(oc().fwht_512(dev(x))), O.fwht_512(x))


def test_fwht_bf16_input():
    x = bf16_round(np.random.RandomState(2).randn(512, 96))
    y = host(oc().fwht_512(dev(x, torch.bfloat16)))
    assert np.array_equal(y, O.fwht_512(x))


def test_fwht_rejects_bad_shape():
    with pytest.raises(ValueError):
        oc().fwht_512(torch.zeros(256, 4, device="cuda"))


@pytest.mark.parametrize("mode", [1, 2])
def test_golden_bands(mode):
    from orthocache_b200 import score_blocks
    r = score_blocks(dev(X["bands_keys"]), want=("dc", "e_low", "e_mid", "e_high"), mode=mode)
    for name, key in (("dc", "bands_dc"), ("e_low", "bands_low"), ("e_mid", "bands_mid"), ("e_high", "bands_high")):
        np.testing.assert_allclose(host(r[name]), GOLD[key], rtol=1e-4, atol=1e-4)
    z = host(oc().compute_spectral_decay_ratio(dev(X["zeta_keys"])))
    np.testing.assert_allclose(z, GOLD["zeta"], rtol=1e-4, atol=1e-4)


def test_golden_bounds_and_energy():
    b = host(oc().compute_query_aware_bounds(dev(X["bounds_q"]), dev(X["bounds_keys"])))
    np.testing.assert_allclose(b, GOLD["bounds"], rtol=1e-5, atol=1e-5)
    e = host(oc().compute_block_energy_jax(dev(X["energy_keys"])))
    np.testing.assert_allclose(e, GOLD["energy"], rtol=1e-5, atol=1e-5)


def test_golden_masks():
    m = host(oc().compute_multiband_mask(dev(X["twogate_q"]), dev(X["twogate_keys"]), -100.0, 1.0))
    np.testing.assert_array_equal(m, GOLD["twogate_mask"])
    tau, zmax = float(GOLD["mask_tau"]), float(GOLD["mask_zeta_max"])
    m = host(oc().compute_multiband_mask(dev(X["mask_q"]), dev(X["mask_keys"]), tau, zmax))
    np.testing.assert_array_equal(m, GOLD["mask"])
    m1 = host(oc().compute_query_aware_mask(dev(X["mask_q"]), dev(X["mask_keys"]), tau))
    np.testing.assert_array_equal(m1, GOLD["mask_maxbound"] >= tau)


def test_threshold_mask_literal():
    m = host(oc().generate_threshold_mask(torch.tensor([[10.5, 2.3], [1.1, 15.6]]), 5.0))
    np.testing.assert_array_equal(m, [[True, False], [False, True]])


CASES = [  # (nb, Hkv, Hq, Sq, D, dtype, smooth_frac, mid_frac)
    (16, 8, 8, 1, 128, torch.bfloat16, 0.5, 0.0),    # config 0
    (8, 8, 32, 1, 128, torch.bfloat16, 0.75, 0.0),   # config 1 head layout (GQA 4)
    (6, 4, 8, 3, 64, torch.float32, 0.3, 0.4),       # fp32, D=64, Sq=3, mid-band blocks
    (4, 2, 4, 2, 256, torch.bfloat16, 0.3, 0.4),     # D=256 (config 4 head_dim)
    (3, 2, 2, 1, 256, torch.float32, 0.5, 0.0),
]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("mode", [1, 2, 3])
def test_scorer_vs_oracle(case, mode):
    from orthocache_b200 import synthetic as syn, score_blocks
    nb, hkv, hq, sq, d, dt, fs, fm = case
    kinds = syn.block_kinds(nb, fs, fm, seed=nb)
    k = syn.make_keys(nb, hkv, d, kinds, seed=nb, device="cuda", dtype=dt)
    q = syn.make_queries(sq, hq, d, seed=nb, device="cuda", dtype=dt)
    kf, qf = host(k).astype(np.float32), host(q).astype(np.float32)
    ref0 = O.score_blocks(qf, kf, -1e30, 5.0)
    tau, _ = syn.calibrate_tau(torch.tensor(ref0["zeta"]), torch.tensor(ref0["bound_max"]), 5.0, fs)
    ref = O.score_blocks(qf, kf, tau, 5.0)
    r = score_blocks(k, q, tau=tau, zeta_max=5.0, want=("dc", "e_low", "e_mid", "e_high", "zeta", "bound_max",
                                                          "bounds", "keep"), mode=mode)
    for n in ("e_low", "e_mid", "e_high"):
        np.testing.assert_allclose(host(r[n]), ref[n], rtol=2e-5, atol=1e-3)
    np.testing.assert_allclose(host(r["dc"]), ref["dc"], rtol=1e-5, atol=2e-4)
    np.testing.assert_allclose(host(r["zeta"]), ref["zeta"], rtol=2e-5)
    np.testing.assert_allclose(host(r["bound_max"]), ref["bound_max"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(host(r["bounds"]), O.query_aware_bounds(qf, kf), rtol=1e-5, atol=1e-5)
    assert_mask_parity(host(r["keep"]), ref["keep"], ref["zeta"], ref["bound_max"], tau, 5.0)


def test_scorer_batched_matches_per_item():
    from orthocache_b200 import synthetic as syn, score_blocks
    ks, qs = [], []
    for b in range(3):
        ks.append(syn.make_keys(4, 2, 128, syn.block_kinds(4, 0.5, seed=b), seed=b, device="cuda"))
        qs.append(syn.make_queries(2, 8, 128, seed=b, device="cuda"))
    kb, qb = torch.stack(ks), torch.stack(qs)
    rb = score_blocks(kb, qb, tau=1.0, zeta_max=5.0, want=("zeta", "bound_max", "keep"))
    for b in range(3):
        r = score_blocks(ks[b], qs[b], tau=1.0, zeta_max=5.0, want=("zeta", "bound_max", "keep"))
        for n in r:
            assert torch.equal(rb[n][b], r[n])


def test_scorer_custom_bands_use_full_butterfly():
    rs = np.random.RandomState(11)
    k = rs.randn(1024, 2, 64).astype(np.float32)
    bands = ((1, 10), (10, 300), (300, 512))
    dc, lo, mi, hi = oc().compute_spectral_bands(dev(k), 512, *bands)
    rdc, rlo, rmi, rhi = O.spectral_bands(k, 512, *bands)
    for g, w in ((lo, rlo), (mi, rmi), (hi, rhi)):
        np.testing.assert_allclose(host(g), w, rtol=2e-5)
    assert np.array_equal(host(dc), rdc)  # coefficient 0 of the exact butterfly


def test_scorer_edge_errors():
    from orthocache_b200 import score_blocks, _lib
    with pytest.raises(ValueError):
        score_blocks(torch.zeros(1000, 2, 64, device="cuda"))
    with pytest.raises(_lib.OrthoCacheError):
        score_blocks(torch.zeros(512, 2, 96, device="cuda"))
    with pytest.raises(_lib.OrthoCacheError):  # Hq not a multiple of Hkv
        score_blocks(torch.zeros(512, 2, 64, device="cuda"), torch.zeros(1, 3, 64, device="cuda"))
    r = score_blocks(torch.zeros(0, 2, 64, device="cuda"), want=("zeta",))
    assert r["zeta"].shape == (0, 2)


def test_tma_scorer_status_clean_and_matches_register_path():
    """The bulk-tensor pipeline and the per-thread-load scorer agree bit for bit
    on a multi-tile, multi-batch input, and no bounded wait gave up."""
    from orthocache_b200 import synthetic as syn, score_blocks, _lib
    nb = 300  # > SM count: several tiles per CTA, uneven split
    k = syn.make_keys(nb, 4, 128, syn.block_kinds(nb, 0.5, seed=9), seed=9, device="cuda")
    q = syn.make_queries(1, 16, 128, seed=9, device="cuda")
    kb = torch.stack([k, k.flip(0)])
    qb = torch.stack([q, -q])
    want = ("dc", "e_low", "e_mid", "e_high", "zeta", "bound_max", "keep")
    r1 = score_blocks(kb, qb, tau=0.0, zeta_max=5.0, want=want, mode=1)
    r3 = score_blocks(kb, qb, tau=0.0, zeta_max=5.0, want=want, mode=3)
    for n in want:
        if n in ("keep",):
            assert torch.equal(r1[n], r3[n])
        else:
            torch.testing.assert_close(r1[n], r3[n], rtol=2e-6, atol=1e-5)
    assert _lib.load().oc_device_status(1) == 0
