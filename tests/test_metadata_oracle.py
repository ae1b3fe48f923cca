"""Write-time spectral metadata in the oracle (CPU): the query-aware bound
rebuilt from the cached DC coefficients and E_AC equals the bound computed
from the keys (spectral_energy.py:141-177), so a cache of (dc, E_AC, zeta)
gives the same two-gate mask as compute_multiband_mask."""
import numpy as np

from oracle import oc_oracle as O


def _keys(seed, nb=3, h=2, d=16):
    rs = np.random.RandomState(seed)
    base = rs.randn(nb, 1, h, d)
    return (base + rs.randn(nb, 512, h, d) * rs.rand(nb, 1, h, 1)).reshape(nb * 512, h, d).astype(np.float32)


def test_bounds_from_metadata_equal_bounds_from_keys():
    for seed, hq in ((0, 2), (1, 4), (2, 8)):
        k = _keys(seed)
        q = np.random.RandomState(seed + 10).randn(3, hq, 16).astype(np.float32) * 0.25
        dc, e_ac, zeta = O.block_metadata(k)
        np.testing.assert_allclose(O.bounds_from_metadata(q, dc, e_ac), O.query_aware_bounds(q, k),
                                   rtol=1e-6, atol=1e-6)
        np.testing.assert_array_equal(zeta, O.spectral_decay_ratio(k))


def test_metadata_matches_score_blocks_and_mask():
    k = _keys(5, nb=4)
    q = np.random.RandomState(6).randn(1, 4, 16).astype(np.float32) * 0.25
    dc, e_ac, zeta = O.block_metadata(k)
    r = O.score_blocks(q, k, -1e30, np.inf)
    np.testing.assert_allclose(dc, r["dc"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(e_ac, r["e_low"] + r["e_mid"] + r["e_high"], rtol=1e-5)
    bmax = O.bounds_from_metadata(q, dc, e_ac).reshape(1, 4, 2, 2).max(axis=(0, 3))
    tau = float(np.median(bmax))
    want = O.multiband_mask(q, k, tau, 5.0)
    got = (bmax >= np.float32(tau)) & (zeta <= np.float32(5.0))
    near = O.near_threshold(zeta, bmax, tau, 5.0)
    assert not ((got != want) & ~near).any()
