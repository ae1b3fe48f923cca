"""Write-time spectral metadata on the GPU (oc_block_metadata,
oc_score_from_metadata, SpectralMetadataCache) against the CPU oracle and
against the key-reading scorer: dc / E_AC / zeta within the scorer's float32
summation-order tolerance (2e-5 relative), bounds within 1e-5, the keep mask
bit-exact away from the thresholds, and a partial refresh after rewriting
blocks equal to a rebuild."""
import numpy as np
import pytest
import torch

from oracle import oc_oracle as O
from gpu_util import host, assert_mask_parity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nb,hq,hkv,d,sq,dtype", [
    (24, 16, 4, 128, 1, torch.bfloat16),
    (128, 32, 8, 128, 1, torch.bfloat16),   # config 1 size
    (10, 8, 2, 64, 3, torch.float32),
    # long query chunks: the bounds run as the tiled GEMM (rows per KV head > 32)
    (16, 8, 2, 128, 100, torch.bfloat16),
    (12, 8, 4, 64, 40, torch.float32),
    (70, 32, 8, 128, 256, torch.bfloat16),   # two block tiles of 64, 1024 rows per KV head
])
def test_metadata_cache_vs_oracle(nb, hq, hkv, d, sq, dtype):
    import orthocache_b200 as oc
    from orthocache_b200 import synthetic as syn
    kinds = syn.block_kinds(nb, 0.5, seed=nb + d)
    k = syn.make_keys(nb, hkv, d, kinds, seed=nb + d, dtype=dtype)
    q = syn.make_queries(sq, hq, d, seed=nb + d, dtype=dtype)
    kf, qf = host(k), host(q)
    cache = oc.SpectralMetadataCache.from_keys(k)
    dc, e_ac, zeta = O.block_metadata(kf)
    np.testing.assert_allclose(host(cache.dc[0]), dc, rtol=2e-5, atol=2e-5 * float(np.abs(dc).max()))
    np.testing.assert_allclose(host(cache.e_ac[0]), e_ac, rtol=2e-5)
    np.testing.assert_allclose(host(cache.zeta[0]), zeta, rtol=2e-5)
    r0 = O.score_blocks(qf, kf, -1e30, 5.0)
    tau, _ = syn.calibrate_tau(torch.tensor(r0["zeta"]), torch.tensor(r0["bound_max"]), 5.0, 0.5)
    keep, bmax, bounds = cache.multiband_mask(q, tau, 5.0, want_bounds=True)
    np.testing.assert_allclose(host(bounds), O.query_aware_bounds(qf, kf), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(host(bmax), r0["bound_max"], rtol=1e-5, atol=1e-5)
    want = (r0["bound_max"] >= np.float32(tau)) & (r0["zeta"] <= np.float32(5.0))
    assert_mask_parity(host(keep), want, r0["zeta"], r0["bound_max"], tau, 5.0)
    # without per-row bounds the maxima come from a separate fast path (scale
    # applied once per block): the same floats and the same mask
    keep2, bmax2 = cache.multiband_mask(q, tau, 5.0)
    assert torch.equal(bmax2, bmax) and torch.equal(keep2, keep)
    # the same mask as the key-reading scorer
    sc = oc.score_blocks(k, q, tau=tau, zeta_max=5.0, want=("keep",))
    assert_mask_parity(host(keep), host(sc["keep"]), r0["zeta"], r0["bound_max"], tau, 5.0)


def test_metadata_cache_refresh_after_rewrite():
    """Blocks 3..4 of batch row 1 are rewritten; refreshing just those blocks
    gives the metadata of a full rebuild."""
    import orthocache_b200 as oc
    from orthocache_b200 import synthetic as syn
    B, nb, hkv, d = 2, 9, 4, 128
    k = torch.stack([syn.make_keys(nb, hkv, d, syn.block_kinds(nb, 0.5, seed=b), seed=b) for b in range(B)])
    cache = oc.SpectralMetadataCache.from_keys(k)
    g = torch.Generator(device="cuda").manual_seed(77)
    k[1, 3 * 512:5 * 512] = torch.randn((2 * 512, hkv, d), generator=g, device="cuda").to(k.dtype)
    cache.update_blocks(k, 3, 2)
    ref = oc.SpectralMetadataCache.from_keys(k)
    for name in ("dc", "e_ac", "zeta"):
        assert torch.equal(getattr(cache, name), getattr(ref, name)), name
