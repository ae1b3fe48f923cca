"""Pin the CPU oracle to the reference: golden vectors from the reference's own
NumPy model (tests/golden/make_golden.py) and the known answers of the
reference's test suite.  CPU only."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

from make_golden import inputs  # noqa: E402
from oracle import oc_oracle as O  # noqa: E402

GOLD = np.load(os.path.join(HERE, "golden", "reference_golden.npz"))
X = inputs()


def test_fwht_2d_matches_reference():          # test_fwht.py:8-20
    np.testing.assert_allclose(O.fwht_512(X["fwht2d_x"]), GOLD["fwht2d"], rtol=1e-5, atol=1e-5)


def test_fwht_1d_matches_reference():          # test_fwht.py:22-29
    np.testing.assert_allclose(O.fwht_512(X["fwht1d_x"]), GOLD["fwht1d"], rtol=1e-5, atol=1e-5)


def test_fwht_is_involution_up_to_scale():
    x = X["fwht2d_x"]
    np.testing.assert_allclose(O.fwht_512(O.fwht_512(x)), x, rtol=1e-4, atol=1e-4)


def test_block_energy_matches_reference():     # test_energy.py:16-31
    np.testing.assert_allclose(O.block_energy(X["energy_keys"]), GOLD["energy"], rtol=1e-5, atol=1e-5)


def test_bounds_match_reference():             # test_energy.py:33-52
    np.testing.assert_allclose(O.query_aware_bounds(X["bounds_q"], X["bounds_keys"]), GOLD["bounds"],
                               rtol=1e-5, atol=1e-5)


def test_bands_match_reference():              # test_spectral_bands.py:28-52
    dc, lo, mi, hi = O.spectral_bands(X["bands_keys"])
    for got, key in ((dc, "bands_dc"), (lo, "bands_low"), (mi, "bands_mid"), (hi, "bands_high")):
        np.testing.assert_allclose(got, GOLD[key], rtol=1e-4, atol=1e-4)


def test_zeta_matches_reference():             # test_spectral_bands.py:55-67
    np.testing.assert_allclose(O.spectral_decay_ratio(X["zeta_keys"]), GOLD["zeta"], rtol=1e-4, atol=1e-4)


def test_two_gate_mask_matches_reference():    # test_spectral_bands.py:177-213
    m = O.multiband_mask(X["twogate_q"], X["twogate_keys"], -100.0, 1.0)
    np.testing.assert_array_equal(m, GOLD["twogate_mask"])
    assert not m.all()


def test_mask_inside_distribution_matches_reference():
    tau, zmax = float(GOLD["mask_tau"]), float(GOLD["mask_zeta_max"])
    np.testing.assert_allclose(O.max_bounds(X["mask_q"], X["mask_keys"]), GOLD["mask_maxbound"], rtol=1e-5)
    np.testing.assert_allclose(O.spectral_decay_ratio(X["mask_keys"]), GOLD["mask_zeta"], rtol=1e-5)
    m = O.multiband_mask(X["mask_q"], X["mask_keys"], tau, zmax)
    np.testing.assert_array_equal(m, GOLD["mask"])
    assert m.any() and not m.all()


def _walsh(j):
    i = np.arange(512)
    return np.array([(-1.0) ** bin(j & t).count("1") for t in i])


def test_zeta_high_for_alternating_noise():    # test_spectral_bands.py:70-86
    rs = np.random.RandomState(99)
    blk = np.stack([(1.0 if i % 2 == 0 else -1.0) * rs.randn(64) * 2.0 for i in range(512)])
    _, lo, _, hi = O.spectral_bands(blk[:, None, :].astype(np.float32))
    assert float(O.zeta_from_energies(lo, hi)[0, 0]) > 1.0


def test_zeta_low_for_walsh_coherent():        # test_spectral_bands.py:89-117
    rng = np.random.RandomState(42)
    blk = sum(np.outer(_walsh(j), rng.randn(64) * 0.5) for j in range(1, 16))
    _, lo, _, hi = O.spectral_bands(blk[:, None, :].astype(np.float32))
    assert float(O.zeta_from_energies(lo, hi)[0, 0]) < 0.01


def test_equal_variance_different_zeta():      # test_spectral_bands.py:120-174
    rng_a = np.random.RandomState(2026)
    a = sum(np.outer(_walsh(j), rng_a.randn(64) * 0.5) for j in range(1, 16))
    b = np.random.RandomState(42).randn(512, 64)
    ma, mb = a.mean(0), b.mean(0)
    b = mb + (b - mb) * np.sqrt(np.sum((a - ma) ** 2) / np.sum((b - mb) ** 2))
    za = O.spectral_decay_ratio(a[:, None, :].astype(np.float32))[0, 0]
    zb = O.spectral_decay_ratio(b[:, None, :].astype(np.float32))[0, 0]
    assert za < 0.01 and zb > 1.0


def test_stream_compact_known_answers():       # test_alltoallv.py:60-67, test_distributed.py:57-64
    perm, n = O.stream_compact_mask(np.array([False, True, False, True, True, False]))
    assert n == 3 and list(perm[:3]) == [1, 3, 4] and list(perm[3:]) == [0, 2, 5]
    perm, n = O.stream_compact_mask(np.array([True, False, True, True, False]))
    assert n == 3 and list(perm[:3]) == [0, 2, 3]
    perm, n = O.stream_compact_mask(np.zeros(8, bool))
    assert n == 0 and list(perm) == list(range(8))
    # union over heads (compaction.py:65)
    perm, n = O.stream_compact_mask(np.array([[0, 0], [0, 1], [1, 0], [0, 0]], bool))
    assert n == 2 and list(perm) == [1, 2, 0, 3]


def test_offsets_known_answers():              # test_alltoallv.py:76-105
    off, tot = O.compute_offsets([3, 2, 5, 1])
    assert list(off) == [0, 3, 5, 10] and tot == 11
    off, tot = O.compute_offsets([0, 0, 0, 0])
    assert list(off) == [0, 0, 0, 0] and tot == 0
    off, tot = O.compute_offsets([7])
    assert list(off) == [0] and tot == 7


def test_buckets_known_answers():              # test_indirect_attention.py:55-74
    for b in (1, 2, 4, 8, 16, 32, 64, 128, 256, 512):
        assert O.next_bucket(b) == b
    assert [O.next_bucket(n) for n in (3, 5, 9, 17)] == [4, 8, 16, 32]
    assert O.next_bucket(612) == 612


def test_stratified_buckets():                 # phase_e_stratified.py:182-197
    assert O.stratified_buckets(16) == (4, 8, 12, 16)
    assert O.stratified_buckets(1) == (1, 1, 1, 1)
    assert O.stratified_buckets(2) == (1, 2, 2, 2)
    assert O.stratified_bucket(5, (4, 8, 12, 16)) == 8
    assert O.stratified_bucket(16, (4, 8, 12, 16)) == 16


def test_global_block_index():                 # distributed_attention.py:182-191
    order, tot = O.global_block_index([2, 0, 3], 4)
    assert tot == 5 and list(order[:5]) == [0, 1, 8, 9, 10]


def test_unpack_offsets():                     # test_alltoallv.py:185-212
    kv = np.arange(3 * 4 * 512 * 2 * 4, dtype=np.float32).reshape(3 * 4 * 512, 2, 4)
    _, off = O.unpack_received(kv, [1, 3, 2], 3, 4)
    assert list(off) == [0, 512, 4 * 512]


def test_oracle_attention_matches_bruteforce():
    rs = np.random.RandomState(3)
    q = rs.randn(2, 4, 16).astype(np.float32)
    k = rs.randn(4 * 64, 2, 16).astype(np.float32)
    v = rs.randn(4 * 64, 2, 16).astype(np.float32)
    out = O.indirect_attention(q, k, v, np.array([1, 3, 0, 2]), 2, block_size=64)
    toks = np.r_[64:128, 192:256]
    for s in range(2):
        for hq in range(4):
            h = hq // 2
            lg = k[toks, h] @ q[s, hq] / 4.0
            w = np.exp(lg - lg.max())
            w /= w.sum()
            np.testing.assert_allclose(out[s, hq], w @ v[toks, h], rtol=1e-5, atol=1e-5)
    assert np.all(O.indirect_attention(q, k, v, np.arange(4), 0, block_size=64) == 0)


def test_sparse_attention_equals_indirect_on_union_mask():  # test_compaction.py:162-183
    rs = np.random.RandomState(5)
    q = rs.randn(3, 2, 16).astype(np.float32)
    k = rs.randn(6 * 64, 2, 16).astype(np.float32)
    v = rs.randn(6 * 64, 2, 16).astype(np.float32)
    m = np.array([1, 0, 1, 1, 0, 0], bool)
    perm, n = O.stream_compact_mask(m)
    a = O.indirect_attention(q, k, v, perm, n, block_size=64)
    b = O.block_sparse_attention(q, k, v, np.repeat(m[:, None], 2, 1), block_size=64)
    np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-6)


def test_bounds_from_write_time_metadata_match_reference():  # test_energy.py:33-52
    """The bound rebuilt from cached (dc, E_AC) equals the reference's bound."""
    dc, e_ac, _ = O.block_metadata(X["bounds_keys"])
    np.testing.assert_allclose(O.bounds_from_metadata(X["bounds_q"], dc, e_ac), GOLD["bounds"],
                               rtol=1e-5, atol=1e-5)


def test_partial_states_merge_to_the_union_attention():
    """Splitting the retained blocks over shards and merging the shards'
    (m, l, o) in log-sum-exp form gives the attention over the union
    (distributed_attention.py:95-128 applied across shards)."""
    rs = np.random.RandomState(7)
    q = rs.randn(2, 8, 16) * 0.5
    shards = [(rs.randn(4 * 8, 2, 16), rs.randn(4 * 8, 2, 16)) for _ in range(3)]
    perms = [np.array([2, 0, 1, 3]), np.array([1, 3, 0, 2]), np.array([0, 1, 2, 3])]
    counts = [2, 0, 3]
    parts = [O.partial_attention(q, k, v, p, n, block_size=8) for (k, v), p, n in zip(shards, perms, counts)]
    got = O.merge_partials(parts)
    k_all = np.concatenate([k for k, _ in shards])
    v_all = np.concatenate([v for _, v in shards])
    gperm = np.concatenate([p[:n] + 4 * i for i, (p, n) in enumerate(zip(perms, counts))])
    want = O.indirect_attention(q, k_all, v_all, gperm, len(gperm), block_size=8)
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)
    empty = O.merge_partials([O.partial_attention(q, *shards[1], perms[1], 0, block_size=8)])
    assert np.all(empty == 0)
