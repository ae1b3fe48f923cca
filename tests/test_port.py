"""The C port used as the timed CPU baseline agrees with the oracle (CPU only)."""
import numpy as np
import torch

from oracle import oc_oracle as O, port
from orthocache_b200 import synthetic as syn


def bits(t):
    return t.view(torch.int16).numpy().view(np.uint16)


def test_port_decode_matches_oracle():
    nb, hkv, hq = 8, 4, 8
    kinds = syn.block_kinds(nb, 0.5, seed=1)
    k = syn.make_keys(nb, hkv, 64, kinds, seed=1, device="cpu")
    v = syn.make_values(nb * 512, hkv, 64, seed=1, device="cpu")
    q = syn.make_queries(2, hq, 64, seed=1, device="cpu")
    kf, qf, vf = k.float().numpy(), q.float().numpy(), v.float().numpy()
    r0 = O.score_blocks(qf, kf, -1e30, 5.0)
    tau, kept = syn.calibrate_tau(torch.tensor(r0["zeta"]), torch.tensor(r0["bound_max"]), 5.0, 0.5)
    keep, perm, n, out = port.decode(bits(k), bits(v), bits(q), tau, 5.0)
    ref = O.score_blocks(qf, kf, tau, 5.0)
    assert np.array_equal(keep, ref["keep"])
    rp, rn = O.stream_compact_mask(ref["keep"])
    assert n == rn == kept and np.array_equal(perm, rp)
    np.testing.assert_allclose(out, O.indirect_attention(qf, kf, vf, rp, rn), rtol=1e-4, atol=1e-5)


def test_synthetic_spectra_and_calibration():
    """Smooth blocks have large ζ, noise blocks ζ ≈ 4 (natural-order bands), and
    calibrate_tau hits the requested union eviction exactly."""
    nb = 16
    kinds = syn.block_kinds(nb, 0.75, seed=3)
    assert (kinds == syn.KIND_SMOOTH).sum() == 12
    k = syn.make_keys(nb, 4, 64, kinds, seed=3, device="cpu")
    q = syn.make_queries(1, 8, 64, seed=3, device="cpu")
    r = O.score_blocks(q.float().numpy(), k.float().numpy(), -1e30, 5.0)
    assert (r["zeta"][kinds == syn.KIND_SMOOTH] > 5.0).all()
    assert (np.abs(r["zeta"][kinds == syn.KIND_NOISE] - 4.06) < 0.5).all()
    for e in (0.75, 0.875):
        tau, kept = syn.calibrate_tau(torch.tensor(r["zeta"]), torch.tensor(r["bound_max"]), 5.0, e)
        keep = O.score_blocks(q.float().numpy(), k.float().numpy(), tau, 5.0)["keep"]
        assert keep.any(1).sum() == kept == round((1 - e) * nb)
        assert not O.near_threshold(r["zeta"], r["bound_max"], tau, 5.0).any()
