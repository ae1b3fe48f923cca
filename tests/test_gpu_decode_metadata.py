"""The decode step over write-time spectral metadata
(`oc_decode_step_from_metadata`): the blocks' gates from the DC
coefficients, E_AC and zeta written once per block by `oc_block_metadata`,
attention over the retained blocks, in the same one-launch layer as
`oc_decode_step`.  Against the CPU oracle: keep mask bit-exact away from the
thresholds, permutation and count exact, attention within 1e-2 relative /
2e-2 absolute (bf16).  Also: calls alternate with the key-scoring step on
one workspace, and a shape outside the one-kernel path (head_dim 64) takes
the separate kernels with the same results."""
import ctypes

import numpy as np
import pytest
import torch

from test_gpu_decode_fused import (ZMAX, _lib, check_against_oracle, decode, epoch, make_batch, tau_for,
                                   workspace)

pytestmark = pytest.mark.gpu


def metadata(k):
    B, S, Hkv, D = k.shape
    nb = S // 512
    dc = torch.empty((B, nb, Hkv, D), dtype=torch.float32, device="cuda")
    eac = torch.empty((B, nb, Hkv), dtype=torch.float32, device="cuda")
    zeta = torch.empty((B, nb, Hkv), dtype=torch.float32, device="cuda")
    rc = _lib().oc_block_metadata(k.data_ptr(), 1, B, S, Hkv, D, dc.data_ptr(), eac.data_ptr(), zeta.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib().oc_last_error()
    return dc, eac, zeta


def decode_meta(q, k, v, meta, tau, ws):
    lib = _lib()
    B, Sq, Hq, D = q.shape
    _, S, Hkv, _ = k.shape
    nb = S // 512
    dc, eac, zeta = meta
    keep = torch.full((B, nb, Hkv), 7, dtype=torch.uint8, device="cuda")
    perm = torch.full((B, nb), -5, dtype=torch.int32, device="cuda")
    count = torch.full((B,), -5, dtype=torch.int32, device="cuda")
    out = torch.full((B, Sq, Hq, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    rc = lib.oc_decode_step_from_metadata(q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, dc.data_ptr(),
                                          eac.data_ptr(), zeta.data_ptr(), B, Sq, Hq, Hkv, D, S,
                                          ctypes.c_float(tau), ctypes.c_float(ZMAX), keep.data_ptr(),
                                          perm.data_ptr(), count.data_ptr(), out.data_ptr(), 1, ws.data_ptr(),
                                          ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.oc_last_error()
    torch.cuda.synchronize()
    assert lib.oc_device_status(1) == 0, "a bounded wait gave up"
    return keep, perm, count, out


@pytest.mark.parametrize("B,nb,hq,hkv,sq,evicts", [
    (1, 128, 32, 8, 1, [0.75]),           # config 1 at full size
    (1, 128, 32, 8, 1, [0.5]),
    (1, 128, 32, 8, 1, [0.9]),
    (2, 40, 32, 8, 1, [0.5, 0.9]),        # two batch rows, different retained counts
    (3, 12, 16, 4, 2, [0.6, 0.0, 1.0]),   # R = 8 rows; nothing evicted; everything evicted
    (1, 2, 4, 1, 1, [0.5]),               # a grid of 2 CTAs
])
def test_metadata_decode_vs_oracle(B, nb, hq, hkv, sq, evicts):
    q, k, v = make_batch(B, nb, hq, hkv, 128, sq, evicts, seed=77 * nb + B)
    tau = tau_for(q[0], k[0], evicts[0])
    meta = metadata(k)
    ws = workspace(B, sq, hq, hkv, 128, nb * 512)
    keep, perm, count, out = decode_meta(q, k, v, meta, tau, ws)
    check_against_oracle(q, k, v, tau, keep, perm, count, out)
    assert epoch(ws) == 1, "the call did not run the fused kernel"


def test_metadata_and_key_decode_share_a_workspace():
    """Metadata and key-scoring calls alternate on one workspace; each equals
    the oracle and the two agree on mask, permutation and count."""
    B, nb, hq, hkv, sq = 2, 24, 16, 4, 1
    ws = workspace(B, sq, hq, hkv, 128, nb * 512)
    for it, ev in enumerate([[0.5, 0.75], [0.9, 0.25]]):
        q, k, v = make_batch(B, nb, hq, hkv, 128, sq, ev, seed=300 + it)
        tau = tau_for(q[0], k[0], ev[0])
        meta = metadata(k)
        km, pm, cm, om = decode_meta(q, k, v, meta, tau, ws)
        check_against_oracle(q, k, v, tau, km, pm, cm, om)
        kk, pk, ck, ok = decode(q, k, v, tau, ws)
        check_against_oracle(q, k, v, tau, kk, pk, ck, ok)
        assert torch.equal(cm, ck)
    assert epoch(ws) == 4


def test_metadata_decode_separate_kernels_head_dim_64():
    """head_dim 64 is outside the one-kernel layer: the separate metadata
    gates, compaction and split-KV attention run, with the oracle's results."""
    from oracle import oc_oracle as O
    from gpu_util import host, ATT_RTOL, ATT_ATOL
    B, nb, hq, hkv, sq, d = 1, 16, 8, 2, 1, 64
    q, k, v = make_batch(B, nb, hq, hkv, d, sq, [0.6], seed=5)
    tau = tau_for(q[0], k[0], 0.6)
    meta = metadata(k)
    ws = torch.zeros(_lib().oc_decode_step_workspace_bytes(B, sq, hq, hkv, d, nb * 512), dtype=torch.uint8,
                     device="cuda")
    keep, perm, count, out = decode_meta(q, k, v, meta, tau, ws)
    assert epoch(ws) == 0
    qf, kf, vf = host(q[0]), host(k[0]), host(v[0])
    got = host(keep[0]).astype(bool)
    rp, rn = O.stream_compact_mask(got)
    assert int(count[0]) == rn and np.array_equal(host(perm[0]), rp)
    ref = O.indirect_attention(qf, kf, vf, rp, rn)
    np.testing.assert_allclose(host(out[0]).astype(np.float32), ref, rtol=ATT_RTOL, atol=ATT_ATOL)


def test_metadata_cache_decode_step_python_api():
    """SpectralMetadataCache.decode_step (the Python entry of the same
    kernel) against the oracle, workspace reused across two steps."""
    from orthocache_b200 import SpectralMetadataCache
    B, nb, hq, hkv, sq = 2, 32, 32, 8, 1
    q, k, v = make_batch(B, nb, hq, hkv, 128, sq, [0.75, 0.5], seed=900)
    tau = tau_for(q[0], k[0], 0.75)
    cache = SpectralMetadataCache.from_keys(k)
    ws = workspace(B, sq, hq, hkv, 128, nb * 512)
    for _ in range(2):
        out, keep, perm, count = cache.decode_step(q, k, v, tau, ZMAX, workspace=ws)
        torch.cuda.synchronize()
        check_against_oracle(q, k, v, tau, keep, perm, count, out)
    assert epoch(ws) == 2
