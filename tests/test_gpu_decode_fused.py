"""The one-launch decode layer (scorer, block decisions, attention over the
retained blocks and merge in one persistent kernel) through the C ABI
`oc_decode_step`, against the CPU oracle: keep mask bit-exact away from the
thresholds, the stable active-first permutation and count exact, attention
within the parity contract's 1e-2 relative / 2e-2 absolute (bf16 inputs).

Also checks the workspace contract of the fused path: the workspace is
zero-filled once, then calls follow each other on it (the kernel keeps an
epoch and two counter sets there), interleaved with calls the fused kernel
does not cover and with CUDA-graph replays."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oc_oracle as O
from gpu_util import host, assert_mask_parity, ATT_RTOL, ATT_ATOL

pytestmark = pytest.mark.gpu
ZMAX = 5.0


def _lib():
    from orthocache_b200 import _lib
    return _lib.load()


def make_batch(B, nb, hq, hkv, d, sq, evicts, seed):
    """Per batch row: keys with its own smooth fraction, values, queries."""
    from orthocache_b200 import synthetic as syn
    ks, vs, qs = [], [], []
    for b in range(B):
        kinds = syn.block_kinds(nb, min(evicts[b], 0.99), seed=seed + b)
        ks.append(syn.make_keys(nb, hkv, d, kinds, seed=seed + b))
        vs.append(syn.make_values(nb * 512, hkv, d, seed=seed + b))
        qs.append(syn.make_queries(sq, hq, d, seed=seed + b))
    return torch.stack(qs), torch.stack(ks), torch.stack(vs)


def tau_for(q, k, evict):
    from orthocache_b200 import synthetic as syn
    r0 = O.score_blocks(host(q), host(k), -1e30, ZMAX)
    tau, _ = syn.calibrate_tau(torch.tensor(r0["zeta"]), torch.tensor(r0["bound_max"]), ZMAX, evict)
    return tau


def epoch(ws):
    """Fused calls made on this workspace (its first int32)."""
    return int(ws[:4].view(torch.int32)[0])


def decode(q, k, v, tau, ws, out_dtype=torch.bfloat16):
    lib = _lib()
    B, Sq, Hq, D = q.shape
    _, S, Hkv, _ = k.shape
    nb = S // 512
    keep = torch.full((B, nb, Hkv), 7, dtype=torch.uint8, device="cuda")
    perm = torch.full((B, nb), -5, dtype=torch.int32, device="cuda")
    count = torch.full((B,), -5, dtype=torch.int32, device="cuda")
    out = torch.full((B, Sq, Hq, D), float("nan"), dtype=out_dtype, device="cuda")
    rc = lib.oc_decode_step(q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, B, Sq, Hq, Hkv, D, S,
                            ctypes.c_float(tau), ctypes.c_float(ZMAX), keep.data_ptr(), perm.data_ptr(),
                            count.data_ptr(), out.data_ptr(), 1 if out_dtype == torch.bfloat16 else 0,
                            ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.oc_last_error()
    torch.cuda.synchronize()
    assert lib.oc_device_status(1) == 0, "a bounded wait gave up"
    return keep, perm, count, out


def workspace(B, Sq, Hq, Hkv, D, S):
    n = _lib().oc_decode_step_workspace_bytes(B, Sq, Hq, Hkv, D, S)
    return torch.zeros(n, dtype=torch.uint8, device="cuda")


def check_against_oracle(q, k, v, tau, keep, perm, count, out):
    B = q.shape[0]
    for b in range(B):
        qf, kf, vf = host(q[b]), host(k[b]), host(v[b])
        r0 = O.score_blocks(qf, kf, -1e30, ZMAX)
        ref_keep = (r0["bound_max"] >= np.float32(tau)) & (r0["zeta"] <= np.float32(ZMAX))
        got = host(keep[b]).astype(bool)
        assert_mask_parity(got, ref_keep, r0["zeta"], r0["bound_max"], tau, ZMAX)
        rp, rn = O.stream_compact_mask(got)
        assert int(count[b]) == rn, (b, int(count[b]), rn)
        assert np.array_equal(host(perm[b]), rp), b
        ref = O.indirect_attention(qf, kf, vf, rp, rn)
        np.testing.assert_allclose(host(out[b]).astype(np.float32), ref, rtol=ATT_RTOL, atol=ATT_ATOL)


@pytest.mark.parametrize("B,nb,hq,hkv,sq,evicts", [
    (1, 128, 32, 8, 1, [0.75]),           # config 1 at full size
    (1, 128, 32, 8, 1, [0.5]),            # config 1's eviction sweep at full size
    (1, 128, 32, 8, 1, [0.9]),
    (1, 16, 8, 8, 1, [0.5]),              # config 0
    (2, 40, 32, 8, 1, [0.5, 0.9]),        # two batch rows, different retained counts
    (3, 12, 16, 4, 2, [0.6, 0.0, 1.0]),   # R = 8 rows; nothing evicted; everything evicted
    (4, 6, 64, 16, 1, [0.5, 0.5, 0.7, 0.3]),  # 64 (batch, head) groups on the grid
    (1, 2, 4, 1, 1, [0.5]),               # fewer tiles than SMs: a grid of 2 CTAs
])
def test_fused_decode_vs_oracle(B, nb, hq, hkv, sq, evicts):
    q, k, v = make_batch(B, nb, hq, hkv, 128, sq, evicts, seed=31 * nb + B)
    tau = tau_for(q[0], k[0], evicts[0])
    ws = workspace(B, sq, hq, hkv, 128, nb * 512)
    keep, perm, count, out = decode(q, k, v, tau, ws)
    check_against_oracle(q, k, v, tau, keep, perm, count, out)
    assert epoch(ws) == 1, "the call did not run the fused kernel"


def test_fused_decode_repeated_calls_and_mixed_shapes():
    """Back-to-back calls on one workspace (new inputs each time), with a call
    the fused kernel does not cover (head_dim 64) in between, and a float32
    output; every result against the oracle."""
    B, nb, hq, hkv, sq = 2, 24, 16, 4, 1
    S = nb * 512
    ws = workspace(B, sq, hq, hkv, 128, S)
    n64 = _lib().oc_decode_step_workspace_bytes(B, sq, hq, hkv, 64, S)
    assert n64 <= ws.numel()
    for it, ev in enumerate([[0.5, 0.75], [0.9, 0.25], [0.75, 0.75]]):
        q, k, v = make_batch(B, nb, hq, hkv, 128, sq, ev, seed=100 + it)
        tau = tau_for(q[0], k[0], ev[0])
        out_dt = torch.float32 if it == 2 else torch.bfloat16
        check_against_oracle(q, k, v, tau, *decode(q, k, v, tau, ws, out_dt))
        if it == 0:
            q6, k6, v6 = make_batch(B, nb, hq, hkv, 64, sq, [0.5, 0.5], seed=7)
            tau6 = tau_for(q6[0], k6[0], 0.5)
            check_against_oracle(q6, k6, v6, tau6, *decode(q6, k6, v6, tau6, ws))
    assert epoch(ws) == 3  # the head_dim 64 call took the separate kernels


def test_fused_decode_in_cuda_graph():
    """The layer captured once in a CUDA graph and replayed on new queries
    (each replay advances the epoch and switches counter sets)."""
    B, nb, hq, hkv, sq = 1, 32, 32, 8, 1
    q, k, v = make_batch(B, nb, hq, hkv, 128, sq, [0.75], seed=5)
    tau = tau_for(q[0], k[0], 0.75)
    ws = workspace(B, sq, hq, hkv, 128, nb * 512)
    lib = _lib()
    qbuf = q.clone()
    keep = torch.empty((B, nb, hkv), dtype=torch.uint8, device="cuda")
    perm = torch.empty((B, nb), dtype=torch.int32, device="cuda")
    count = torch.empty((B,), dtype=torch.int32, device="cuda")
    out = torch.empty((B, sq, hq, 128), dtype=torch.bfloat16, device="cuda")

    def call():
        rc = lib.oc_decode_step(qbuf.data_ptr(), k.data_ptr(), v.data_ptr(), 1, B, sq, hq, hkv, 128, nb * 512,
                                ctypes.c_float(tau), ctypes.c_float(ZMAX), keep.data_ptr(), perm.data_ptr(),
                                count.data_ptr(), out.data_ptr(), 1, ws.data_ptr(), ws.numel(),
                                torch.cuda.current_stream().cuda_stream)
        assert rc == 0

    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        call()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        call()
    e0 = epoch(ws)
    for seed in (11, 12, 13):
        qn = make_batch(B, nb, hq, hkv, 128, sq, [0.75], seed=seed)[0]
        qbuf.copy_(qn)
        g.replay()
        torch.cuda.synchronize()
        assert lib.oc_device_status(1) == 0
        check_against_oracle(qbuf, k, v, tau, keep, perm, count, out)
    assert epoch(ws) == e0 + 3


@pytest.mark.parametrize("sq,hq,hkv,evicts", [(1, 32, 8, [0.75, 0.6]), (2, 16, 4, [0.9, 0.5, 0.7])])
def test_fused_shard_partials_and_packed_merge(sq, hq, hkv, evicts):
    """Sequence-parallel decode on one GPU: each shard runs
    oc_decode_step_partial into its slice of one packed buffer
    [m | l | o], oc_merge_partials_packed combines the shards, and the result
    equals attention over the union of every shard's retained blocks."""
    lib = _lib()
    P, nb, d = len(evicts), 20, 128
    rows = sq * hq
    shards = [make_batch(1, nb, hq, hkv, d, sq, [ev], seed=400 + 7 * p) for p, ev in enumerate(evicts)]
    q = shards[0][0]
    tau = tau_for(q[0], shards[0][1][0], evicts[0])
    packed = torch.full((P, rows * (d + 2)), float("nan"), dtype=torch.float32, device="cuda")
    kept_k, kept_v, n_all = [], [], 0
    for p, (_, k, v) in enumerate(shards):
        ws = workspace(1, sq, hq, hkv, d, nb * 512)
        keep = torch.empty((1, nb, hkv), dtype=torch.uint8, device="cuda")
        perm = torch.empty((1, nb), dtype=torch.int32, device="cuda")
        count = torch.empty((1,), dtype=torch.int32, device="cuda")
        buf = packed[p]
        rc = lib.oc_decode_step_partial(q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, 1, sq, hq, hkv, d, nb * 512,
                                        ctypes.c_float(tau), ctypes.c_float(ZMAX), keep.data_ptr(), perm.data_ptr(),
                                        count.data_ptr(), buf.data_ptr(), buf[rows:].data_ptr(),
                                        buf[2 * rows:].data_ptr(), ws.data_ptr(), ws.numel(),
                                        torch.cuda.current_stream().cuda_stream)
        assert rc == 0, lib.oc_last_error()
        torch.cuda.synchronize()
        assert epoch(ws) == 1
        rp, rn = O.stream_compact_mask(host(keep[0]).astype(bool))
        assert int(count[0]) == rn and np.array_equal(host(perm[0]), rp)
        kf, vf = host(k[0]).reshape(nb, 512, hkv, d), host(v[0]).reshape(nb, 512, hkv, d)
        kept_k.append(kf[rp[:rn]])
        kept_v.append(vf[rp[:rn]])
        n_all += rn
    out = torch.empty((rows, d), dtype=torch.bfloat16, device="cuda")
    rc = lib.oc_merge_partials_packed(packed.data_ptr(), P, rows, d, out.data_ptr(), 1,
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.oc_last_error()
    torch.cuda.synchronize()
    kc = np.concatenate(kept_k).reshape(-1, hkv, d)
    vc = np.concatenate(kept_v).reshape(-1, hkv, d)
    ref = O.indirect_attention(host(q[0]), kc, vc, np.arange(n_all, dtype=np.int32), n_all)
    np.testing.assert_allclose(host(out).reshape(ref.shape), ref, rtol=ATT_RTOL, atol=ATT_ATOL)
