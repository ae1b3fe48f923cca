"""Sequence-parallel path on the GPU: packing, the receive-side layout and
the global block index bit-exact against the oracle; attention over the
gathered blocks (replicated gather, stratified buckets) and the log-sum-exp
merge of per-shard partials against the oracle's attention over the union
of all shards' retained blocks.  P shards are emulated in one process (the
collective is a concatenation); the public entry points run on a one-rank
NCCL group."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist

from oracle import oc_oracle as O
from gpu_util import dev, host, ATT_RTOL, ATT_ATOL

pytestmark = pytest.mark.gpu

BS = 512


def _shards(P, nb, hkv, hq, d, seed):
    rs = np.random.RandomState(seed)
    ks, vs, ms = [], [], []
    for p in range(P):
        k = torch.randn(nb * BS, hkv, d, generator=torch.Generator().manual_seed(seed * 31 + p)).to(torch.bfloat16)
        v = torch.randn(nb * BS, hkv, d, generator=torch.Generator().manual_seed(seed * 37 + p)).to(torch.bfloat16)
        m = rs.rand(nb) < 0.4
        if p == 0:
            m[:] = False  # a shard with nothing retained
        ks.append(k)
        vs.append(v)
        ms.append(m)
    q = (torch.randn(1, hq, d, generator=torch.Generator().manual_seed(seed)) * d ** -0.5).to(torch.bfloat16)
    return q, ks, vs, ms


def _f32(t):
    return t.float().numpy()


def _oracle_union_attention(q, ks, vs, ms):
    """Attention over every shard's retained blocks (the union across shards)."""
    k_all = np.concatenate([_f32(k) for k in ks])
    v_all = np.concatenate([_f32(v) for v in vs])
    nb = ks[0].shape[0] // BS
    blocks = np.concatenate([np.nonzero(m)[0] + p * nb for p, m in enumerate(ms)]).astype(np.int32)
    return O.indirect_attention(_f32(q), k_all, v_all, blocks, len(blocks))


@pytest.mark.parametrize("P,nb,hkv,hq,d", [(3, 8, 2, 4, 128), (4, 6, 1, 2, 64)])
def test_pack_unpack_index_bit_exact(P, nb, hkv, hq, d):
    from orthocache_b200 import distributed as ocd
    q, ks, vs, ms = _shards(P, nb, hkv, hq, d, seed=P * 10 + nb)
    packed, counts = [], []
    for k, m in zip(ks, ms):
        idx, n = ocd.stream_compact(dev(m))
        rp, rn = O.stream_compact_mask(m)
        assert int(n) == rn and np.array_equal(host(idx), rp)
        pk = ocd.pack_active_blocks(k.cuda(), idx, n, nb)
        want = O.pack_active_blocks(_f32(k), rp, rn, nb)
        assert np.array_equal(_f32(pk.cpu()), want)
        packed.append(pk)
        counts.append(rn)
    recv = torch.cat(packed)  # what the all-gather delivers
    act, off = ocd.unpack_received_blocks(recv, torch.tensor(counts, dtype=torch.int32), P, nb)
    ract, roff = O.unpack_received(_f32(recv.cpu()), counts, P, nb)
    assert np.array_equal(_f32(act.cpu()), ract)
    assert np.array_equal(host(off), roff)
    order, total, offs = ocd.global_block_index(torch.tensor(counts, dtype=torch.int32), nb)
    rorder, rtotal = O.global_block_index(counts, nb)
    assert np.array_equal(host(order), rorder) and int(total) == rtotal
    assert np.array_equal(host(offs), O.compute_offsets(counts)[0])


@pytest.mark.parametrize("P,nb,hkv,hq,d", [(3, 8, 2, 4, 128), (4, 6, 1, 2, 64)])
def test_gathered_and_stratified_attention(P, nb, hkv, hq, d):
    from orthocache_b200 import distributed as ocd
    q, ks, vs, ms = _shards(P, nb, hkv, hq, d, seed=P * 10 + nb + 1)
    ref = _oracle_union_attention(q, ks, vs, ms)
    comp = [ocd.stream_compact(dev(m)) for m in ms]
    counts = [int(n) for _, n in comp]
    # replicated gather (distributed_attention.py:131-195)
    kp = torch.cat([ocd.pack_active_blocks(k.cuda(), i, n, nb) for k, (i, n) in zip(ks, comp)])
    vp = torch.cat([ocd.pack_active_blocks(v.cuda(), i, n, nb) for v, (i, n) in zip(vs, comp)])
    order, total, _ = ocd.global_block_index(torch.tensor(counts, dtype=torch.int32), nb)
    out = ocd._attend_gathered(q.cuda(), kp, vp, order, total, BS)
    np.testing.assert_allclose(host(out), ref, rtol=ATT_RTOL, atol=ATT_ATOL)
    # stratified buckets (phase_e_stratified.py:164-273)
    bucket = ocd.stratified_bucket(max(counts), nb)
    assert bucket >= max(counts)
    kp = torch.cat([ocd.pack_active_blocks(k.cuda(), i, n, bucket) for k, (i, n) in zip(ks, comp)])
    vp = torch.cat([ocd.pack_active_blocks(v.cuda(), i, n, bucket) for v, (i, n) in zip(vs, comp)])
    order, total, _ = ocd.global_block_index(torch.tensor(counts, dtype=torch.int32), bucket)
    out = ocd._attend_gathered(q.cuda(), kp, vp, order, total, BS)
    np.testing.assert_allclose(host(out), ref, rtol=ATT_RTOL, atol=ATT_ATOL)


@pytest.mark.parametrize("P,nb,hkv,hq,d", [(3, 8, 2, 4, 128), (8, 4, 2, 8, 128)])
def test_lse_merge_of_shard_partials(P, nb, hkv, hq, d):
    from orthocache_b200 import distributed as ocd, _core
    q, ks, vs, ms = _shards(P, nb, hkv, hq, d, seed=P * 10 + nb + 2)
    ref = _oracle_union_attention(q, ks, vs, ms)
    parts = []
    for k, v, m in zip(ks, vs, ms):
        q4, k4, v4, _ = _core.batched_qkv(q, k, v)
        idx, n = ocd.stream_compact(dev(m))
        parts.append(_core.partial_attend(q4, k4, v4, idx.reshape(1, -1), n, BS, max_blocks=nb))
    gm = torch.stack([p[0] for p in parts])
    gl = torch.stack([p[1] for p in parts])
    go = torch.stack([p[2] for p in parts])
    out = _core.merge_partials(gm, gl, go, (1, hq, d), torch.bfloat16)
    np.testing.assert_allclose(host(out), ref, rtol=ATT_RTOL, atol=ATT_ATOL)


@pytest.fixture
def one_rank_group():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            device_id=torch.device("cuda", 0))
    yield
    dist.destroy_process_group()


def test_public_entry_points_on_one_rank(one_rank_group):
    from orthocache_b200 import distributed as ocd
    nb = 8
    q, ks, vs, ms = _shards(2, nb, 2, 8, 128, seed=77)
    k, v, m = ks[1].cuda(), vs[1].cuda(), ms[1]
    ref = _oracle_union_attention(q, [ks[1]], [vs[1]], [m])
    out = ocd.distributed_orthocache_attention(q.cuda(), k, v, dev(m))
    np.testing.assert_allclose(host(out), ref, rtol=ATT_RTOL, atol=ATT_ATOL)
    out = ocd.sequence_parallel_attention(q.cuda(), k, v, dev(m))
    np.testing.assert_allclose(host(out), ref, rtol=ATT_RTOL, atol=ATT_ATOL)
    idx, n = ocd.stream_compact(dev(m))
    out, bucket = ocd.stratified_allgather_attention(q.cuda(), k, v, idx, n)
    assert bucket == O.stratified_bucket(int(m.sum()), O.stratified_buckets(nb))
    np.testing.assert_allclose(host(out), ref, rtol=ATT_RTOL, atol=ATT_ATOL)
    ka, va, counts, offs, stats = ocd.alltoallv_kv_exchange(k, v, dev(m))
    n = int(m.sum())
    rp, _ = O.stream_compact_mask(m)
    want = O.pack_active_blocks(_f32(ks[1]), rp, n, nb)
    assert np.array_equal(_f32(ka.cpu()), want)
    assert counts.tolist() == [n] and offs.tolist() == [0]
    assert int(stats["total_active"]) == n and stats["dense_blocks"] == nb
    assert int(stats["bytes_saved"]) == (nb - n) * BS * 2 * 128 * 2 * 2
