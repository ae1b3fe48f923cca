"""Rank bodies of the world-size-2 gloo tests (run in spawned processes).

Each rank builds its shard's data from a rank-seeded generator, so every
rank can rebuild every other rank's inputs and check the collective results
against the oracle without further communication.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

NB, BS, H, D = 6, 8, 2, 4  # tiny blocks: the exchange logic does not depend on the block size


def shard(rank):
    rs = np.random.RandomState(100 + rank)
    kv = rs.randn(NB * BS, H, D).astype(np.float32)
    mask = rs.rand(NB) < 0.5
    mask[rank % NB] = True  # at least one active block per rank
    return kv, mask


def run(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist
    from oracle import oc_oracle as O
    from orthocache_b200 import distributed as ocd

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shards = [shard(r) for r in range(world)]
        counts = [int(m.sum()) for _, m in shards]

        # a15: count sync + offsets
        all_counts = ocd.count_sync(torch.tensor(counts[rank], dtype=torch.int32))
        assert all_counts.tolist() == counts, (all_counts, counts)
        off, total = ocd.compute_offsets(all_counts)
        ref_off, ref_total = O.compute_offsets(counts)
        assert off.tolist() == ref_off.tolist() and int(total) == ref_total

        # a16: exchange of packed buffers (packed here by the oracle; the
        # packing kernel itself is covered by the GPU tests)
        packed = []
        for kv, m in shards:
            perm, n = O.stream_compact_mask(m)
            packed.append(O.pack_active_blocks(kv, perm, n, NB, BS))
        mine = torch.from_numpy(packed[rank])
        kr, vr = ocd.alltoallv_exchange(mine, mine * 2)
        want = np.concatenate(packed, axis=0)
        assert np.array_equal(kr.numpy(), want)
        assert np.array_equal(vr.numpy(), want * 2)
        act, dev_off = O.unpack_received(want, counts, world, NB, BS)
        assert dev_off.tolist() == (np.asarray(ref_off) * BS).tolist()
        assert np.array_equal(act[: ref_total * BS], np.concatenate(
            [packed[r][: counts[r] * BS] for r in range(world)], axis=0))

        # a18: stratified consensus -- every rank picks the same bucket
        gmax = torch.tensor([counts[rank]], dtype=torch.int32)
        dist.all_reduce(gmax, op=dist.ReduceOp.MAX)
        assert int(gmax) == max(counts)
        assert ocd.stratified_buckets(NB) == O.stratified_buckets(NB)
        b = ocd.stratified_bucket(int(gmax), NB)
        assert b == O.stratified_bucket(int(gmax), O.stratified_buckets(NB))
        picked = torch.tensor([b], dtype=torch.int32)
        lst = [torch.zeros(1, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(lst, picked)
        assert len({int(t) for t in lst}) == 1

        # (m, l, o) partials travel as float32 rows; the exchange keeps rank order
        part = torch.full((3, 5), float(rank))
        g = ocd._all_gather_cat(part)
        assert g.shape == (3 * world, 5) and all(float(g[3 * r, 0]) == r for r in range(world))

        open(os.path.join(result_dir, f"ok{rank}"), "w").write("ok")
    finally:
        dist.destroy_process_group()
