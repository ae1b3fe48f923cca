"""Rank body of the multi-GPU NCCL parity test (one process per GPU, launched
by torchrun from tests/test_gpu_nccl.py).

Every rank builds every rank's shard from rank-seeded generators, so it can
check what it received against the oracle without further communication:
  * oc_exchange_stratified: the gathered blocks are bit-exact copies of each
    rank's first `bucket` retained blocks (oracle packing), the bucket is the
    oracle's, the valid-slot order is the oracle's;
  * oc_alltoallv_heads: this rank's KV heads of every rank's retained blocks,
    bit-exact, in rank order;
  * attention over the union of all shards' retained blocks, four ways —
    the stratified exchange + indirect attention, the head-partitioned
    AllToAllv + attention + output all-gather, and the fused sharded decode
    layer (oc_decode_step_sharded) with its partials exchanged by an NCCL
    all-gather and by NVLink peer stores inside the one kernel (also as a
    replayed CUDA graph) — each against the oracle's attention over the
    concatenated shards (1e-2 relative / 2e-2 absolute, bf16).
Writes ok<rank> into the result directory when every check passed.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

NB, BS, HQ, HKV, D = 16, 512, 32, 8, 128
RTOL, ATOL = 1e-2, 2e-2
ZETA_MAX = 5.0


def shard(rank, device):
    """Keys of the smooth / noise mixture (share of smooth blocks differs per
    rank, so the retained counts are uneven), values, the shared query."""
    import torch
    from orthocache_b200 import synthetic as syn
    kinds = syn.block_kinds(NB, 0.5 + 0.1 * (rank % 4), seed=500 + rank)
    k = syn.make_keys(NB, HKV, D, kinds, seed=500 + rank, device=device)
    v = syn.make_values(NB * BS, HKV, D, seed=500 + rank, device=device)
    return k, v


def bits(t):
    import torch
    return t.contiguous().view(torch.int16).cpu().numpy()


def main():
    import torch
    import torch.distributed as dist
    from oracle import oc_oracle as O
    import orthocache_b200 as oc
    from orthocache_b200 import distributed as ocd, synthetic as syn
    from orthocache_b200.comm import NcclComm

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    comm = NcclComm(device=dev)
    stop = comm.watchdog(0.2)
    try:
        shards = [shard(r, dev) for r in range(world)]
        q = syn.make_queries(1, HQ, D, seed=900, device=dev)
        qf = q.float().cpu().numpy()
        # per-shard two-gate masks from the scorer (tau = -inf: the zeta gate)
        keeps, perms, counts = [], [], []
        for k, _ in shards:
            kf = k.float().cpu().numpy()
            ref = O.score_blocks(qf, kf, -np.inf, ZETA_MAX)
            perm, n = O.stream_compact_mask(ref["keep"])
            keeps.append(ref["keep"])
            perms.append(perm)
            counts.append(int(n))
        assert len(set(counts)) > 1 or world == 1, counts
        k_me, v_me = shards[rank]
        keep_me = oc.score_blocks(k_me, q, tau=-float("inf"), zeta_max=ZETA_MAX, want=("keep",))["keep"]
        assert np.array_equal(keep_me.cpu().numpy(), keeps[rank])
        idx_me, n_me = ocd.stream_compact(keep_me)
        assert int(n_me) == counts[rank]

        # -- stratified exchange: bit-exact blocks ---------------------------------
        kr, vr, all_counts, order, total, bucket = ocd.stratified_exchange(comm, k_me, v_me, idx_me, n_me)
        assert all_counts.cpu().tolist() == counts
        assert bucket == O.stratified_bucket(max(counts), O.stratified_buckets(NB))
        for r in range(world):
            k_r, v_r = shards[r]
            want_k = O.pack_active_blocks(bits(k_r), perms[r], counts[r], bucket, BS)
            want_v = O.pack_active_blocks(bits(v_r), perms[r], counts[r], bucket, BS)
            sl = slice(r * bucket * BS, (r + 1) * bucket * BS)
            assert np.array_equal(bits(kr[sl]), want_k), f"stratified K chunk of rank {r}"
            assert np.array_equal(bits(vr[sl]), want_v), f"stratified V chunk of rank {r}"
        want_order, want_total = O.global_block_index(counts, bucket)
        assert int(total) == want_total == sum(counts)
        assert np.array_equal(order.cpu().numpy(), want_order)

        # -- attention over the union, the oracle's reference -----------------------
        k_all = np.concatenate([s[0].float().cpu().numpy() for s in shards], axis=0)
        v_all = np.concatenate([s[1].float().cpu().numpy() for s in shards], axis=0)
        gperm = np.concatenate([np.asarray(perms[r][:counts[r]]) + r * NB for r in range(world)])
        want_out = O.indirect_attention(qf, k_all, v_all, gperm, len(gperm))

        out_s, b2 = ocd.stratified_allgather_attention(q, k_me, v_me, idx_me, n_me)
        np.testing.assert_allclose(out_s.float().cpu().numpy(), want_out, rtol=RTOL, atol=ATOL)
        q4 = q.unsqueeze(0)
        kk, vv = kr.unsqueeze(0), vr.unsqueeze(0)
        from orthocache_b200 import _core
        out_x = _core.attend(q4, kk, vv, order.reshape(1, -1), total, BS, out_dtype=torch.bfloat16)[0]
        np.testing.assert_allclose(out_x.float().cpu().numpy(), want_out, rtol=RTOL, atol=ATOL)

        # -- AllToAllv by KV head: bit-exact ---------------------------------------
        if HKV % world == 0:
            hper = HKV // world
            kh, vh, c2, t2 = ocd.alltoallv_heads(comm, k_me, v_me, idx_me, n_me)
            assert t2 == sum(counts) and c2.cpu().tolist() == counts
            heads = slice(rank * hper, (rank + 1) * hper)
            want_k = np.concatenate([
                bits(shards[r][0][torch.as_tensor(
                    (np.asarray(perms[r][:counts[r]])[:, None] * BS + np.arange(BS)).reshape(-1), device=dev),
                    heads]) for r in range(world)], axis=0)
            want_v = np.concatenate([
                bits(shards[r][1][torch.as_tensor(
                    (np.asarray(perms[r][:counts[r]])[:, None] * BS + np.arange(BS)).reshape(-1), device=dev),
                    heads]) for r in range(world)], axis=0)
            assert np.array_equal(bits(kh), want_k), "alltoallv K"
            assert np.array_equal(bits(vh), want_v), "alltoallv V"
            out_h = ocd.head_partitioned_attention(q, k_me, v_me, keep_me, comm)
            np.testing.assert_allclose(out_h.float().cpu().numpy(), want_out, rtol=RTOL, atol=ATOL)

        # -- fused sharded decode layer: NCCL all-gather of the partials, then
        #    the one-kernel form that merges them over NVLink peer stores -------
        from orthocache_b200 import _lib
        for peer in (False, True):
            dec = ocd.ShardedDecoder(comm, HQ, HKV, D, NB * BS, peer=peer)
            if peer:
                assert dec.peer, dec.connect_error
            dist.barrier()
            for _ in range(3):  # repeated calls reuse the workspace's counter sets and exchange slots
                out_d = dec(q, k_me, v_me, -float("inf"), ZETA_MAX)
            torch.cuda.synchronize()
            np.testing.assert_allclose(out_d[0].float().cpu().numpy(), want_out, rtol=RTOL, atol=ATOL)
            assert int(dec.count[0]) == counts[rank]
            assert np.array_equal(dec.perm[0].cpu().numpy(), perms[rank])
            assert _lib.load().oc_device_status(1) == 0, f"bounded wait gave up (peer={peer})"
            if peer:
                # the one-kernel step captured in a CUDA graph and replayed
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=side):
                    dec(q, k_me, v_me, -float("inf"), ZETA_MAX)
                    dec(q, k_me, v_me, -float("inf"), ZETA_MAX)
                dist.barrier()
                for _ in range(3):
                    dec.out.zero_()
                    g.replay()
                torch.cuda.synchronize()
                np.testing.assert_allclose(dec.out[0].float().cpu().numpy(), want_out, rtol=RTOL, atol=ATOL)
                assert _lib.load().oc_device_status(1) == 0, "bounded wait gave up in the graph replay"
            dec.close()

        comm.check()
        dist.barrier()
        with open(os.path.join(sys.argv[1], f"ok{rank}"), "w") as f:
            f.write("ok\n")
    finally:
        stop()
        comm.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
