"""Stream compaction, gather/scatter and exchange-index kernels: bit-exact
against the CPU oracle, including the edge cases of the reference's tests."""
import numpy as np
import pytest
import torch

from oracle import oc_oracle as O
from gpu_util import dev, host

pytestmark = pytest.mark.gpu


def compact(mask):
    from orthocache_b200 import _core
    perm, count = _core.compact(dev(mask))
    return host(perm[0]), int(count[0])


@pytest.mark.parametrize("mask", [
    [False, True, False, True, True, False],
    [True, False, True, True, False],
    [False] * 8, [True] * 8, [True], [False],
])
def test_known_answers(mask):
    m = np.array(mask)
    perm, n = compact(m)
    rp, rn = O.stream_compact_mask(m)
    assert n == rn and np.array_equal(perm, rp)


@pytest.mark.parametrize("nb,h,p", [(5, 1, 0.5), (128, 8, 0.1), (1023, 4, 0.5), (1024, 2, 0.3),
                                    (1025, 1, 0.7), (5000, 3, 0.2), (3000, 8, 0.97)])
def test_random_masks(nb, h, p):
    rs = np.random.RandomState(nb + h)
    m = rs.rand(nb, h) < p / h
    perm, n = compact(m)
    rp, rn = O.stream_compact_mask(m)
    assert n == rn and np.array_equal(perm, rp)


def test_batched_compaction():
    from orthocache_b200 import _core
    rs = np.random.RandomState(3)
    m = rs.rand(4, 300, 2) < 0.3
    perm, count = _core.compact(dev(m), batched=True)
    for b in range(4):
        rp, rn = O.stream_compact_mask(m[b])
        assert int(count[b]) == rn and np.array_equal(host(perm[b]), rp)


def test_stream_compact_dropin_and_decompact_roundtrip():
    import orthocache_b200 as oc
    rs = np.random.RandomState(4)
    k = rs.randn(8 * 512, 4, 64).astype(np.float32)
    v = rs.randn(8 * 512, 4, 64).astype(np.float32)
    mask = np.broadcast_to((np.arange(8) % 2 == 0)[:, None], (8, 4))
    ck, cv, idx, n = oc.stream_compact(dev(k), dev(v), dev(mask), 512)
    rk, rv, ridx, rn = O.stream_compact(k, v, mask)
    assert int(n) == rn == 4
    assert np.array_equal(host(idx), ridx)
    assert np.array_equal(host(ck), rk) and np.array_equal(host(cv), rv)
    back = host(oc.stream_decompact(ck, idx, n, 8))
    assert np.array_equal(back, O.stream_decompact(rk, ridx, rn, 8))
    # 100 % eviction: all-zero compact tensors (test_compaction.py:128-137)
    ck, _, _, n = oc.stream_compact(dev(k), dev(v), dev(np.zeros((8, 4), bool)), 512)
    assert int(n) == 0 and float(ck.abs().sum()) == 0.0
    # bf16 and a single block
    kb = torch.randn(512, 2, 64, device="cuda").bfloat16()
    ck, cv, idx, n = oc.stream_compact(kb, kb, torch.ones(1, 2, dtype=torch.bool, device="cuda"), 512)
    assert int(n) == 1 and torch.equal(ck[0], kb.reshape(512, 2, 64))


def test_mask_only_form():
    import orthocache_b200 as oc
    idx, n = oc.stream_compact(dev(np.array([True, False, True, False])))
    assert int(n) == 2 and list(host(idx)[:2]) == [0, 2]


def test_pack_active_blocks_matches_oracle():
    from orthocache_b200 import _core
    rs = np.random.RandomState(5)
    kv = rs.randn(6 * 512, 2, 64).astype(np.float32)
    m = np.array([1, 0, 0, 1, 1, 0], bool)
    perm, count = _core.compact(dev(m))
    packed = _core.gather_blocks(dev(kv).unsqueeze(0), perm, count, 6, 512)[0]
    rp, rn = O.stream_compact_mask(m)
    assert np.array_equal(host(packed), O.pack_active_blocks(kv, rp, rn, 6))


@pytest.mark.parametrize("counts,slots", [([2, 0, 3], 4), ([4, 4, 4, 4], 4), ([0, 0], 3), ([1, 3, 2], 4),
                                          ([300, 17, 1000, 0, 5, 999, 1000, 2], 1000)])
def test_exchange_index(counts, slots):
    from orthocache_b200 import _lib
    c = torch.tensor(counts, dtype=torch.int32, device="cuda")
    order = torch.empty(len(counts) * slots, dtype=torch.int32, device="cuda")
    total = torch.empty(1, dtype=torch.int32, device="cuda")
    off = torch.empty(len(counts), dtype=torch.int32, device="cuda")
    _lib.call("oc_exchange_index", _lib.ptr(c), len(counts), slots, _lib.ptr(order), _lib.ptr(total),
              _lib.ptr(off), _lib.stream_ptr())
    ro, rt = O.global_block_index(counts, slots)
    roff, _ = O.compute_offsets(counts)
    assert int(total) == rt and np.array_equal(host(order), ro) and np.array_equal(host(off), roff)


def test_bucket_count():
    from orthocache_b200 import _lib
    c = torch.tensor([0, 1, 3, 5, 9, 17, 100, 512, 513, 700], dtype=torch.int32, device="cuda")
    out = torch.empty_like(c)
    _lib.call("oc_bucket_count", _lib.ptr(c), 10, 600, _lib.ptr(out), _lib.stream_ptr())
    want = [0 if n == 0 else min(O.next_bucket(n), 600) for n in c.tolist()]
    assert out.tolist() == want
