"""Indirect block attention, the drop-in wrappers around it and the one-call
decode step (through the C ABI) against the CPU oracle.  Tolerance: the
parity contract's 1e-2 relative / 2e-2 absolute for bf16; 2e-4 for fp32."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oc_oracle as O
from gpu_util import dev, host, bf16_round, ATT_RTOL, ATT_ATOL

pytestmark = pytest.mark.gpu


def rand_qkv(rs, sq, hq, hkv, d, nb, bs=512, dtype=np.float32):
    q = rs.randn(sq, hq, d).astype(np.float32) * d ** -0.25
    k = rs.randn(nb * bs, hkv, d).astype(np.float32)
    v = rs.randn(nb * bs, hkv, d).astype(np.float32)
    return q, k, v


CASES = [  # (Sq, Hq, Hkv, D, nb, bs, dtype, keep_prob)
    (1, 8, 8, 128, 16, 512, torch.bfloat16, 0.5),
    (1, 32, 8, 128, 12, 512, torch.bfloat16, 0.25),
    (4, 4, 4, 64, 8, 512, torch.float32, 0.5),
    (3, 8, 2, 64, 10, 128, torch.float32, 0.6),     # R = 12 rows -> 2 row tiles
    (1, 16, 16, 256, 4, 512, torch.bfloat16, 0.5),
    (2, 8, 2, 256, 3, 256, torch.bfloat16, 1.0),   # R = 8 at D=256 -> tiles of 4
    (1, 2, 2, 128, 5, 64, torch.float32, 0.4),      # 64-token blocks
    (3, 16, 4, 128, 6, 512, torch.bfloat16, 0.5),   # R = 12 rows -> two 8-row tensor-core tiles
    (1, 8, 8, 64, 6, 512, torch.bfloat16, 0.5),     # D = 64 on tensor cores
    (2, 4, 1, 128, 9, 128, torch.bfloat16, 0.7),    # 128-token blocks, R = 8
]


@pytest.mark.parametrize("case", CASES)
def test_indirect_attention_vs_oracle(case):
    from orthocache_b200 import _core
    sq, hq, hkv, d, nb, bs, dt, p = case
    rs = np.random.RandomState(sq * 100 + hq + nb)
    q, k, v = rand_qkv(rs, sq, hq, hkv, d, nb, bs)
    if dt == torch.bfloat16:
        q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    m = rs.rand(nb) < p
    m[rs.randint(nb)] = True
    perm, count = _core.compact(dev(m))
    qq, kk, vv, _ = _core.batched_qkv(dev(q, dt), dev(k, dt), dev(v, dt))
    out = host(_core.attend(qq, kk, vv, perm, count, bs)[0])
    rp, rn = O.stream_compact_mask(m)
    ref = O.indirect_attention(q, k, v, rp, rn, bs)
    tol = (ATT_RTOL, ATT_ATOL) if dt == torch.bfloat16 else (2e-4, 2e-4)
    np.testing.assert_allclose(out, ref, rtol=tol[0], atol=tol[1])


def test_zero_active_gives_zeros():
    import orthocache_b200 as oc
    rs = np.random.RandomState(0)
    q, k, v = rand_qkv(rs, 8, 4, 4, 64, 4)
    out, meta = oc.indirect_attention(dev(q), dev(k), dev(v), dev(np.zeros((4, 4), bool)), 512)
    assert float(out.abs().max()) == 0.0 and out.shape == (8, 4, 64)
    assert meta["num_active"] == 0 and meta["eviction_rate"] == 1.0 and meta["bucket"] == 0


def test_indirect_attention_bucket_semantics():
    """The reference attends to the first bucket(n) permutation entries
    (indirect_attention.py:153-157): n = 3 active -> 4 blocks attended."""
    import orthocache_b200 as oc
    rs = np.random.RandomState(1)
    q, k, v = rand_qkv(rs, 1, 4, 4, 64, 8)
    m = np.zeros(8, bool)
    m[[1, 4, 6]] = True
    out, meta = oc.indirect_attention(dev(q), dev(k), dev(v), dev(np.repeat(m[:, None], 4, 1)), 512)
    rp, _ = O.stream_compact_mask(m)
    ref = O.indirect_attention(q, k, v, rp, 4)
    np.testing.assert_allclose(host(out), ref, rtol=2e-4, atol=2e-4)
    assert meta["num_active"] == 3 and meta["bucket"] == 4 and meta["num_blocks"] == 8


def test_zero_eviction_matches_dense():   # test_indirect_attention.py:121-158 (TPU-only there)
    import orthocache_b200 as oc
    rs = np.random.RandomState(2)
    q, k, v = rand_qkv(rs, 4, 4, 4, 64, 4)
    out, _ = oc.indirect_attention(dev(q), dev(k), dev(v), dev(np.ones((4, 4), bool)), 512)
    np.testing.assert_allclose(host(out), O.block_sparse_attention(q, k, v, np.ones((4, 4), bool)),
                               rtol=2e-4, atol=2e-4)


def test_compact_and_attend_and_sparse():   # test_compaction.py:162-222
    import orthocache_b200 as oc
    rs = np.random.RandomState(3)
    q, k, v = rand_qkv(rs, 4, 4, 4, 64, 8)
    m = np.broadcast_to((np.arange(8) % 2 == 0)[:, None], (8, 4)).copy()
    out, meta = oc.compact_and_attend(dev(q), dev(k), dev(v), dev(m), 512)
    sp = oc.jax_block_sparse_attention(dev(q), dev(k), dev(v), dev(m), 512)
    ref = O.block_sparse_attention(q, k, v, m)
    np.testing.assert_allclose(host(out), ref, rtol=1e-3, atol=1e-3)
    np.testing.assert_allclose(host(sp), ref, rtol=1e-3, atol=1e-3)
    assert meta["num_active"] == 4 and meta["num_blocks"] == 8 and abs(meta["eviction_rate"] - 0.5) < 0.01


def test_sparse_per_head_masks():
    import orthocache_b200 as oc
    rs = np.random.RandomState(4)
    q, k, v = rand_qkv(rs, 2, 8, 4, 64, 6)
    m = rs.rand(6, 4) < 0.5
    m[0] = True  # every head keeps at least one block
    sp = oc.jax_block_sparse_attention(dev(q), dev(k), dev(v), dev(m), 512)
    np.testing.assert_allclose(host(sp), O.block_sparse_attention(q, k, v, m), rtol=2e-4, atol=2e-4)


def test_adaptive_orthocache_attention_bf16():
    import orthocache_b200 as oc
    rs = np.random.RandomState(5)
    q, k, v = (bf16_round(x) for x in rand_qkv(rs, 1, 4, 4, 128, 16))
    m = rs.rand(16) < 0.25
    m[3] = True
    out, stats = oc.orthocache_attention(dev(q, torch.bfloat16), dev(k, torch.bfloat16),
                                         dev(v, torch.bfloat16), dev(m))
    assert out.dtype == torch.bfloat16
    rp, rn = O.stream_compact_mask(m)
    np.testing.assert_allclose(host(out), O.indirect_attention(q, k, v, rp, rn), rtol=ATT_RTOL, atol=ATT_ATOL)
    assert stats["num_active"] == rn
    # batched form: one mask shared by the batch
    qb = np.stack([q, q * 0.5]); kb = np.stack([k, k[::-1].copy()]); vb = np.stack([v, v])
    ob, _ = oc.orthocache_attention_batched(dev(qb, torch.bfloat16), dev(kb, torch.bfloat16),
                                            dev(vb, torch.bfloat16), dev(m))
    for b in range(2):
        np.testing.assert_allclose(host(ob[b]), O.indirect_attention(qb[b], kb[b], vb[b], rp, rn),
                                   rtol=ATT_RTOL, atol=ATT_ATOL)


def test_compile_indirect_attention_table():
    import orthocache_b200 as oc
    rs = np.random.RandomState(6)
    q, k, v = rand_qkv(rs, 1, 2, 2, 64, 6)
    tab = np.array([[5, 1], [2, 2], [0, 4]], np.int32)  # (bucket, H): per-head lists
    out = host(oc.compile_indirect_attention(dev(q), dev(k), dev(v), dev(tab), 3, 512))
    for h in range(2):
        ref = O.indirect_attention(q[:, h:h + 1], k[:, h:h + 1], v[:, h:h + 1], tab[:, h], 3)
        np.testing.assert_allclose(out[:, h:h + 1], ref, rtol=2e-4, atol=2e-4)


def test_orthocache_forward_modes():   # test_pipeline.py / test_compaction.py:225-276
    import orthocache_b200 as oc
    rs = np.random.RandomState(7)
    q, k, v = rand_qkv(rs, 4, 4, 4, 64, 4)
    out, meta = oc.orthocache_forward(dev(q), dev(k), dev(v), mode="dense")
    np.testing.assert_allclose(host(out), O.block_sparse_attention(q, k, v, np.ones((4, 4), bool)),
                               rtol=2e-4, atol=2e-4)
    assert meta["mode"] == "dense" and meta["eviction_rate"] == 0.0
    for mode in ("sparse", "compact"):
        qd, kd, vd = dev(q), dev(k), dev(v)
        torch.cuda.synchronize()
        torch.cuda.set_sync_debug_mode("error")  # the call itself never waits for the GPU
        try:
            out, meta = oc.orthocache_forward(qd, kd, vd, zeta_max=100.0, mode=mode)
        finally:
            torch.cuda.set_sync_debug_mode(0)
        tau = O.auto_tau(q, k)
        assert abs(meta["tau"] - tau) < 1e-4 * max(1, abs(tau))
        keep = O.multiband_mask(q, k, meta["tau"], 100.0)
        ref = O.block_sparse_attention(q, k, v, keep) if mode == "sparse" else \
            O.indirect_attention(q, k, v, *O.stream_compact_mask(keep))
        np.testing.assert_allclose(host(out), ref, rtol=2e-4, atol=2e-4)
        assert "zeta_mean" in meta and "eviction_rate" in meta
    assert meta["compact_num_active"] == O.stream_compact_mask(keep)[1]
    with pytest.raises(ValueError, match="Unknown mode"):
        oc.orthocache_forward(dev(q), dev(k), dev(v), mode="invalid")


def _decode_step_cabi(q, k, v, tau, zmax):
    """Call oc_decode_step through ctypes with raw device pointers."""
    from orthocache_b200 import _lib
    lib = _lib.load()
    Sq, Hq, D = q.shape
    S, Hkv, _ = k.shape
    nb = S // 512
    keep = torch.empty((nb, Hkv), dtype=torch.uint8, device="cuda")
    perm = torch.empty((nb,), dtype=torch.int32, device="cuda")
    count = torch.empty((1,), dtype=torch.int32, device="cuda")
    out = torch.empty((Sq, Hq, D), dtype=torch.bfloat16, device="cuda")
    ws_bytes = lib.oc_decode_step_workspace_bytes(1, Sq, Hq, Hkv, D, S)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")  # zero before first use
    rc = lib.oc_decode_step(q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, 1, Sq, Hq, Hkv, D, S,
                            ctypes.c_float(tau), ctypes.c_float(zmax), keep.data_ptr(), perm.data_ptr(),
                            count.data_ptr(), out.data_ptr(), 1, ws.data_ptr(), ws_bytes,
                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.oc_last_error()
    torch.cuda.synchronize()
    return keep, perm, count, out


@pytest.mark.parametrize("nb,hq,hkv,evict,d,sq", [
    (16, 8, 8, 0.5, 128, 1),     # config 0 (8/8 heads, 8K tokens)
    (128, 32, 8, 0.75, 128, 1),  # config 1 (32/8, 64K tokens) at full size
    (128, 32, 8, 0.9, 128, 1),
    (24, 16, 4, 0.5, 64, 1),     # head_dim 64
    (20, 16, 4, 0.6, 128, 2),    # two query rows x GQA 4: 8-row tiles
    (12, 8, 8, 1.0, 128, 1),     # every block evicted: zeros
    (1100, 2, 1, 0.5, 64, 1),    # more blocks than the in-kernel list holds: separate compaction
])
def test_decode_step_cabi_vs_oracle(nb, hq, hkv, evict, d, sq):
    """The one-call decode step (scorer, compaction fused into the attention
    prologue, attention, merge) against the oracle's mask, stable permutation,
    count and attention."""
    from orthocache_b200 import synthetic as syn
    from gpu_util import assert_mask_parity
    kinds = syn.block_kinds(nb, min(evict, 0.99), seed=nb)
    k = syn.make_keys(nb, hkv, d, kinds, seed=nb)
    v = syn.make_values(nb * 512, hkv, d, seed=nb)
    q = syn.make_queries(sq, hq, d, seed=nb)
    kf, qf, vf = host(k), host(q), host(v)
    r0 = O.score_blocks(qf, kf, -1e30, 5.0)
    tau, _ = syn.calibrate_tau(torch.tensor(r0["zeta"]), torch.tensor(r0["bound_max"]), 5.0, evict)
    keep, perm, count, out = _decode_step_cabi(q, k, v, tau, 5.0)
    ref_keep = (r0["bound_max"] >= np.float32(tau)) & (r0["zeta"] <= np.float32(5.0))
    assert_mask_parity(host(keep).astype(bool), ref_keep, r0["zeta"], r0["bound_max"], tau, 5.0)
    rp, rn = O.stream_compact_mask(host(keep).astype(bool))
    assert int(count) == rn == round((1 - evict) * nb)
    assert np.array_equal(host(perm), rp)
    ref = O.indirect_attention(qf, kf, vf, rp, rn)
    np.testing.assert_allclose(host(out), ref, rtol=ATT_RTOL, atol=ATT_ATOL)


def test_sparse_head_with_no_kept_block_is_uniform():
    """sparse_attention.py:49-57: a head whose blocks are all masked gets the
    uniform softmax over all tokens, i.e. the mean of its value rows."""
    import orthocache_b200 as oc
    rs = np.random.RandomState(8)
    q, k, v = rand_qkv(rs, 2, 4, 2, 64, 4)
    m = np.array([[1, 0], [0, 0], [1, 0], [0, 0]], bool)  # head 1 keeps nothing
    sp = oc.jax_block_sparse_attention(dev(q), dev(k), dev(v), dev(m), 512)
    np.testing.assert_allclose(host(sp), O.block_sparse_attention(q, k, v, m), rtol=2e-4, atol=2e-4)
