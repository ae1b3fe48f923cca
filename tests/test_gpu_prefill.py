"""Chunked-prefill indirect attention (oc_prefill_attention: tcgen05 tensor
cores, accumulators in tensor memory) against the CPU oracle's attention
(the reference's indirect_attention / _multihead_loop numerics), through the
C ABI.  Tolerance: the parity contract's 1e-2 relative / 2e-2 absolute for
bf16 attention output.

At the full configuration-2 size (batch 4, 2048-query chunks, 32/8 heads,
32,768 tokens, 75 % eviction) the float64 oracle is evaluated on a seeded
sample of query rows (attention rows are independent), and every row is
checked against a float32 torch evaluation of the same softmax on the GPU.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oc_oracle as O
from gpu_util import ATT_RTOL, ATT_ATOL

pytestmark = pytest.mark.gpu


def _lib():
    from orthocache_b200 import _lib as L
    return L.load()


def _run(q, k, v, idx, cnt, bs, idx_stride, idx_hstride=0, cnt_stride=1, cnt_hstride=0, out_dtype=torch.bfloat16,
         max_blocks=None):
    lib = _lib()
    B, Sq, Hq, D = q.shape
    S, Hkv = k.shape[1], k.shape[2]
    out = torch.full((B, Sq, Hq, D), float("nan"), dtype=out_dtype, device="cuda")
    mb = S // bs if max_blocks is None else max_blocks
    rc = lib.oc_prefill_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, idx.data_ptr(), idx_stride,
                                  idx_hstride, cnt.data_ptr(), cnt_stride, cnt_hstride, B, Sq, Hq, Hkv, D, S, bs, mb,
                                  out.data_ptr(), 1 if out_dtype == torch.bfloat16 else 0,
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.oc_last_error()
    torch.cuda.synchronize()
    assert lib.oc_device_status(1) == 0, "a bounded wait in the prefill kernel gave up"
    return out


def _inputs(seed, B, Sq, Hq, Hkv, S):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = (torch.randn((B, Sq, Hq, 128), generator=g, device="cuda") * 128 ** -0.25).bfloat16()
    k = torch.randn((B, S, Hkv, 128), generator=g, device="cuda").bfloat16()
    v = torch.randn((B, S, Hkv, 128), generator=g, device="cuda").bfloat16()
    return q, k, v


def _perm(rs, nb, keep_p):
    m = rs.rand(nb) < keep_p
    m[rs.randint(nb)] = True
    return O.stream_compact_mask(m)


def _oracle(q, k, v, perm, n, bs, rows=None):
    qf = q.float().cpu().numpy()
    if rows is not None:
        qf = qf[rows]
    return O.indirect_attention(qf, k.float().cpu().numpy(), v.float().cpu().numpy(), perm, n, bs)


CASES = [  # (B, Sq, Hq, Hkv, nb, bs, keep_p)
    (1, 128, 2, 1, 2, 512, 1.0),      # one unit, two row tiles of one KV head
    (1, 128, 1, 1, 3, 512, 0.7),      # a single row tile (the unit's second tile is empty)
    (2, 200, 8, 2, 5, 512, 0.5),      # partial last row tile, GQA 4
    (1, 256, 4, 4, 4, 128, 0.6),      # 128-token blocks (one K/V tile per block)
    (3, 96, 6, 2, 6, 256, 0.5),       # odd row-tile count per KV head, 256-token blocks
    (2, 512, 32, 8, 16, 512, 0.25),   # reduced configuration 2
]


@pytest.mark.parametrize("case", CASES)
def test_prefill_vs_oracle(case):
    B, Sq, Hq, Hkv, nb, bs, p = case
    rs = np.random.RandomState(B * 1000 + Sq + nb)
    q, k, v = _inputs(7 + Sq, B, Sq, Hq, Hkv, nb * bs)
    perms, counts = zip(*[_perm(rs, nb, p) for _ in range(B)])
    idx = torch.tensor(np.stack(perms), dtype=torch.int32, device="cuda")
    cnt = torch.tensor(counts, dtype=torch.int32, device="cuda")
    out = _run(q, k, v, idx, cnt, bs, nb).float().cpu().numpy()
    for b in range(B):
        ref = _oracle(q[b], k[b], v[b], perms[b], counts[b], bs)
        np.testing.assert_allclose(out[b], ref, rtol=ATT_RTOL, atol=ATT_ATOL)


def test_prefill_float32_output_and_zero_count():
    B, Sq, Hq, Hkv, nb, bs = 2, 160, 4, 2, 4, 512
    q, k, v = _inputs(3, B, Sq, Hq, Hkv, nb * bs)
    idx = torch.tensor([[2, 0, 1, 3], [0, 1, 2, 3]], dtype=torch.int32, device="cuda")
    cnt = torch.tensor([2, 0], dtype=torch.int32, device="cuda")  # batch row 1 retains nothing
    out = _run(q, k, v, idx, cnt, bs, nb, out_dtype=torch.float32).cpu().numpy()
    ref = _oracle(q[0], k[0], v[0], [2, 0, 1, 3], 2, bs)
    np.testing.assert_allclose(out[0], ref, rtol=ATT_RTOL, atol=ATT_ATOL)
    assert np.all(out[1] == 0.0)  # indirect_attention.py:150-151


def test_prefill_per_head_lists():
    """Per-KV-head index lists (the sparse-mode semantics of
    sparse_attention.py:46-49): idx (B, Hkv, nb), count (B, Hkv)."""
    B, Sq, Hq, Hkv, nb, bs = 1, 128, 4, 2, 6, 512
    rs = np.random.RandomState(5)
    q, k, v = _inputs(11, B, Sq, Hq, Hkv, nb * bs)
    lists = [_perm(rs, nb, 0.5) for _ in range(Hkv)]
    idx = torch.tensor(np.stack([p for p, _ in lists])[None], dtype=torch.int32, device="cuda")
    cnt = torch.tensor([[n for _, n in lists]], dtype=torch.int32, device="cuda")
    out = _run(q, k, v, idx, cnt, bs, Hkv * nb, idx_hstride=nb, cnt_stride=Hkv, cnt_hstride=1)
    out = out.float().cpu().numpy()[0]
    G = Hq // Hkv
    for h in range(Hkv):
        perm, n = lists[h]
        ref = O.indirect_attention(q[0, :, h * G:(h + 1) * G].float().cpu().numpy(),
                                   k[0, :, h:h + 1].float().cpu().numpy(), v[0, :, h:h + 1].float().cpu().numpy(),
                                   perm, n, bs)
        np.testing.assert_allclose(out[:, h * G:(h + 1) * G], ref, rtol=ATT_RTOL, atol=ATT_ATOL)


def test_prefill_max_blocks_clips_count():
    B, Sq, Hq, Hkv, nb, bs = 1, 128, 2, 2, 4, 512
    q, k, v = _inputs(13, B, Sq, Hq, Hkv, nb * bs)
    idx = torch.tensor([[3, 1, 0, 2]], dtype=torch.int32, device="cuda")
    cnt = torch.tensor([4], dtype=torch.int32, device="cuda")
    out = _run(q, k, v, idx, cnt, bs, nb, max_blocks=2).float().cpu().numpy()
    ref = _oracle(q[0], k[0], v[0], [3, 1, 0, 2], 2, bs)
    np.testing.assert_allclose(out[0], ref, rtol=ATT_RTOL, atol=ATT_ATOL)


def test_prefill_large_logits_rescale():
    """Logits that grow from one K/V tile to the next force the lazy rescale
    of the accumulator in tensor memory (row max up by more than 2^8)."""
    B, Sq, Hq, Hkv, nb, bs = 1, 128, 2, 1, 4, 512
    q, k, v = _inputs(17, B, Sq, Hq, Hkv, nb * bs)
    q = (q.float() * 4).bfloat16()
    k = k.float()
    for j in range(nb):  # later blocks have larger keys
        k[:, j * bs:(j + 1) * bs] *= 1 + j
    k = k.bfloat16()
    idx = torch.tensor([[0, 1, 2, 3]], dtype=torch.int32, device="cuda")
    cnt = torch.tensor([4], dtype=torch.int32, device="cuda")
    out = _run(q, k, v, idx, cnt, bs, nb).float().cpu().numpy()
    ref = _oracle(q[0], k[0], v[0], [0, 1, 2, 3], 4, bs)
    np.testing.assert_allclose(out[0], ref, rtol=ATT_RTOL, atol=ATT_ATOL)


def test_prefill_wide_logit_range():
    """Logits spread over hundreds of log2 units below the row max: the
    exponentials computed on the FMA pipe must flush to zero there, never
    wrap the exponent field into a NaN or a large value."""
    B, Sq, Hq, Hkv, nb, bs = 1, 256, 2, 1, 4, 512
    q, k, v = _inputs(23, B, Sq, Hq, Hkv, nb * bs)
    q = (q.float() * 64).bfloat16()
    k = (k.float() * 8).bfloat16()
    idx = torch.tensor([[2, 0, 3, 1]], dtype=torch.int32, device="cuda")
    cnt = torch.tensor([4], dtype=torch.int32, device="cuda")
    out = _run(q, k, v, idx, cnt, bs, nb).float().cpu().numpy()
    assert np.isfinite(out).all()
    ref = _oracle(q[0], k[0], v[0], [2, 0, 3, 1], 4, bs)
    np.testing.assert_allclose(out[0], ref, rtol=ATT_RTOL, atol=ATT_ATOL)


def test_prefill_config2_full_size():
    """Configuration 2 end to end at full size: keys of the 30/40/30 smooth /
    mid-band / noise mixture, the fused scorer's two-gate mask per batch row
    at 75 % eviction, compaction, then the tensor-core attention."""
    import orthocache_b200 as oc
    from orthocache_b200 import synthetic as syn, _core
    B, Sq, Hq, Hkv, S, bs = 4, 2048, 32, 8, 32768, 512
    nb = S // bs
    ks, vs, qs = [], [], []
    for b in range(B):
        kinds = syn.block_kinds(nb, 0.3, 0.4, seed=100 + b)
        ks.append(syn.make_keys(nb, Hkv, 128, kinds, seed=100 + b))
        vs.append(syn.make_values(S, Hkv, 128, seed=200 + b))
        qs.append(syn.make_queries(Sq, Hq, 128, seed=300 + b))
    k, v, q = torch.stack(ks), torch.stack(vs), torch.stack(qs)
    idx = torch.empty((B, nb), dtype=torch.int32, device="cuda")
    cnt = torch.empty((B,), dtype=torch.int32, device="cuda")
    for b in range(B):
        sc = oc.score_blocks(k[b], q[b], tau=-1e30, zeta_max=5.0, want=("zeta", "bound_max"))
        tau, kept = syn.calibrate_tau(sc["zeta"], sc["bound_max"], 5.0, 0.75)
        keep = oc.score_blocks(k[b], q[b], tau=tau, zeta_max=5.0, want=("keep",))["keep"]
        p, n = _core.compact(keep)
        idx[b], cnt[b] = p[0], n[0]
        assert kept == nb // 4
    assert [int(c) for c in cnt.cpu()] == [nb // 4] * B
    out = _run(q, k, v, idx, cnt, bs, nb)
    assert torch.isfinite(out.float()).all()
    rs = np.random.RandomState(0)
    for b in range(B):
        perm = idx[b].cpu().numpy()
        n = int(cnt[b])
        # float32 torch softmax over the retained tokens, every row
        tok = (torch.tensor(perm[:n], device="cuda")[:, None] * bs + torch.arange(bs, device="cuda")).reshape(-1)
        kk, vv = k[b, tok].float(), v[b, tok].float()
        for h in range(Hkv):
            qh = q[b, :, h * 4:(h + 1) * 4].float().reshape(-1, 128)
            w = torch.softmax(qh @ kk[:, h].T / 128 ** 0.5, dim=-1)
            ref = (w @ vv[:, h]).reshape(Sq, 4, 128)
            got = out[b, :, h * 4:(h + 1) * 4].float()
            assert torch.allclose(got, ref, rtol=ATT_RTOL, atol=ATT_ATOL), float((got - ref).abs().max())
        # the float64 oracle on a seeded sample of rows
        rows = np.sort(rs.choice(Sq, 48, replace=False))
        ref = _oracle(q[b], k[b], v[b], perm, n, bs, rows=rows)
        np.testing.assert_allclose(out[b].float().cpu().numpy()[rows], ref, rtol=ATT_RTOL, atol=ATT_ATOL)


def test_prefill_rejects_bad_arguments():
    lib = _lib()
    t = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    p = t.data_ptr()
    assert lib.oc_prefill_attention(p, p, p, 0, p, 1, 0, p, 1, 0, 1, 128, 1, 1, 128, 512, 512, 1, p, 1, None) == -5
    assert lib.oc_prefill_attention(p, p, p, 1, p, 1, 0, p, 1, 0, 1, 128, 1, 1, 64, 512, 512, 1, p, 1, None) == -2
    assert lib.oc_prefill_attention(p, p, p, 1, p, 1, 0, p, 1, 0, 1, 128, 1, 1, 128, 512, 192, 1, p, 1, None) == -2
    assert lib.oc_prefill_attention(p + 2, p, p, 1, p, 1, 0, p, 1, 0, 1, 128, 1, 1, 128, 512, 512, 1, p, 1,
                                    None) == -3
