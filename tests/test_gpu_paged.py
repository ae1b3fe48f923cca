"""Paged KV cache (block table + page pool, write-time metadata) against the
oracle run on the same sequences laid out contiguously: the keep mask of the
logical blocks (bit-exact away from the thresholds), the compaction, and the
attention (1e-2 relative / 2e-2 absolute in bf16), for decode (split-KV
kernel) and for a chunked-prefill step (tensor-core kernel).  Batch rows of
different lengths share one table width; the padding entries point at no
page and are never kept."""
import numpy as np
import pytest
import torch

from oracle import oc_oracle as O
from gpu_util import ATT_RTOL, ATT_ATOL, assert_mask_parity

pytestmark = pytest.mark.gpu


def _setup(seed, lengths, hkv, num_pages):
    from orthocache_b200 import synthetic as syn, PagedKVCache
    rs = np.random.RandomState(seed)
    cache = PagedKVCache(num_pages, hkv, 128)
    width = max(lengths)
    table = np.full((len(lengths), width), -1, np.int32)
    free = list(rs.permutation(num_pages))
    seqs = []
    for b, nb in enumerate(lengths):
        kinds = syn.block_kinds(nb, 0.5, seed=seed + b)
        k = syn.make_keys(nb, hkv, 128, kinds, seed=seed + b)
        v = syn.make_values(nb * 512, hkv, 128, seed=seed + b)
        pages = [free.pop() for _ in range(nb)]
        table[b, :nb] = pages
        cache.write(pages, k, v)
        seqs.append((k, v))
    return cache, table, seqs


@pytest.mark.parametrize("sq,hq", [(1, 32), (128, 16)])
def test_paged_cache_vs_contiguous_oracle(sq, hq):
    from orthocache_b200 import synthetic as syn
    hkv, lengths = 8, [16, 11]
    cache, table, seqs = _setup(11 + sq, lengths, hkv, 48)
    B, width = len(lengths), table.shape[1]
    q = torch.stack([syn.make_queries(sq, hq, 128, seed=70 + b) for b in range(B)])
    # one tau for the batch, placed between block scores of both rows
    refs = [O.score_blocks(q[b].float().cpu().numpy(), seqs[b][0].float().cpu().numpy(), -1e30, 5.0)
            for b in range(B)]
    zeta = torch.tensor(np.concatenate([r["zeta"] for r in refs]))
    bmax = torch.tensor(np.concatenate([r["bound_max"] for r in refs]))
    tau, _ = syn.calibrate_tau(zeta, bmax, 5.0, 0.6)
    out, keep, perm, count = cache.attend(q, torch.tensor(table), width, tau, 5.0)
    torch.cuda.synchronize()
    keep = keep.cpu().numpy().astype(bool)
    for b, nb in enumerate(lengths):
        ref = O.score_blocks(q[b].float().cpu().numpy(), seqs[b][0].float().cpu().numpy(), tau, 5.0)
        assert_mask_parity(keep[b, :nb], ref["keep"], ref["zeta"], ref["bound_max"], tau, 5.0)
        assert not keep[b, nb:].any(), "padding entries of the block table must never be kept"
        rp, rn = O.stream_compact_mask(keep[b, :nb])
        assert int(count[b]) == rn
        assert np.array_equal(perm[b, :rn].cpu().numpy(), rp[:rn])
        want = O.indirect_attention(q[b].float().cpu().numpy(), seqs[b][0].float().cpu().numpy(),
                                    seqs[b][1].float().cpu().numpy(), rp, rn)
        np.testing.assert_allclose(out[b].float().cpu().numpy(), want, rtol=ATT_RTOL, atol=ATT_ATOL)


def test_paged_rewrite_updates_metadata():
    """Rewriting a page refreshes its metadata: the gates follow the new keys."""
    from orthocache_b200 import synthetic as syn
    cache, table, seqs = _setup(5, [6], 4, 10)
    page = int(table[0, 2])
    noise = syn.make_keys(1, 4, 128, np.array([1]), seed=99)     # iid noise block: low zeta
    smooth = syn.make_keys(1, 4, 128, np.array([0]), seed=99)    # smooth block: high zeta
    cache.write([page], smooth, syn.make_values(512, 4, 128, seed=1))
    z_smooth = cache.zeta[page].clone()
    cache.write([page], noise, syn.make_values(512, 4, 128, seed=1))
    ref = O.block_metadata(noise.float().cpu().numpy())[2]
    np.testing.assert_allclose(cache.zeta[page].cpu().numpy(), ref[0], rtol=2e-5)
    assert float(z_smooth.min()) > float(cache.zeta[page].max())
