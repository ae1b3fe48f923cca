"""A reduced decode stack of the configuration-4 structure (sliding-window
layers interleaved with global eviction layers; head_dim 256, GQA 2, batch 2)
on one GPU, every layer's output against the oracle: sliding layers attend
densely to the last 1024 tokens, global layers to the union of the blocks
that pass the two gates (bit-exact masks away from the thresholds, attention
1e-2 relative / 2e-2 absolute in bf16)."""
import numpy as np
import pytest
import torch

from oracle import oc_oracle as O
from gpu_util import ATT_RTOL, ATT_ATOL

pytestmark = pytest.mark.gpu


def test_reduced_stack_vs_oracle():
    from orthocache_b200 import synthetic as syn
    from orthocache_b200.stack import DecodeStack
    kinds = ["sliding", "sliding", "global", "sliding", "global"]
    B, Hq, Hkv, D, nb = 2, 8, 4, 256, 8
    S = nb * 512
    rs = np.random.RandomState(3)
    qs, ks, vs, taus = [], [], [], []
    for li, kind in enumerate(kinds):
        fs, fm = rs.uniform(0.2, 0.4), rs.uniform(0.2, 0.4)  # band mixture re-drawn per layer
        k = torch.stack([syn.make_keys(nb, Hkv, D, syn.block_kinds(nb, fs, fm, seed=10 * li + b), seed=10 * li + b)
                         for b in range(B)])
        v = torch.stack([syn.make_values(S, Hkv, D, seed=10 * li + b) for b in range(B)])
        q = torch.stack([syn.make_queries(1, Hq, D, seed=100 + 10 * li + b) for b in range(B)])
        tau = 0.0
        if kind == "global":
            refs = [O.score_blocks(q[b].float().cpu().numpy(), k[b].float().cpu().numpy(), -1e30, 5.0)
                    for b in range(B)]
            tau, _ = syn.calibrate_tau(torch.tensor(np.concatenate([r["zeta"] for r in refs])),
                                       torch.tensor(np.concatenate([r["bound_max"] for r in refs])), 5.0, 0.75)
        qs.append(q); ks.append(k); vs.append(v); taus.append(tau)
    st = DecodeStack(kinds, B, Hq, Hkv, D, S, window=1024)
    outs = [torch.empty((B, 1, Hq, D), dtype=torch.bfloat16, device="cuda") for _ in kinds]
    for _ in range(2):  # buffers are reused from step to step
        st.step(qs, ks, vs, taus, outs)
    torch.cuda.synchronize()
    for li, kind in enumerate(kinds):
        for b in range(B):
            qf, kf, vf = (t[b].float().cpu().numpy() for t in (qs[li], ks[li], vs[li]))
            if kind == "sliding":
                perm, n = np.array([nb - 2, nb - 1]), 2
            else:
                keep = O.score_blocks(qf, kf, taus[li], 5.0)["keep"]
                perm, n = O.stream_compact_mask(keep)
            want = O.indirect_attention(qf, kf, vf, perm, n)
            np.testing.assert_allclose(outs[li][b].float().cpu().numpy(), want, rtol=ATT_RTOL, atol=ATT_ATOL,
                                       err_msg=f"layer {li} ({kind}) batch row {b}")
