"""Failure detection on the GPU without a GPU fault: a bounded wait that runs
out.  The fused decode layer's attention producers poll the block-decision
queue; a workspace whose block 0 can never be decided (its head counter is
pre-set so that the last head never brings it to the decision) leaves a
queue slot unpublished, the poll gives up after the wait limit, the
kernel records the status and returns, and the context stays usable: a call
on a re-zeroed workspace is correct again."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oc_oracle as O

pytestmark = pytest.mark.gpu


def _call(lib, q, k, v, tau, ws, outs):
    keep, perm, count, out = outs
    hq, d = q.shape[1], q.shape[2]
    s, hkv = k.shape[0], k.shape[1]
    return lib.oc_decode_step(q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, 1, 1, hq, hkv, d, s,
                              ctypes.c_float(tau), ctypes.c_float(5.0), keep.data_ptr(), perm.data_ptr(),
                              count.data_ptr(), out.data_ptr(), 1, ws.data_ptr(), ws.numel(),
                              torch.cuda.current_stream().cuda_stream)


def test_expired_wait_is_reported_and_the_next_call_is_correct():
    from orthocache_b200 import _lib, synthetic as syn
    lib = _lib.load()
    nb, hkv, hq, d = 16, 8, 32, 128
    kinds = syn.block_kinds(nb, 0.5, seed=3)
    k = syn.make_keys(nb, hkv, d, kinds, seed=3)
    v = syn.make_values(nb * 512, hkv, d, seed=3)
    q = syn.make_queries(1, hq, d, seed=3)
    kf, vf, qf = k.float().cpu().numpy(), v.float().cpu().numpy(), q.float().cpu().numpy()
    ref = O.score_blocks(qf, kf, -np.inf, 5.0)
    keep_ref = ref["keep"]
    rp, rn = O.stream_compact_mask(keep_ref)
    b0 = int(rp[0])  # a retained block
    want = O.indirect_attention(qf, kf, vf, rp, rn)
    ws_bytes = lib.oc_decode_step_workspace_bytes(1, 1, hq, hkv, d, nb * 512)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    outs = (torch.empty((nb, hkv), dtype=torch.uint8, device="cuda"),
            torch.empty((nb,), dtype=torch.int32, device="cuda"),
            torch.empty((1,), dtype=torch.int32, device="cuda"),
            torch.empty((1, hq, d), dtype=torch.bfloat16, device="cuda"))
    assert lib.oc_device_status(1) == 0
    try:
        assert lib.oc_set_wait_limit_ns(2_000_000) == 0  # 2 ms
        # epoch 0 -> counter set 0, whose first words are blk_state[0 .. nb):
        # retained block b0 starts with a head count its last head never
        # completes, so it is never published in the queue
        ws.view(torch.int32)[1 + b0] = 0x4000
        assert _call(lib, q, k, v, -float("inf"), ws, outs) == 0
        torch.cuda.synchronize()  # the kernel returned: the waits are bounded
        status = lib.oc_device_status(1)
        assert status & 1, f"expected the fused layer's status bit, got {status}"
    finally:
        assert lib.oc_set_wait_limit_ns(2_000_000_000) == 0
    # the context is usable; a re-zeroed workspace gives the right answer
    ws.zero_()
    assert _call(lib, q, k, v, -float("inf"), ws, outs) == 0
    torch.cuda.synchronize()
    assert lib.oc_device_status(1) == 0
    keep, perm, count, out = outs
    assert np.array_equal(keep.cpu().numpy().astype(bool), keep_ref)
    assert int(count[0]) == rn and np.array_equal(perm.cpu().numpy(), rp)
    np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=1e-2, atol=2e-2)


def test_wait_limit_bounds_are_checked():
    from orthocache_b200 import _lib
    lib = _lib.load()
    assert lib.oc_set_wait_limit_ns(10) == -2
    assert lib.oc_set_wait_limit_ns(61_000_000_000) == -2
