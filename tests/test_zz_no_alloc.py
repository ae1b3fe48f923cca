"""The allocation-free attention entry point, through the C ABI.

oc_indirect_attention_noalloc serves callers that cannot allocate device
memory while they run the attention (for example an FFI host without a CUDA
allocator, or a serving loop whose memory pool forbids allocation inside a
step): it takes its scratch from a fixed per-device array instead of a
caller workspace.  Its output must match oc_indirect_attention's on the same
inputs, on consecutive calls that reuse the same scratch.

This file is collected last so that a run stopping at the first failure has
already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oc_oracle as O

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-2  # the bf16 attention tolerance of the parity tests


def _case(seed, nb, hq, hkv, d, keep_p, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = (torch.randn((1, hq, d), generator=g, device="cuda") * d ** -0.5).to(dtype)
    k = torch.randn((nb * 512, hkv, d), generator=g, device="cuda").to(dtype)
    v = torch.randn((nb * 512, hkv, d), generator=g, device="cuda").to(dtype)
    rs = np.random.RandomState(seed)
    m = rs.rand(nb) < keep_p
    m[0] = True
    idx = torch.tensor(np.concatenate([np.flatnonzero(m), np.flatnonzero(~m)]), dtype=torch.int32, device="cuda")
    cnt = torch.tensor([int(m.sum())], dtype=torch.int32, device="cuda")
    return q, k, v, idx, cnt


def _code(t):
    return 1 if t.dtype == torch.bfloat16 else 0


def _args(q, k, v, idx, cnt):
    sq, hq, d = q.shape
    s, hkv, _ = k.shape
    nb = s // 512
    return [ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(v.data_ptr()), _code(q),
            ctypes.c_void_p(idx.data_ptr()), nb, 0, ctypes.c_void_p(cnt.data_ptr()), 1, 0,
            1, sq, hq, hkv, d, s, 512, nb]


def _with_workspace(lib, q, k, v, idx, cnt):
    out = torch.empty_like(q)
    sq, hq, d = q.shape
    s, hkv, _ = k.shape
    ws_bytes = lib.oc_indirect_attention_workspace_bytes(1, sq, hq, hkv, d, 512, s // 512)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    rc = lib.oc_indirect_attention(*_args(q, k, v, idx, cnt), ctypes.c_void_p(out.data_ptr()), _code(out),
                                   ctypes.c_void_p(ws.data_ptr()), ws_bytes,
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.oc_last_error()
    return out


def _no_alloc(lib, q, k, v, idx, cnt, out):
    return lib.oc_indirect_attention_noalloc(*_args(q, k, v, idx, cnt), ctypes.c_void_p(out.data_ptr()), _code(out),
                                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_no_alloc_matches_workspace_entry_point_twice():
    from orthocache_b200 import _lib
    lib = _lib.load()
    # calls in a row on the same scratch: a large shape, then smaller ones
    # that leave most of it holding the earlier call's partials; bf16 with
    # head_dim 128 and 256, and float32 (three different partial kernels)
    cases = [_case(1, 128, 32, 8, 128, 0.25), _case(2, 16, 8, 8, 128, 0.6),
             _case(3, 12, 16, 4, 256, 0.5), _case(4, 8, 8, 2, 64, 0.5, torch.float32)]
    outs = [torch.full_like(c[0], float("nan")) for c in cases]
    for c, o in zip(cases, outs):
        rc = _no_alloc(lib, *c, o)
        assert rc == 0, lib.oc_last_error()
    torch.cuda.synchronize()
    for c, o in zip(cases, outs):
        want = _with_workspace(lib, *c)
        torch.cuda.synchronize()
        got = o.float().cpu().numpy()
        np.testing.assert_allclose(got, want.float().cpu().numpy(), rtol=RTOL, atol=ATOL)
        # and against the CPU restatement of the reference's attention loop
        q, k, v, idx, cnt = c
        ref = O.indirect_attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                                   idx.cpu().numpy(), int(cnt[0]))
        np.testing.assert_allclose(got, ref, rtol=RTOL, atol=ATOL)
    assert lib.oc_device_status(1) == 0


def test_no_alloc_rejects_shapes_above_the_limit():
    from orthocache_b200 import _lib
    lib = _lib.load()
    limit = lib.oc_indirect_attention_noalloc_max_scratch_bytes()
    # 32 query rows per kv head over 1024 blocks needs far more than the limit
    need = lib.oc_indirect_attention_workspace_bytes(1, 8, 32, 8, 128, 512, 1024)
    assert need > limit
    q = torch.zeros((8, 32, 128), dtype=torch.bfloat16, device="cuda")
    k = torch.zeros((512, 8, 128), dtype=torch.bfloat16, device="cuda")
    idx = torch.zeros(1024, dtype=torch.int32, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    args = _args(q, k, k, idx, cnt)
    args[15], args[17] = 1024 * 512, 1024  # seq_len, max_blocks (checked before any launch)
    rc = lib.oc_indirect_attention_noalloc(*args, ctypes.c_void_p(q.data_ptr()), 1, None)
    assert rc == -4 and b"limit" in lib.oc_last_error()
