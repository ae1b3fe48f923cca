"""Helpers shared by the GPU parity tests."""
import numpy as np
import pytest
import torch

from oracle import oc_oracle as O

needs_gpu = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")

# attention parity contract (bf16): 1e-2 relative / 2e-2 absolute
ATT_RTOL, ATT_ATOL = 1e-2, 2e-2


def dev(x, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(x)).cuda()
    return t.to(dtype) if dtype is not None else t


def host(t):
    return t.detach().float().cpu().numpy() if t.dtype in (torch.bfloat16, torch.float16) else t.detach().cpu().numpy()


def bf16_round(x):
    return torch.as_tensor(np.asarray(x, np.float32)).to(torch.bfloat16).float().numpy()


def assert_mask_parity(got, want, zeta, bmax, tau, zeta_max):
    """Bit-exact keep mask except cells within 1e-5 relative of a threshold;
    returns the number of exempt cells that differ (reported, not hidden)."""
    got = np.asarray(got, bool)
    want = np.asarray(want, bool)
    near = O.near_threshold(zeta, bmax, tau, zeta_max)
    bad = (got != want) & ~near
    assert not bad.any(), f"{bad.sum()} mask cells differ away from the thresholds: {np.argwhere(bad)[:10]}"
    diff_near = int(((got != want) & near).sum())
    if diff_near:
        print(f"[parity] {diff_near} near-threshold cells differ (exempt)")
    return diff_near
