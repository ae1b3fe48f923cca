"""``fwht_512`` drop-in (reference: src/orthocache/fwht.py:4-65)."""
from __future__ import annotations

import torch

from . import _lib


def fwht_512(x) -> torch.Tensor:
    """512-row Fast Walsh–Hadamard Transform along axis 0, normalised by 1/sqrt(512).

    Same contract as the reference: ``x`` of shape (512, d) or (512,);
    natural (Hadamard) coefficient order; the butterfly stages run in the
    reference's order (h = 1, ..., 256) with ``a + b`` / ``a - b`` and the
    final float32 division by 22.627416997969522 (``fwht.py:25-61``), so the
    float32 result is bit-identical to the reference's float32 butterfly.
    Input float32 or bfloat16 (widened to float32); output float32 on the
    device of ``x``.
    """
    x = _lib.as_device(x)
    if x.dim() not in (1, 2) or x.shape[0] != 512:
        raise ValueError(f"fwht_512 expects shape (512, d) or (512,), got {tuple(x.shape)}")
    x2 = x.reshape(512, -1)
    y = torch.empty(x2.shape, dtype=torch.float32, device=x.device)
    _lib.call("oc_fwht512", _lib.ptr(x2), _lib.dtype_code(x2), x2.shape[1], _lib.ptr(y),
              _lib.stream_ptr(x.device))
    return y.reshape(x.shape)
