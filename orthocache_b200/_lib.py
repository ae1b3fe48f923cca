"""ctypes binding of ``liborthocache_b200.so`` (the C ABI in include/orthocache_b200.h).

The shared library is built in-tree by ``orthocache_b200.build``.  Nothing here
has a fallback: if the library is missing or a call fails, an exception is
raised.  Device buffers are torch CUDA tensors; the current torch stream is
passed to every call.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liborthocache_b200.so")

OC_F32 = 0
OC_BF16 = 1

_p = C.c_void_p
_i = C.c_int
_i64 = C.c_int64
_f = C.c_float
_sz = C.c_size_t

# name -> (restype, argtypes); mirrors include/orthocache_b200.h
SIGNATURES = {
    "oc_version": (_i, []),
    "oc_status_string": (C.c_char_p, [_i]),
    "oc_last_error": (C.c_char_p, []),
    "oc_device_status": (_i, [_i]),
    "oc_set_wait_limit_ns": (_i, [C.c_uint64]),
    "oc_fwht512": (_i, [_p, _i, _i64, _p, _p]),
    "oc_score_blocks": (_i, [_p, _p, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _f, _f,
                             _p, _p, _p, _p, _p, _p, _p, _p, _i, _p]),
    "oc_block_energy": (_i, [_p, _i, _i, _i, _i, _i, _i, _p, _p]),
    "oc_block_metadata": (_i, [_p, _i, _i, _i, _i, _i, _p, _p, _p, _p]),
    "oc_score_from_metadata": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _f, _p, _p, _p, _p]),
    "oc_stream_compact": (_i, [_p, _i, _i, _i, _p, _p, _p]),
    "oc_gather_blocks": (_i, [_p, _i, _i, _i, _i64, _p, _i, _p, _p, _i, _i, _p]),
    "oc_scatter_blocks": (_i, [_p, _i, _i, _i, _i64, _p, _i, _p, _p, _i, _p]),
    "oc_bucket_count": (_i, [_p, _i, _i, _p, _p]),
    "oc_apply_gates": (_i, [_p, _p, _i64, _p, _f, _f, _p, _p]),
    "oc_indirect_attention_workspace_bytes": (_sz, [_i, _i, _i, _i, _i, _i, _i]),
    "oc_nccl_version": (_i, []),
    "oc_comm_unique_id": (_i, [_p]),
    "oc_comm_init": (_i, [C.POINTER(_p), _p, _i, _i]),
    "oc_comm_destroy": (_i, [_p]),
    "oc_comm_check": (_i, [_p]),
    "oc_comm_abort": (_i, [_p]),
    "oc_exchange_workspace_bytes": (_sz, [_i, _i, _i, _i, _i]),
    "oc_exchange_stratified": (_i, [_p, _p, _p, _i, _p, _p, _i, _i, _i, _i, _p, _p, _p, _p, _p, C.POINTER(_i),
                                    _p, _sz, _p]),
    "oc_alltoallv_heads": (_i, [_p, _p, _p, _i, _p, _p, _i, _i, _i, _i, _p, _p, _p, C.POINTER(_i), _p, _sz, _p]),
    "oc_decode_step_sharded_workspace_bytes": (_sz, [_i, _i, _i, _i, _i, _i, _i]),
    "oc_sharded_connect": (_i, [_p, _p, _sz, _i, _i, _i, _i, _i, _i, _p]),
    "oc_sharded_disconnect": (_i, [_p]),
    "oc_decode_step_sharded": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _f, _p, _p, _p, _p, _i, _p, _sz,
                                    _p]),
    "oc_indirect_attention": (_i, [_p, _p, _p, _i, _p, _i, _i, _p, _i, _i, _i, _i, _i, _i, _i, _i, _i,
                                   _i, _p, _i, _p, _sz, _p]),
    "oc_prefill_attention": (_i, [_p, _p, _p, _i, _p, _i, _i, _p, _i, _i, _i, _i, _i, _i, _i, _i, _i,
                                  _i, _p, _i, _p]),
    "oc_indirect_attention_paged_workspace_bytes": (_sz, [_i, _i, _i, _i, _i, _i, _i]),
    "oc_indirect_attention_paged": (_i, [_p, _p, _p, _i, _p, _i, _p, _i, _p, _i, _i, _i, _i, _i, _i, _i, _i, _i,
                                         _p, _i, _p, _sz, _p]),
    "oc_prefill_attention_paged_workspace_bytes": (_sz, [_i, _i]),
    "oc_prefill_attention_paged": (_i, [_p, _p, _p, _i, _p, _i, _p, _i, _p, _i, _i, _i, _i, _i, _i, _i, _i, _i,
                                        _p, _i, _p, _sz, _p]),
    "oc_score_from_metadata_paged": (_i, [_p, _p, _p, _i, _p, _i, _p, _i, _i, _i, _i, _i, _i, _i, _f, _f, _p, _p,
                                          _p, _p]),
    "oc_indirect_attention_noalloc_max_scratch_bytes": (_sz, []),
    "oc_indirect_attention_noalloc": (_i, [_p, _p, _p, _i, _p, _i, _i, _p, _i, _i, _i, _i, _i, _i, _i, _i, _i,
                                           _i, _p, _i, _p]),
    "oc_partial_attention": (_i, [_p, _p, _p, _i, _p, _i, _i, _p, _i, _i, _i, _i, _i, _i, _i, _i, _i,
                                  _i, _p, _p, _p, _p, _sz, _p]),
    "oc_empty_heads_mean": (_i, [_p, _i, _p, _i, _i, _i, _i, _i, _i, _i, _i, _p, _i, _p]),
    "oc_merge_partials": (_i, [_p, _p, _p, _i, _i, _i, _p, _i, _p]),
    "oc_decode_step_workspace_bytes": (_sz, [_i, _i, _i, _i, _i, _i]),
    "oc_decode_step": (_i, [_p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _f, _p, _p, _p, _p, _i, _p, _sz,
                            _p]),
    "oc_decode_step_from_metadata": (_i, [_p, _p, _p, _i, _p, _p, _p, _i, _i, _i, _i, _i, _i, _f, _f, _p, _p, _p,
                                          _p, _i, _p, _sz, _p]),
    "oc_decode_step_partial": (_i, [_p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _f, _p, _p, _p, _p, _p, _p, _p,
                                    _sz, _p]),
    "oc_merge_partials_packed": (_i, [_p, _i, _i, _i, _p, _i, _p]),
    "oc_exchange_index": (_i, [_p, _i, _i, _p, _p, _p, _p]),
    "oc_stratified_bucket": (_i, [_i, _i]),
}


class OrthoCacheError(RuntimeError):
    """A C-ABI call returned an error status."""


_lock = threading.Lock()
_lib = None


def load():
    """Load the shared library (once) and bind every entry point."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m orthocache_b200.build` "
                "(nvcc, sm_100a). There is no CPU fallback.")
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def call(name, *args):
    """Call entry point ``name``; raise OrthoCacheError on a nonzero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.oc_last_error().decode(errors="replace")
        status = lib.oc_status_string(rc).decode()
        raise OrthoCacheError(f"{name}: {status} ({rc}): {msg}")
    return rc


def query(name, *args):
    """Call a size/query entry point and return its value."""
    return getattr(load(), name)(*args)


# ---------------------------------------------------------------------------
# tensor helpers
# ---------------------------------------------------------------------------
def require_cuda():
    if not torch.cuda.is_available():
        raise RuntimeError("orthocache_b200 needs a CUDA device (B200, sm_100a); none is visible")


def stream_ptr(device=None):
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return OC_F32
    if t.dtype == torch.bfloat16:
        return OC_BF16
    raise TypeError(f"unsupported dtype {t.dtype}: use float32 or bfloat16")


def as_device(x, device=None, dtype=None) -> torch.Tensor:
    """A contiguous CUDA tensor view of ``x`` (numpy arrays and CPU tensors are copied)."""
    require_cuda()
    if not isinstance(x, torch.Tensor):
        x = torch.as_tensor(x)
    if device is None:
        device = x.device if x.is_cuda else torch.device("cuda", torch.cuda.current_device())
    x = x.to(device=device, dtype=dtype if dtype is not None else x.dtype, non_blocking=True)
    if x.dtype == torch.float64:
        x = x.float()
    return x.contiguous()


def ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())
