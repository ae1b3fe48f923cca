"""NCCL communicator for the C-ABI exchange entry points.

The reference's ``axis_name`` (a pmap axis) becomes an ``NcclComm``: an NCCL
communicator created through the library (``oc_comm_unique_id`` on rank 0,
shared over the given ``torch.distributed`` group, ``oc_comm_init`` on every
rank), used by ``oc_exchange_stratified``, ``oc_alltoallv_heads`` and
``oc_decode_step_sharded``.  The library resolves NCCL at run time and
prefers the copy already loaded in the process (PyTorch's).

Failure detection is host-side: ``check()`` raises if NCCL holds an
asynchronous error (a peer failed or aborted), and ``watchdog()`` polls it
from a thread and aborts the communicator so that ranks blocked in a
collective return.
"""
from __future__ import annotations

import ctypes as C
import threading

import torch
import torch.distributed as dist

from . import _lib

UNIQUE_ID_BYTES = 128


class NcclComm:
    """One rank's NCCL communicator (collective creation over ``group``)."""

    def __init__(self, group=None, device=None):
        _lib.require_cuda()
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        lib = _lib.load()
        if lib.oc_nccl_version() < 0:
            raise _lib.OrthoCacheError(lib.oc_last_error().decode())
        uid = (C.c_char * UNIQUE_ID_BYTES)()
        if self.rank == 0:
            _lib.call("oc_comm_unique_id", C.cast(uid, C.c_void_p))
        obj = [bytes(uid) if self.rank == 0 else None]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        uid = (C.c_char * UNIQUE_ID_BYTES).from_buffer_copy(obj[0])
        ptr = C.c_void_p()
        with torch.cuda.device(self.device):
            _lib.call("oc_comm_init", C.byref(ptr), C.cast(uid, C.c_void_p), self.size, self.rank)
        self.ptr = ptr.value
        self._stop = None

    # -- failure detection -------------------------------------------------
    def check(self):
        """Raise OrthoCacheError if NCCL reports an asynchronous error."""
        _lib.call("oc_comm_check", self.ptr)

    def abort(self):
        """Abort the communicator: blocked collectives on this rank return."""
        if self.ptr:
            _lib.load().oc_comm_abort(self.ptr)
            self.ptr = None

    def watchdog(self, interval=0.5, on_error=None):
        """Poll ``check()`` every ``interval`` s in a daemon thread; on an error,
        abort and call ``on_error(exc)``.  Returns a stop function."""
        stop = threading.Event()

        def run():
            while not stop.wait(interval):
                if not self.ptr:
                    return
                try:
                    self.check()
                except _lib.OrthoCacheError as e:
                    self.abort()
                    if on_error is not None:
                        on_error(e)
                    return

        threading.Thread(target=run, daemon=True).start()
        self._stop = stop
        return stop.set

    def close(self):
        if self._stop is not None:
            self._stop.set()
        if self.ptr:
            _lib.load().oc_comm_destroy(self.ptr)
            self.ptr = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
