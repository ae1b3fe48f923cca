"""Module-name twin of the reference's ``orthocache.alltoallv`` (``alltoallv.py``):
the exchange protocol, implemented in :mod:`orthocache_b200.distributed`."""
from .distributed import (  # noqa: F401
    BLOCK_SIZE, stream_compact, count_sync, compute_offsets, pack_active_blocks, alltoallv_exchange,
    unpack_received_blocks, alltoallv_kv_exchange,
)
