"""Module-name twin of the reference's ``orthocache.distributed_attention``
(``distributed_attention.py``), implemented in :mod:`orthocache_b200.distributed`."""
from .distributed import (  # noqa: F401
    BLOCK_SIZE, stream_compact, distributed_orthocache_attention, ici_data_volume,
    sequence_parallel_attention, stratified_allgather_attention,
)
