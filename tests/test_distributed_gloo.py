"""Sequence-parallel exchange logic on two gloo ranks (CPU, no GPU needed):
count sync, offsets, the packed-buffer exchange, the receive-side layout and
the stratified bucket consensus, each checked against the oracle."""
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import dist_cases  # noqa: E402


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _entry(rank, world, port, result_dir):
    dist_cases.run(rank, world, port, result_dir)


@pytest.mark.timeout(300)
def test_exchange_two_gloo_ranks(tmp_path):
    world = 2
    mp.spawn(_entry, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert (tmp_path / f"ok{r}").exists()


def test_ici_data_volume_and_buckets():
    from orthocache_b200 import distributed as ocd
    from oracle import oc_oracle as O
    v = ocd.ici_data_volume(128, 8, [32] * 8, 8, 128)
    assert v["dense_bytes"] == 128 * 8 * 512 * 8 * 128 * 2
    assert v["sparse_bytes"] == 256 * 512 * 8 * 128 * 2
    assert abs(v["savings_pct"] - 75.0) < 1e-9
    for nb in (1, 2, 3, 4, 7, 16, 128):
        assert ocd.stratified_buckets(nb) == O.stratified_buckets(nb)
        for g in range(0, nb + 1):
            assert ocd.stratified_bucket(g, nb) == O.stratified_bucket(g, O.stratified_buckets(nb))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_block_data_paths_fail_without_gpu():
    """Packing, unpacking and attention run only on the CUDA kernels."""
    from orthocache_b200 import distributed as ocd
    with pytest.raises(Exception):
        ocd.pack_active_blocks(torch.zeros(1024, 1, 8), torch.arange(2, dtype=torch.int32),
                               torch.tensor([1]), 2)
