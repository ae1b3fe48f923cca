"""Sequence-parallel exchange logic on two gloo ranks (CPU, no GPU needed):
count sync, offsets, the packed-buffer exchange, the receive-side layout and
the stratified bucket consensus, each checked against the oracle."""
import os
import socket
from pathlib import Path
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


def _warmup_entry(rank, world, port, result_dir):
    """Ranks whose steps take different times must still agree on the number
    of warm-up steps (each step of the sequence-parallel bench is a
    collective)."""
    import time
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(HERE))
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        t = torch.zeros(1)

        def step(i):
            time.sleep(0.0005 * (rank + 1))  # rank 1 is twice as slow
            dist.all_reduce(t)

        n = bench.warmup_steps(step, 5, 0.2, world, lambda: None, torch.device("cpu"))
        got = torch.tensor([n])
        dist.all_reduce(got, op=dist.ReduceOp.MAX)
        assert int(got) == n and n % 64 == 0 and n >= 64
        (Path(result_dir) / f"warm{rank}").write_text(str(n))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_bench_warmup_step_count_agrees_across_ranks(tmp_path):
    world = 2
    mp.spawn(_warmup_entry, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    counts = {(tmp_path / f"warm{r}").read_text() for r in range(world)}
    assert len(counts) == 1
