"""Multi-GPU parity of the NCCL exchange entry points (oc_exchange_stratified,
oc_alltoallv_heads, oc_decode_step_sharded) on 2, 4 or 8 GPUs, one process
per GPU under torchrun; the rank bodies are in tests/dist_nccl_cases.py.
Skipped on a machine with fewer than two GPUs."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.timeout(600)
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_nccl_exchange_and_sharded_decode(tmp_path):
    world = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "dist_nccl_cases.py"), str(tmp_path)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=540)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    for rank in range(world):
        assert (tmp_path / f"ok{rank}").exists(), rank
