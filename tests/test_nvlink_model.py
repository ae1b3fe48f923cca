"""The interconnect byte model: the restated reference model against its
outputs (tests/golden/ici_model.json, made by make_ici_golden.py from the
reference's ici_bandwidth_model.py), and the exchange byte counts of the
three sharded paths against hand-computed values."""
import json
import os

import pytest

from orthocache_b200 import nvlink_model as M

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ici_model.json")


def test_ici_model_matches_reference_outputs():
    g = json.load(open(GOLDEN))
    for args, want in g["per_step"]:
        assert M.ici_bytes_per_step(*args) == want, args
    for (args, want), levels in zip(g["table"], [None, [0.0, 0.25, 0.75]]):
        assert M.ici_bandwidth_table(*args, 2, levels) == want


def test_ici_model_rejects_bad_sparsity():
    with pytest.raises(ValueError):
        M.ici_bytes_per_step(1, 512, 128, 8, 1, 1.5)


def test_exchange_bytes():
    # config 3 at 8 GPUs, one layer: 32 query heads x (128 + 2) words of 8 bytes to 7 peers
    assert M.exchange_bytes("partials", 1, 8, 128, 8, num_q_heads=32) == 7 * 32 * 130 * 8
    # one GPU exchanges nothing
    assert M.exchange_bytes("partials", 60, 1, 128, 8, num_q_heads=32) == 0
    blk = 512 * 128 * 2 * 2
    assert M.exchange_bytes("stratified", 1, 8, 128, 8, kept_blocks=30, bucket_blocks=32) == 7 * 32 * 8 * blk
    assert M.exchange_bytes("alltoallv_heads", 1, 8, 128, 8, kept_blocks=30) == 7 * 30 * 1 * blk
    with pytest.raises(ValueError):
        M.exchange_bytes("alltoallv_heads", 1, 3, 128, 8, kept_blocks=1)
    with pytest.raises(ValueError):
        M.exchange_bytes("ring", 1, 2, 128, 8)
    assert M.exchange_time_us(770_000) == pytest.approx(1.0)
