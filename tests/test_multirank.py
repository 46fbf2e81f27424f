"""The multi-GPU path on the CPU: two gloo ranks (127.0.0.1), each running its own rows of the
workload, the way ``bench.py --gpus 2`` shards it (weak scaling, no data-path collective).

Checks the host-side logic that the N > 1 bench relies on: the max-over-ranks timing
reduction, the whole-job rate, and that per-rank shards processed independently give the same
coefficients as one process over all rows (rows are independent for every op).
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import bench
    from oracle import dwt_oracle as D
    from pytorch_morlet_fdwt_b200.wavelets import get_filter_bank
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # timings differ per rank; every rank must see the element-wise maximum
        mine = [10.0 + rank, 3.0 - rank, 5.0 * (rank + 1)]
        got = bench.max_over_ranks(mine, world, torch.device("cpu"))
        expect = [10.0 + world - 1, 3.0, 5.0 * world]
        assert got == expect, (got, expect)
        # this rank's shard of a (4, 300) batch through the CPU oracle
        b = get_filter_bank("db4")
        tb = (b.dec_lo, b.dec_hi, b.rec_lo, b.rec_hi)
        x = np.random.default_rng(7).standard_normal((4, 300))
        shard = x[rank::world]
        c = D.wavedec(shard, tb, "symmetric", 3)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), *c)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_shards_and_reduction(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    from oracle import dwt_oracle as D
    from pytorch_morlet_fdwt_b200.wavelets import get_filter_bank
    b = get_filter_bank("db4")
    tb = (b.dec_lo, b.dec_hi, b.rec_lo, b.rec_hi)
    x = np.random.default_rng(7).standard_normal((4, 300))
    full = D.wavedec(x, tb, "symmetric", 3)
    for r in range(world):
        got = np.load(tmp_path / f"rank{r}.npz")
        for k, ref in enumerate(full):
            np.testing.assert_array_equal(got[f"arr_{k}"], ref[r::world])


def test_job_throughput_is_weak_scaling_aggregate():
    import sys
    sys.path.insert(0, ROOT)
    import bench
    # two ranks, each 100 units per step, 10 steps, slowest rank 500 ms -> 4000 units/s
    assert bench.job_throughput(100, 10, 2, 500.0) == pytest.approx(4000.0)
    assert bench.job_throughput(2e9, 1, 1, 1000.0, 1e9) == pytest.approx(2.0)
