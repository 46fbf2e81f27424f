"""The multi-GPU path on the CPU: gloo ranks (127.0.0.1) running the package's own sharding
helper (``pytorch_morlet_fdwt_b200.sharding``) the way ``bench.py --gpus N`` uses it.

* every rank takes its ``shard_batch`` of a batch, runs the op on it (the CPU oracle stands in
  for the GPU kernels, which need a device), and ``gather_batch`` reassembles the full result
  in rank order: equal to one process over the whole batch (rows are independent);
* uneven shards (a batch that does not divide by the world size) gather correctly too;
* ``all_reduce_grads`` of per-shard parameter gradients equals the full-batch gradient (the
  loss is a sum over batch entries) -- the data-parallel training step of the learnable layers;
* the max-over-ranks timing reduction and the whole-job rate of ``bench.py``.
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


def _attention_grads(x, freq_weight, log_scales):
    """Oracle MorletAttention-style forward + backward of sum(y^2) on CPU fp64: the gradients
    of the (shared) parameters."""
    from oracle import cwt_oracle as C
    po = C.Plan([2.0, 5.0, 11.0], support_margin=1.25)
    y = C.attention(x, po, po.filters(log_scales.exp(), 6.0), freq_weight, 0.8)
    y.square().sum().backward()
    return y


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import bench
    from oracle import dwt_oracle as D
    from pytorch_morlet_fdwt_b200.sharding import (all_reduce_grads, gather_batch, shard_batch,
                                                   shard_bounds)
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

        b = get_filter_bank("db4")
        tb = (b.dec_lo, b.dec_hi, b.rec_lo, b.rec_hi)
        for batch in (4, 5):  # even and uneven shards
            x = torch.from_numpy(np.random.default_rng(7).standard_normal((batch, 3, 300)))
            mine = shard_batch(x, rank, world)
            lo, hi = shard_bounds(batch, rank, world)
            assert mine.shape[0] == hi - lo
            coeffs = D.wavedec(mine.reshape(-1, 300).numpy(), tb, "symmetric", 3)
            parts = [gather_batch(torch.from_numpy(c).reshape(hi - lo, 3, -1)) for c in coeffs]
            if rank == 0:
                np.savez(os.path.join(out_dir, f"gathered{batch}.npz"),
                         *[p.numpy() for p in parts])

        # data-parallel gradients of shared parameters
        x = torch.from_numpy(np.random.default_rng(3).standard_normal((4, 2, 3, 2, 40)))
        fw = torch.from_numpy(np.random.default_rng(4).standard_normal((3, 3))).requires_grad_()
        ls = torch.tensor([2.0, 5.0, 11.0], dtype=torch.float64).log().requires_grad_()
        _attention_grads(shard_batch(x, rank, world).clone(), fw, ls)
        all_reduce_grads([fw, ls])
        if rank == 0:
            np.savez(os.path.join(out_dir, "grads.npz"), fw=fw.grad.numpy(), ls=ls.grad.numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_shard_gather_and_gradient_all_reduce(tmp_path, world):
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    from oracle import dwt_oracle as D
    from pytorch_morlet_fdwt_b200.wavelets import get_filter_bank
    b = get_filter_bank("db4")
    tb = (b.dec_lo, b.dec_hi, b.rec_lo, b.rec_hi)
    for batch in (4, 5):
        x = np.random.default_rng(7).standard_normal((batch, 3, 300))
        full = D.wavedec(x.reshape(-1, 300), tb, "symmetric", 3)
        got = np.load(tmp_path / f"gathered{batch}.npz")
        for k, ref in enumerate(full):
            np.testing.assert_array_equal(got[f"arr_{k}"], ref.reshape(batch, 3, -1))
    x = torch.from_numpy(np.random.default_rng(3).standard_normal((4, 2, 3, 2, 40)))
    fw = torch.from_numpy(np.random.default_rng(4).standard_normal((3, 3))).requires_grad_()
    ls = torch.tensor([2.0, 5.0, 11.0], dtype=torch.float64).log().requires_grad_()
    _attention_grads(x, fw, ls)
    g = np.load(tmp_path / "grads.npz")
    np.testing.assert_allclose(g["fw"], fw.grad.numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(g["ls"], ls.grad.numpy(), rtol=1e-12, atol=1e-12)


def test_shard_bounds_cover_the_batch():
    from pytorch_morlet_fdwt_b200.sharding import shard_bounds
    for batch in (0, 1, 7, 16, 64):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(batch, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def test_job_throughput_is_weak_scaling_aggregate():
    import sys
    sys.path.insert(0, ROOT)
    import bench
    # two ranks, each 100 units per step, 10 steps, slowest rank 500 ms -> 4000 units/s
    assert bench.job_throughput(100, 10, 2, 500.0) == pytest.approx(4000.0)
    assert bench.job_throughput(2e9, 1, 1, 1000.0, 1e9) == pytest.approx(2.0)
