"""Batch sharding across the GPUs of one node (one process per GPU).

Every op of this package acts on independent rows (the leading dimensions), so a batch splits
across ranks with no collective on the data path.  The helpers here cover what is left:

* :func:`shard_batch` -- the contiguous slice of the batch dimension a rank owns;
* :func:`gather_batch` -- the optional all-gather of per-rank results along the batch
  dimension (``all_gather_into_tensor`` over NCCL on GPUs; a list all-gather on backends
  without it, e.g. gloo on the CPU);
* :func:`all_reduce_grads` -- one bucketed all-reduce (sum) of the parameter gradients of a
  module, for training the learnable layers on sharded batches (their gradients are a few
  KB: log-scales, w0, mix weights, frequency weights).

The row -> channel maps of the fused consumers (``d = r % dim`` for the mix, ``c = r % nch``
for the spectral softmax) survive sharding because shards are whole batch entries.
"""

from __future__ import annotations

from typing import Iterable, Optional, Tuple

import torch
import torch.distributed as dist

__all__ = ["shard_bounds", "shard_batch", "gather_batch", "all_reduce_grads"]


def shard_bounds(batch: int, rank: int, world: int) -> Tuple[int, int]:
    """``[begin, end)`` of the batch entries rank ``rank`` of ``world`` owns.  Shards differ in
    size by at most one entry; the first ``batch % world`` ranks take the larger ones."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a world of {world}")
    if batch < 0:
        raise ValueError("batch must be >= 0")
    base, extra = divmod(batch, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def shard_batch(x: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    """The rank's slice of ``x`` along the batch dimension ``dim`` (a view)."""
    b, e = shard_bounds(x.shape[dim], rank, world)
    return x.narrow(dim, b, e - b)


def gather_batch(y: torch.Tensor, group: Optional[dist.ProcessGroup] = None,
                 dim: int = 0) -> torch.Tensor:
    """Concatenation over ranks (in rank order) of every rank's ``y`` along ``dim``.

    Equal shard shapes on NCCL take one ``all_gather_into_tensor`` into a preallocated output;
    otherwise (uneven shards, or a backend without it) an ``all_gather`` of padded tensors."""
    world = dist.get_world_size(group)
    if world == 1:
        return y
    y = y.movedim(dim, 0).contiguous()
    sizes = torch.tensor([y.shape[0]], device=y.device, dtype=torch.int64)
    all_sizes = [torch.zeros_like(sizes) for _ in range(world)]
    dist.all_gather(all_sizes, sizes, group=group)
    n = [int(s.item()) for s in all_sizes]
    backend = dist.get_backend(group)
    if len(set(n)) == 1 and backend == "nccl":
        out = torch.empty((world * n[0],) + tuple(y.shape[1:]), device=y.device, dtype=y.dtype)
        dist.all_gather_into_tensor(out, y, group=group)
    else:
        m = max(n)
        pad = y.new_zeros((m,) + tuple(y.shape[1:]))
        pad[:y.shape[0]] = y
        parts = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(parts, pad, group=group)
        out = torch.cat([p[:k] for p, k in zip(parts, n)], 0)
    return out.movedim(0, dim)


def all_reduce_grads(params: Iterable[torch.nn.Parameter],
                     group: Optional[dist.ProcessGroup] = None, average: bool = False) -> None:
    """Sum (or average) the gradients of ``params`` over ranks with one all-reduce of a flat
    bucket.  Parameters without a gradient are skipped on every rank alike (the set must be
    the same on all ranks)."""
    grads = [p.grad for p in params if p.grad is not None]
    if not grads or dist.get_world_size(group) == 1:
        return
    flat = torch.cat([g.reshape(-1).to(torch.float64) for g in grads])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    if average:
        flat /= dist.get_world_size(group)
    off = 0
    for g in grads:
        k = g.numel()
        g.copy_(flat[off:off + k].view_as(g))
        off += k
