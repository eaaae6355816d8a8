"""Batch sharding of a complex Conv2d over the GPUs of one node.

The reference has no multi-GPU path.  A convolution's output image depends
only on its own input image, so the batch shards across ranks with no data
exchange: one process per GPU, weights replicated (identical parameters on
every rank), each rank convolving its slice of the batch.  Collectives are
used only outside the data path: the max-over-ranks timing reduction and an
optional gather of the outputs for validation.
"""

from __future__ import annotations

from typing import Tuple

import torch


def batch_shard(global_batch: int, world_size: int, rank: int) -> Tuple[int, int]:
    """(start, count) of `rank`'s slice when `global_batch` images are split as
    evenly as possible over `world_size` ranks (the first ranks take one extra
    image when the split is uneven)."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} for world size {world_size}")
    if global_batch < 0:
        raise ValueError("global_batch must be non-negative")
    base, extra = divmod(global_batch, world_size)
    start = rank * base + min(rank, extra)
    count = base + (1 if rank < extra else 0)
    return start, count


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of a per-rank scalar over the default process group (the
    job's time is the slowest rank's).  Identity without a process group."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_batch(local: torch.Tensor, global_batch: int) -> torch.Tensor:
    """Concatenate every rank's output slice along the batch dimension on
    every rank (validation only; ranks may hold different slice sizes)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return local
    world = dist.get_world_size()
    counts = [batch_shard(global_batch, world, r)[1] for r in range(world)]
    width = max(counts)
    # Collectives move equal-sized buffers: pad every slice to the largest.
    buf = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    buf[: local.shape[0]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    if buf.is_complex():
        # Complex tensors travel as pairs of floats.
        dist.all_gather([torch.view_as_real(p) for p in parts], torch.view_as_real(buf))
    else:
        dist.all_gather(parts, buf)
    return torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0)
