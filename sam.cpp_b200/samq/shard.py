"""Image sharding across GPUs (one process per GPU, no exchange on the data path).

SAM 3 images are independent, so G GPUs each hold a full weight replica and
run whole images: the batch of a throughput sweep is cut into G contiguous
ranges, rank g taking images [g * n / G, (g + 1) * n / G), processed in
per-GPU batches.  The only collectives are host-side bookkeeping around the
timed region: a barrier and the maximum of the ranks' device times, which is
the job's time (the slowest rank finishes the job).
"""
from __future__ import annotations


def image_range(n_images: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous share [start, end) of rank `rank` among `world` ranks."""
    if world <= 0 or not 0 <= rank < world or n_images < 0:
        raise ValueError("need world > 0, 0 <= rank < world and n_images >= 0")
    return rank * n_images // world, (rank + 1) * n_images // world


def batches(start: int, end: int, batch: int) -> list[tuple[int, int]]:
    """[start, end) cut into per-GPU batches of at most `batch` images."""
    if batch <= 0:
        raise ValueError("batch must be positive")
    return [(b, min(b + batch, end)) for b in range(start, end, batch)]


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """The maximum of `value` over all ranks of the default process group
    (`dist` is torch.distributed, None for a single process).  `device` is
    where the reduction tensor lives: a CUDA device for NCCL, the CPU for gloo."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
