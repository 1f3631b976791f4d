"""Multi-GPU sharding logic on the CPU: the image partition and the
max-over-ranks timing of bench.py, run as two gloo ranks (world_size 2, no
GPU).  Images are independent, so the partition must be contiguous, disjoint
and complete, and every rank must see the slowest rank's time."""
import os
import socket

import pytest

from samq.shard import batches, image_range, max_over_ranks


def test_partition_is_contiguous_disjoint_and_complete():
    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 4, 8):
            ranges = [image_range(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            for (a0, a1), (b0, _) in zip(ranges, ranges[1:]):
                assert a1 == b0 and a0 <= a1
            sizes = [e - s for s, e in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_config5_protocol_batches():
    """64 images over G = 1, 2, 4, 8 GPUs in per-GPU batches of 8."""
    for world in (1, 2, 4, 8):
        for rank in range(world):
            s, e = image_range(64, world, rank)
            assert (s, e) == (rank * 64 // world, (rank + 1) * 64 // world)
            bs = batches(s, e, 8)
            assert len(bs) == 8 // world and all(b1 - b0 == 8 for b0, b1 in bs)
    assert batches(0, 5, 8) == [(0, 5)]
    with pytest.raises(ValueError):
        image_range(64, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, queue):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        start, end = image_range(64, world, rank)
        own = list(range(start, end))
        gathered = [None] * world
        dist.all_gather_object(gathered, own)
        # rank r "took" 10 + r ms: every rank must report the slowest.
        slowest = max_over_ranks(10.0 + rank, dist)
        dist.barrier()
        queue.put((rank, gathered, slowest))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_partition_and_max_over_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, gathered, slowest in results:
        assert slowest == 11.0
        flat = [i for part in gathered for i in part]
        assert flat == list(range(64))
        assert gathered[0] == list(range(32)) and gathered[1] == list(range(32, 64))
