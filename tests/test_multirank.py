"""bench.py's N > 1 host path on two gloo ranks (CPU).

Images are independent, so each rank encodes its own shard and nothing crosses
ranks on the data path; the only collectives are the barrier and the max over
ranks of the step time. Checked here: distinct shards per rank, every rank
sees the slowest rank's time, and the job throughput counts all ranks' images.
"""
import os
import socket
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        import bench
        from sparsesam_b200 import host
        ms = bench.max_over_ranks(10.0 * (rank + 1), world, torch.device("cpu"))
        img = host.synthetic_images(1, seed=bench.shard_seed(rank), img_size=64)
        mine = torch.tensor([float(img.double().sum())], dtype=torch.float64)
        sums = [torch.zeros(1, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(sums, mine)  # test-side only: compare the shards
        dist.barrier()
        q.put((rank, ms, [float(t) for t in sums]))
    finally:
        dist.destroy_process_group()


def test_two_ranks_shard_and_time():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    by_rank = dict((r, (ms, sums)) for r, ms, sums in results)
    assert sorted(by_rank) == [0, 1]
    for r in range(world):
        assert by_rank[r][0] == 20.0           # both ranks report the slowest rank's time
    sums = by_rank[0][1]
    assert sums == by_rank[1][1] and sums[0] != sums[1]   # distinct image shards


def test_job_throughput_counts_every_rank():
    import bench
    assert bench.job_throughput(64, 2, 5, 20.0) == 64 * 2 * 5 / 0.02
    assert bench.job_throughput(64, 1, 5, 20.0) * 2 == bench.job_throughput(64, 2, 5, 20.0)
    assert bench.max_over_ranks(3.5, 1, None) == 3.5
    assert bench.shard_seed(0) != bench.shard_seed(1)
