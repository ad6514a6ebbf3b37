"""The N > 1 host logic of bench.py on CPU: two gloo ranks (no GPU).

Ranks time independent replicas; the job's time is the maximum over ranks and
its throughput counts every rank's units. The reference arm runs on rank 0
only and the other ranks return without work.
"""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import sys
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        ms = 100.0 + 50.0 * rank                   # rank 1 is the slower replica
        mx = bench.reduce_max(ms, "cpu")
        value = bench.job_value(world, 32, 10, mx)
        class Args:
            steps, warmup, gpus = 1, 0, world
        ran = bench.run_reference(Args) if rank != 0 else "rank0"
        out.put((rank, mx, value, ran))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_max_and_job_value():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, mx, value, ran in res:
        assert mx == 150.0                          # the slower rank's time, on every rank
        assert abs(value - 2 * 32 * 10 / 0.150) < 1e-6
    assert res[1][3] is None                        # reference arm: rank 1 returns without work


def test_single_process_value():
    import bench
    assert bench.reduce_max(3.5, "cpu") == 3.5
    assert bench.job_value(1, 32, 300, 1200.0) == 32 * 300 / 1.2
