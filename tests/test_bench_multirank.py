"""The multi-GPU bench's host side on CPU: two gloo ranks (world size 2) exchange their
times; the job's time is the slowest rank's and its throughput counts every rank's work
(weak scaling, request replicas, no collective on the data path)."""
import os
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    import datetime

    import torch.distributed as dist
    import bench
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    try:
        assert bench.dist_env() == (rank, world, rank)
        mine = [1.0 + rank, 5.0 - rank]  # device time, wall time of this rank
        t = bench.max_over_ranks(mine, world)
        dist.barrier()
        q.put((rank, [float(v) for v in t], bench.job_throughput(1500, world, float(t[0]))))
    finally:
        dist.destroy_process_group()


def test_two_rank_reduction_is_max_and_throughput_weak():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    for rank, t, thr in res:
        assert t == [2.0, 5.0]          # element-wise max over the two ranks
        assert thr == pytest.approx(1500 * 2 / 2.0)


def test_single_rank_needs_no_process_group():
    sys.path.insert(0, str(ROOT))
    import bench
    assert list(bench.max_over_ranks([3.0, 4.0], 1)) == [3.0, 4.0]
    assert bench.job_throughput(1500, 1, 1.5) == pytest.approx(1000.0)
