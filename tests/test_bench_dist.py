"""The multi-GPU bench path on CPU: world_size-2 gloo ranks check the
replica aggregation (max over ranks of device time, sum of units)."""
import os
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, ws, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(ws))
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    sys.path.insert(0, ROOT)
    import bench
    value, ms = bench.aggregate_throughput(10.0 * (rank + 1), 32, 100, ws)
    q.put((rank, value, ms, bench.dist_max(float(rank), ws)))
    dist.destroy_process_group()


def test_replica_aggregation_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, value, ms, mx in res:
        assert ms == 20.0 and mx == 1.0
        assert abs(value - 2 * 32 * 100 / 0.020) < 1e-6
