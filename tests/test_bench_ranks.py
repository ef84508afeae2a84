"""Host logic of the multi-GPU replica bench on CPU ranks (gloo, world size 2): episodes are
partitioned disjointly by rank and seeded by their global index, each rank's device time is
reduced as the max over ranks, and the job throughput counts every rank's episodes. No GPU and
no collective on a data path: the path does not shard (replicas only)."""
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, str(ROOT))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        import bench
        eps = bench.episodes_of_rank(rank, batch)
        local_ms = [2.0 + 0.5 * rank, 3.0 - 0.25 * rank]    # rank 1 is slower on the first, faster on the second
        ms_max, e2e_max = bench.max_over_ranks(local_ms, world, "cpu")
        q.put((rank, eps, ms_max, e2e_max, bench.job_episodes_per_s(world, batch, ms_max)))
    finally:
        torch.distributed.destroy_process_group()


def test_replica_ranks_partition_and_reduce():
    world, batch = 2, 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    eps = [r[1] for r in res]
    assert eps == [[0, 1, 2], [3, 4, 5]]                     # disjoint, consecutive, cover 0..world*batch-1
    for _, _, ms_max, e2e_max, thr in res:                   # every rank sees the same reduced values
        assert ms_max == 2.5 and e2e_max == 3.0
        assert abs(thr - world * batch * 1000.0 / 2.5) < 1e-9


def test_single_rank_helpers():
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.episodes_of_rank(0, 1) == [0]
    assert bench.max_over_ranks([1.5, 2.5], 1, "cpu") == [1.5, 2.5]
    assert bench.job_episodes_per_s(1, 1, 4.0) == 250.0
