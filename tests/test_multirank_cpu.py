"""The multi-GPU path's host logic with two gloo ranks on the CPU: each rank
gets a disjoint set of utterances (weak scaling, nothing shared), and the job
time is the max over ranks."""
import os
import socket
import sys
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")
ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    import bench
    seeds = bench.rank_seeds(rank, 4, 64)
    times = bench.max_over_ranks([10.0 + rank, 3.0 - rank], world)
    gathered = [None] * world
    dist.all_gather_object(gathered, [s for b in seeds for s in b])
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, times, gathered))


def test_two_gloo_ranks_shard_and_reduce():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, times, gathered in out:
        assert times == [11.0, 3.0]                      # max over ranks, element-wise
        a, b = set(gathered[0]), set(gathered[1])
        assert len(a) == len(b) == 256 and not (a & b)   # disjoint utterance sets
        assert a | b == set(range(512))
