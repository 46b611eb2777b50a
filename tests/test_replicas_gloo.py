"""bench.py's multi-GPU host logic on two gloo ranks (CPU): N replicas decode disjoint sequences, and the job's
time is the slowest rank's, so value = N x batch x steps / max over ranks of the device time."""
import os
import socket

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, batch, out):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        seeds = [bench.prompt_seed(rank, i) for i in range(batch)]
        every = [None] * world
        dist.all_gather_object(every, seeds)
        t = bench.reduce_max(0.25 * (rank + 1), world)
        out.put((rank, every, t))
    finally:
        dist.destroy_process_group()


def test_replicas_two_ranks():
    import torch.multiprocessing as mp
    world, batch = 2, 512
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, batch, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, every, t in got:
        assert t == pytest.approx(0.25 * world)  # the slowest rank's time on every rank
        flat = [s for seeds in every for s in seeds]
        assert len(set(flat)) == world * batch  # no sequence decoded twice across replicas
