"""Multi-process control path on CPU (gloo, world_size 2): the benchmark's
max-over-ranks timing reduction and barrier, as every rank runs them."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import torch.distributed as dist

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    import bench

    w, r, _ = bench._dist()
    assert (w, r) == (world, rank)
    bench._barrier(w)
    results[rank] = bench._max_over_ranks(10.0 + rank, w)
    dist.destroy_process_group()


def test_max_over_ranks_gloo():
    world = 2
    port = _free_port()
    manager = mp.Manager()
    results = manager.dict()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert dict(results) == {0: 11.0, 1: 11.0}
