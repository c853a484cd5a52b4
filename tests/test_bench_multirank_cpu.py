"""The multi-rank logic of bench.py (replicas, one process per GPU) on CPU: two
gloo ranks, each with its own timing; the reported time is the maximum over
ranks and the whole-job throughput counts every rank's tokens."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r, w, local = bench.dist_env()
        assert (r, w, local) == (rank, world, rank)
        # rank 1 is the slower replica
        dev_ms, e2e_ms = bench.max_over_ranks([10.0 + 5.0 * rank, 20.0 - rank], w)
        value = bench.replica_throughput(w, 128, dev_ms)
        dist.barrier()
        out[rank] = (dev_ms, e2e_ms, value)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_report_the_slowest_rank_and_all_tokens():
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    for rank in range(world):
        dev_ms, e2e_ms, value = out[rank]
        assert dev_ms == 15.0 and e2e_ms == 20.0
        assert abs(value - 2 * 128 / 0.015) < 1e-6


def test_single_process_needs_no_collective():
    assert bench.max_over_ranks([3.0, 4.0], 1) == [3.0, 4.0]
    assert bench.replica_throughput(1, 10, 5.0) == 2000.0
