"""The multi-GPU path of bench.py is replicas only (one image per GPU, no collective on the
data path): per-rank image seeds and the max-over-ranks timing, exercised with two gloo
ranks on CPU."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ms = 100.0 + 10.0 * rank  # rank 1 is the slow one
        m = bench.max_over_ranks(ms, world, "cpu")
        out[rank] = (bench.image_seed(rank), m, bench.whole_job_rate(28, world, m))
    finally:
        dist.destroy_process_group()


def test_two_replicas_seed_and_max_time():
    world = 2
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
    seeds = {out[r][0] for r in range(world)}
    assert len(seeds) == world  # every replica denoises a different image
    for r in range(world):
        assert out[r][1] == 110.0  # job time = slowest rank
        assert abs(out[r][2] - world * 28 / 0.110) < 1e-9
