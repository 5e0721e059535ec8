"""Data-parallel host logic on CPU: world_size-2 gloo ranks partition the
requests (disjoint, complete) and reduce the run statistics exactly as the
multi-GPU bench does with NCCL."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import dp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, n, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = dp.partition(n, rank, world)
        stats = {"samples": (1920 * len(mine), "sum"), "frames": (len(mine), "sum"),
                 "device_s": (0.5 + rank, "max")}
        red = dp.reduce_stats(stats)
        out[rank] = (mine, red)
    finally:
        dist.destroy_process_group()


def test_partition_single_rank():
    assert dp.partition(5, 0, 1) == [0, 1, 2, 3, 4]
    with pytest.raises(ValueError):
        dp.partition(5, 2, 2)


def test_reduce_without_process_group():
    assert dp.reduce_stats({"a": (3, "sum"), "b": (2.5, "max")}) == {"a": 3.0, "b": 2.5}
    with pytest.raises(ValueError):
        dp.reduce_stats({"a": (1, "mean")})


def test_two_gloo_ranks():
    n, world = 13, 2
    out = mp.Manager().dict()
    mp.spawn(_rank, args=(world, _free_port(), n, out), nprocs=world, join=True)
    parts = [out[r][0] for r in range(world)]
    assert sorted(parts[0] + parts[1]) == list(range(n))
    assert not set(parts[0]) & set(parts[1])
    for r in range(world):
        red = out[r][1]
        assert red["samples"] == 1920 * n
        assert red["frames"] == n
        assert red["device_s"] == 1.5
