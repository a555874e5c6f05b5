"""The multi-rank timing rule of bench.py on two gloo ranks (CPU): every rank
ends with the largest rank's time, and a rank's timing helper reads nothing
from the others before the reduction."""

from __future__ import annotations

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench

        mine = 0.001 * (rank + 1)
        assert bench._max_over_ranks(mine, dist) == pytest.approx(0.001 * world)
        assert bench._max_over_ranks(mine, None) == mine
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_max_over_ranks_two_gloo_ranks():
    mp.spawn(_rank, args=(2, _free_port()), nprocs=2, join=True)
