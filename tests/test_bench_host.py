"""Host-side multi-rank logic of bench.py on CPU: two gloo ranks (world size 2) agree on the
max-over-ranks timing, and only rank 0 of the reference arm does work."""
from __future__ import annotations

import os
import socket
import sys

import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import torch.distributed as dist
    sys.path.insert(0, REPO)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench
    out[rank] = bench.reduce_max([float(rank), 10.0 - rank, 3.5], world)
    dist.barrier()
    dist.destroy_process_group()


def test_reduce_max_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_rank_main, args=(2, _free_port(), out), nprocs=2, start_method="spawn", join=True)
        assert out[0] == [1.0, 10.0, 3.5] and out[1] == [1.0, 10.0, 3.5]


def test_reference_arm_nonzero_rank_does_nothing(capsys):
    sys.path.insert(0, REPO)
    import bench

    class A:
        steps, warmup, gpus = 1, 3, 2
    assert bench.run_reference(A, rank=1, world=2) == 0
    assert capsys.readouterr().out == ""
