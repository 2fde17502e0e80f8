"""Multi-rank host logic of the benchmark, as two gloo ranks on the CPU.

A multi-GPU run gives every rank its own sequence and reports the slowest
rank's device time; the reference arm runs on rank 0 only.  These checks need
no GPU: the reductions run over gloo.
"""

import os
import socket
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    import bench
    from nlogn_pisa_b200.workloads import WORKLOADS

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # per-rank step times: the reported value is the slowest rank's
        got = bench.max_over_ranks([1.0 + rank, 5.0 - rank, 0.5 * rank], "cpu", world)
        cfg = bench.arm_config(WORKLOADS["prefill32k"], world)

        class Args:
            steps, warmup, cpu_rows, gpus = 1, 0, 1, world

        # the reference arm: ranks other than 0 return at once without work
        ref = bench.run_reference(Args(), WORKLOADS["config1"]) if rank != 0 else 0
        results[rank] = (got, cfg["parallelism"], ref)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_to_the_slowest():
    world = 2
    manager = mp.Manager()
    results = manager.dict()
    mp.spawn(_rank_main, args=(world, _free_port(), results), nprocs=world, join=True)
    for rank in range(world):
        got, parallelism, ref = results[rank]
        assert got == pytest.approx([2.0, 5.0, 0.5])
        assert parallelism.startswith("dp2")
        assert ref == 0
