"""Multi-rank host logic, as two gloo ranks on the CPU.

* the benchmark: a multi-GPU run reports the slowest rank's device time and
  the reference arm runs on rank 0 only;
* the sequence-sharded partition (nlogn_pisa_b200/sharding.py): block-aligned
  shards, the padded all-gather that reassembles every rank's tokens (leaf
  means, keys, values) in rank order, and the KV-head groups.
These checks need no GPU: the collectives run over gloo on CPU tensors.
"""

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(fn, world=2):
    manager = mp.Manager()
    results = manager.dict()
    mp.spawn(fn, args=(world, _free_port(), results), nprocs=world, join=True)
    return dict(results)


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    return dist


def _bench_rank(rank, world, port, results):
    dist = _init(rank, world, port)
    try:
        import bench
        from nlogn_pisa_b200.workloads import WORKLOADS

        # per-rank step times: the reported value is the slowest rank's
        got = bench.max_over_ranks([1.0 + rank, 5.0 - rank, 0.5 * rank], "cpu", world)
        cfg = bench.arm_config(WORKLOADS["prefill32k"], world)

        class Args:
            steps, warmup, cpu_rows, ref_rows, gpus = 1, 0, 1, 1, world

        # the reference arm: ranks other than 0 return at once without work
        ref = bench.run_reference(Args(), WORKLOADS["config1"]) if rank != 0 else 0
        results[rank] = (got, cfg["parallelism"], ref)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_to_the_slowest():
    results = _spawn(_bench_rank)
    for rank in range(2):
        got, parallelism, ref = results[rank]
        assert got == pytest.approx([2.0, 5.0, 0.5])
        assert parallelism.startswith("dp2")
        assert ref == 0


def _shard_rank(rank, world, port, results):
    dist = _init(rank, world, port)
    try:
        from nlogn_pisa_b200.sharding import all_gather_tokens, head_groups, sequence_shards

        out = {}
        for tokens, block in ((1000, 64), (4096, 64), (130, 16)):
            shards = sequence_shards(tokens, block, world)
            # every rank's shard: rows of a seeded sequence, each rank keeping only its own
            g = torch.Generator().manual_seed(tokens)
            full = torch.randn(2, tokens, 3, 8, generator=g)
            a, b = shards[rank]
            gathered = all_gather_tokens(full[:, a:b], shards)
            out[tokens] = (shards, torch.equal(gathered, full))
            # leaf-mean shards: block counts per rank, gathered the same way
            leaf_shards = [(s // block, -(-e // block)) for s, e in shards]
            idx = torch.arange(leaf_shards[rank][0], leaf_shards[rank][1], dtype=torch.float32)
            got = all_gather_tokens(idx.view(1, -1, 1, 1), leaf_shards)
            out[(tokens, "leaves")] = torch.equal(got.view(-1), torch.arange(-(-tokens // block), dtype=torch.float32))
        out["heads"] = [head_groups(32, 8, r, world) for r in range(world)]
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_sequence_shards_gather_back_in_rank_order():
    results = _spawn(_shard_rank)
    for rank in range(2):
        out = results[rank]
        for tokens, block in ((1000, 64), (4096, 64), (130, 16)):
            shards, same = out[tokens]
            assert same, tokens
            assert out[(tokens, "leaves")], tokens
            assert shards[0][0] == 0 and shards[-1][1] == tokens
            assert all(a % block == 0 for a, _ in shards)
            assert all(shards[i][1] == shards[i + 1][0] for i in range(len(shards) - 1))
        kv0, q0 = out["heads"][0]
        kv1, q1 = out["heads"][1]
        assert (kv0, q0) == (slice(0, 4), slice(0, 16)) and (kv1, q1) == (slice(4, 8), slice(16, 32))


def test_head_groups_must_divide():
    from nlogn_pisa_b200.sharding import head_groups, sequence_shards

    with pytest.raises(ValueError):
        head_groups(32, 8, 0, 3)
    assert sequence_shards(64 * 5, 64, 8)[-1] == (256, 320)
