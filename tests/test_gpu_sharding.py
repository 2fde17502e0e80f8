"""The two multi-GPU partitions of one sequence give exactly the one-GPU results.

Run on one GPU by emulating the ranks: each shard's computation is the one a
rank would run, and the all-gather is replaced by concatenation in rank
order (the gather itself is tested over gloo in test_multirank.py).  Ids and
outputs must be bit-identical to a single call over the whole sequence.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(device, N, Hq=32, H=8, D=128, seed=5, offset_std=0.5, C=64):
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(1, N, Hq, D, generator=g, device=device)
    k = torch.randn(1, N, H, D, generator=g, device=device)
    v = torch.randn(1, N, H, D, generator=g, device=device)
    blocks = -(-N // C)
    k = k + (torch.randn(1, blocks, H, D, generator=g, device=device) * offset_std).repeat_interleave(C, 1)[:, :N]
    return (x.to(torch.bfloat16) for x in (q, k, v))


@pytest.mark.parametrize("world,branching", [(2, 4), (4, 4), (3, 2)])
def test_sequence_shards_equal_one_gpu(cuda_device, world, branching):
    import nlogn_pisa_b200 as P
    from nlogn_pisa_b200.sharding import rows_from_gathered, sequence_shards

    N, C, K = 20000, 64, 32
    q, k, v = _inputs(cuda_device, N)
    want_ids = P.select_blocks(q, k, block_size=C, topk=K, force_recent=1, branching=branching)
    want_out = P.sparse_attention(q, k, v, want_ids, block_size=C)
    shards = sequence_shards(N, C, world)
    # what each rank contributes to the all-gathers: its own leaf means and tokens
    leaves = torch.cat([P.mean_pool(k[:, a:b], C) for a, b in shards], 1)
    for a, b in shards:
        ids, out = rows_from_gathered(q[:, a:b], leaves, k, v, a, block_size=C, topk=K, force_recent=1,
                                      branching=branching)
        assert torch.equal(ids, want_ids[:, a:b]), (a, b)
        assert torch.equal(out, want_out[:, a:b]), (a, b)


@pytest.mark.parametrize("world", [2, 8])
def test_kv_head_groups_equal_one_gpu(cuda_device, world):
    import nlogn_pisa_b200 as P
    from nlogn_pisa_b200.sharding import head_groups

    N, C, K = 12000, 64, 32
    q, k, v = _inputs(cuda_device, N, seed=6)
    want_ids = P.select_blocks(q, k, block_size=C, topk=K, force_recent=1, branching=4)
    want_out = P.sparse_attention(q, k, v, want_ids, block_size=C)
    for r in range(world):
        kv, qh = head_groups(q.shape[2], k.shape[2], r, world)
        qs, ks, vs = q[:, :, qh], k[:, :, kv], v[:, :, kv]
        ids = P.select_blocks(qs, ks, block_size=C, topk=K, force_recent=1, branching=4)
        out = P.sparse_attention(qs, ks, vs, ids, block_size=C)
        assert torch.equal(ids, want_ids[:, :, kv]), r
        assert torch.equal(out, want_out[:, :, qh]), r
