"""Multi-GPU partitions of the hot path: one process per GPU over torch.distributed.

Two partitions of one long sequence, both giving every query row exactly the
ids and output of a single-GPU run:

* KV-head groups (no collective): selection and attention never mix KV heads
  (the routing score sums only a KV head's own G query heads,
  top_k_pyramid_torch.py:80), so rank r takes KV heads
  [r*H/P, (r+1)*H/P) and their query heads and runs the whole path on them.

* Sequence shards (NCCL all-gather): rank r owns the contiguous query range
  [start_r, stop_r) (multiples of the block size) and the keys/values of the
  same range.  It pools its own leaf blocks, all-gathers the leaf means and
  the keys/values of every rank, and rebuilds the upper pyramid levels
  locally from the gathered leaf means.  The routing needs the whole
  pyramid (its geometry depends on the key count and a valid coarse node's
  mean covers keys past the query, as in the reference), and leaf scoring and
  attention read raw keys/values of earlier shards, so all of them land in
  this GPU's memory before any kernel reads them.  Rebuilding level l+1 from
  level l pools in the same order as the one-GPU build, so the pyramid is
  bit-identical.

The functions take a process group and work with any backend (NCCL on the
GPUs; the partition and gather logic is tested with gloo on the CPU).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def head_groups(q_heads, kv_heads, rank, world):
    """(kv_slice, q_slice) of rank `rank`: a contiguous group of KV heads and their query heads."""
    if kv_heads % world:
        raise ValueError(f"{kv_heads} KV heads do not split over {world} ranks")
    per = kv_heads // world
    groups = q_heads // kv_heads
    return slice(rank * per, (rank + 1) * per), slice(rank * per * groups, (rank + 1) * per * groups)


def sequence_shards(tokens, block_size, world):
    """Contiguous [start, stop) token ranges, one per rank, on block boundaries,
    as equal as the block size allows (the per-token cost is about constant
    once a query sees more than top-K blocks)."""
    blocks = -(-tokens // block_size)
    bounds = [min(tokens, (blocks * r // world) * block_size) for r in range(world + 1)]
    bounds[-1] = tokens
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


def all_gather_tokens(local, shards, group=None):
    """Concatenate every rank's [B, n_r, ...] token shard along dim 1 (ranks in order).

    Shards of unequal length are padded to the longest for the collective and
    trimmed after it."""
    world = dist.get_world_size(group)
    longest = max(b - a for a, b in shards)
    n = local.shape[1]
    if n < longest:
        pad = local.new_zeros((local.shape[0], longest - n, *local.shape[2:]))
        local = torch.cat([local, pad], 1)
    local = local.contiguous()
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local, group=group)
    return torch.cat([p[:, : b - a] for p, (a, b) in zip(parts, shards)], 1)


def sequence_sharded_prefill(q_local, k_local, v_local, shards, rank, *, method="pisa", block_size=64, topk=32,
                             force_first=True, force_recent=1, branching=2, group=None):
    """Select and attend the query rows [start, stop) of rank `rank` of one
    sequence whose keys/values are sharded the same way.  Returns (ids, out) for
    the local rows, equal to rows [start, stop) of a single-GPU run."""
    from .selection import mean_pool

    start, stop = shards[rank]
    if start % block_size or (stop % block_size and stop != shards[-1][1]):
        raise ValueError("sequence shards must start on block boundaries")
    # leaf means of this rank's own key blocks, then every rank's
    leaves_local = mean_pool(k_local, block_size)
    leaf_shards = [(a // block_size, -(-b // block_size)) for a, b in shards]
    leaves = all_gather_tokens(leaves_local, leaf_shards, group)
    keys = all_gather_tokens(k_local, shards, group)
    values = all_gather_tokens(v_local, shards, group)
    return rows_from_gathered(q_local, leaves, keys, values, start, method=method, block_size=block_size,
                              topk=topk, force_first=force_first, force_recent=force_recent,
                              branching=branching)


def rows_from_gathered(q_local, leaves, keys, values, start, *, method="pisa", block_size=64, topk=32,
                       force_first=True, force_recent=1, branching=2):
    """The local rows' selection and attention once the leaf means and the
    keys/values of the whole sequence are in this GPU's memory."""
    from .attention import sparse_attention
    from .layout import full_level_sizes
    from .selection import build_pyramid, routing_geometry, select_blocks

    # upper levels rebuilt locally: pooling the gathered leaf means by the
    # branching factor is the one-GPU pyramid's next level
    top, _ = routing_geometry(leaves.shape[1], topk, branching)
    levels = [leaves]
    if top > 0:
        levels += build_pyramid(leaves, branching, max_level=top - 1, branching=branching)
    sizes = full_level_sizes(leaves.shape[1], branching)[: len(levels)]
    assert [x.shape[1] for x in levels] == sizes
    ids = select_blocks(q_local, keys, method=method, block_size=block_size, topk=topk, query_offset=start,
                        force_first=force_first, force_recent=force_recent, pyramid=levels,
                        branching=branching)
    out = sparse_attention(q_local, keys, values, ids, block_size=block_size, query_offset=start)
    return ids, out
