"""Pyramid level tables: one place for the node counts and storage offsets.

A pyramid over ``n`` keys with leaf blocks of ``C`` tokens and branching
``b`` has ``ceil(n / C)`` leaves and ``ceil(size / b)`` nodes on each next
level, up to a single root (mean_pooling.py:45-52 with b = 2; b = 4 is this
library's extension).  The PyramidCache storage keeps every level at a
fixed start inside one allocation; the same tables drive
``pisa_build_pyramid``, ``pisa_pyramid_update`` and the validation of a
caller's ``pyramid=`` argument in ``select_blocks``.
"""

from __future__ import annotations


def level_sizes(leaves, branching, levels):
    """Node counts of the first ``levels`` levels above ``leaves`` leaves."""
    sizes, n = [], leaves
    for _ in range(levels):
        sizes.append(n)
        n = -(-n // branching)
    return sizes


def full_level_sizes(leaves, branching):
    """Node counts from the leaves up to (and including) the single root."""
    sizes = [leaves]
    while sizes[-1] > 1:
        sizes.append(-(-sizes[-1] // branching))
    return sizes


def storage_layout(leaf_capacity, branching):
    """(capacities, starts, total) of a storage that can hold ``leaf_capacity`` leaves.

    Every level gets room for the ceil-divided node count of the level below,
    so the layout stays valid for any key count up to ``leaf_capacity * C``.
    """
    capacities = full_level_sizes(max(1, leaf_capacity), branching)
    starts, total = [], 0
    for cap in capacities:
        starts.append(total)
        total += cap
    return tuple(capacities), tuple(starts), total


def check_level_sizes(sizes, keys, block_size, branching, needed):
    """Raise ValueError unless ``sizes`` are the level sizes of ``keys`` keys.

    ``needed`` is the number of levels the routing descends (top + 1); a
    table may stop early only at a single-node level (top_k_pyramid_torch.py:145-147
    keeps using that node).
    """
    leaves = -(-keys // block_size)
    want = level_sizes(leaves, branching, len(sizes))
    if list(sizes) != want:
        raise ValueError(
            f"pyramid level sizes {list(sizes)} do not match {keys} keys with block_size {block_size} "
            f"and branching {branching} (expected {want})")
    if len(sizes) < needed and sizes[-1] != 1:
        raise ValueError(f"pyramid has {len(sizes)} levels but routing needs {needed}")
