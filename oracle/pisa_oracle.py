"""CPU restatement of PISA block selection and selected-block attention (numpy).

TEST INFRASTRUCTURE ONLY.  This module is the parity checker for the CUDA
path in ``nlogn_pisa_b200``.  Only ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The product path never calls it; there is no CPU fallback.

Every function restates the reference algorithm of Aphelios-Tang/NlogN_PISA
(paths are relative to that project's root) in vectorised numpy:

* mean pooling / pyramid  -> pisa/pisa/ops/compress/mean_pooling/mean_pooling_torch.py:7-14,
                             pisa/pisa/ops/compress/mean_pooling/mean_pooling.py:45-52
* routing geometry/masks  -> pisa/pisa/ops/flash_sparse_attn/top_k_pyramid/top_k_pyramid_torch.py:6-14,114-133
* candidate scoring       -> top_k_pyramid_torch.py:48-80
* leaf scores of arbitrary candidates -> pisa/pisa/ops/flash_sparse_attn/top_k_pyramid/leaf_triton.py:23-60,144-232
* bitonic top-K network   -> top_k_pyramid_torch.py:84-110
* coarse-to-fine descent  -> top_k_pyramid_torch.py:137-177
* query positions         -> pisa/pisa/utils/validation.py:38-56
* flat BSA routing        -> pisa/pisa/ops/flash_sparse_attn/bsa/bsa_torch.py:9-106
* selected attention      -> pisa/pisa/ops/flash_sparse_attn/sparse_attn/sparse_attn_torch.py:6-35
  (the log-sum-exp output and the analytic gradient are restated from the
  same masked softmax; the reference obtains gradients through autograd)

Parity is pinned against outputs of the reference's own torch path, committed
as fixtures under ``tests/golden`` by ``tests/golden/make_golden.py``.

Branching factor.  The reference hard-codes a binary pyramid (pool by 2,
children ``2*id+{0,1}``, parent ``ceil(n/2)``).  Every function here takes a
``branching`` argument; ``branching=2`` is the reference.  For ``branching=b``
the pyramid pools by ``b``, children are ``b*id+{0..b-1}``, the parent count is
``ceil(n/b)``, ancestors are ``leaf // b**level`` and the second-order score
over ``b > 2`` children uses the general mean + variance form of
top_k_pyramid_torch.py:76-79 (the binary 1/2-sum + 1/8-difference^2 form of
:69-75 applies only to a support of exactly two).  This extension has no
reference counterpart and is pinned only through its reduction to b=2.

Dtypes.  Arrays are float32 or float64.  ``dtype`` names the torch dtype the
values stand for ("bf16", "f16", "f32", "f64"); pyramid levels are rounded to
it after each pooling, as ``torch_mean_pool`` casts back to ``keys.dtype``.
Scores accumulate in float32 (float64 for f64), as the reference does.
"""

from __future__ import annotations

import numpy as np

NEG_FILL = np.float32(-1e9)
POS_FILL = np.float32(1e9)
METHODS = ("pisa1", "pisa2", "pisa")


# ----------------------------------------------------------------------------
# dtype helpers
# ----------------------------------------------------------------------------

def round_bf16(x):
    """Round float32 values to the nearest-even bfloat16 (returned as float32)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    bias = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    return ((u + bias) & np.uint32(0xFFFF0000)).view(np.float32)


def cast(x, dtype):
    """Value-level stand-in for ``tensor.to(dtype)``."""
    if dtype == "f64":
        return x.astype(np.float64)
    x = x.astype(np.float32)
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    return x


def acc_type(dtype):
    return np.float64 if dtype == "f64" else np.float32


# ----------------------------------------------------------------------------
# pyramid (mean_pooling_torch.py:7-14, mean_pooling.py:45-52)
# ----------------------------------------------------------------------------

def mean_pool(keys, size, dtype="f32"):
    """Mean over the valid tokens of each ``size`` block; a tail divides by its count.

    Follows torch_mean_pool (mean_pooling_torch.py:7-14): sum in float32
    (float64 for f64), divide by ``clamp(length - i*size, 1, size)``, cast back.
    """
    if size < 1:
        raise ValueError("pool size must be positive")
    batch, length, heads, dim = keys.shape
    blocks = -(-length // size)
    acc = acc_type(dtype)
    padded = np.zeros((batch, blocks * size, heads, dim), acc)
    padded[:, :length] = keys
    sums = padded.reshape(batch, blocks, size, heads, dim).sum(2, dtype=acc)
    counts = np.clip(length - np.arange(blocks) * size, 1, size).astype(acc)
    return cast(sums / counts[None, :, None, None], dtype)


def build_pyramid(keys, block_size, dtype="f32", max_level=None, branching=2):
    """Leaf means first, then pools of ``branching`` up to the root (mean_pooling.py:45-52)."""
    if max_level is not None and (type(max_level) is not int or max_level < 0):
        raise ValueError("max_level must be a nonnegative integer or None")
    levels = [mean_pool(keys, block_size, dtype)]
    while levels[-1].shape[1] > 1 and (max_level is None or len(levels) <= max_level):
        levels.append(mean_pool(levels[-1], branching, dtype))
    return levels


# ----------------------------------------------------------------------------
# routing (top_k_pyramid_torch.py)
# ----------------------------------------------------------------------------

def routing_geometry(blocks, topk, branching=2):
    """Traversal depth and first network width (top_k_pyramid_torch.py:124-133)."""
    top = 0
    while blocks > topk:
        parent = -(-blocks // branching)
        if parent < topk or parent == blocks:
            break
        blocks = parent
        top += 1
    width = 1 << (max(blocks, topk) - 1).bit_length()
    return top, max(16, width)


def query_positions(batch, q_len, k_len, query_offset=None):
    """Absolute query positions [B, Tq] (validation.py:38-56)."""
    if query_offset is None or isinstance(query_offset, (int, np.integer)):
        offset = k_len - q_len if query_offset is None else int(query_offset)
        if offset < 0 or offset + q_len > k_len:
            raise ValueError("queries must refer to positions within their key sequence")
        return np.broadcast_to(np.arange(offset, offset + q_len, dtype=np.int64)[None], (batch, q_len))
    offset = np.asarray(query_offset, dtype=np.int64).reshape(-1)
    if offset.size not in (1, batch):
        raise ValueError("query_offset must be a scalar or one offset per batch element")
    positions = offset.reshape(-1, 1) + np.arange(q_len, dtype=np.int64)
    positions = np.broadcast_to(positions, (batch, q_len))
    if (positions < 0).any() or (positions >= k_len).any():
        raise ValueError("queries must refer to positions within their key sequence")
    return positions


def force_mask(ids, positions, block_size, force_first, force_recent, level=0, branching=2):
    """First block and the ancestors of the last ``force_recent`` leaves (:6-14)."""
    leaf = positions // block_size
    result = np.zeros(ids.shape, bool)
    if force_first:
        result |= ids == 0
    span = branching ** level
    for recent in range(force_recent):
        target = leaf - recent
        result |= (target[..., None] >= 0) & (ids == (target[..., None] // span))
    return result & (ids >= 0)


def routing_masks(ids, positions, block_size, topk, force_first, force_recent, level=0, branching=2):
    """valid / forced / scoreable with the all-fit identity shortcut (:114-120)."""
    span = branching ** level
    valid = (ids >= 0) & (ids * (block_size * span) <= positions[..., None])
    forced = force_mask(ids, positions, block_size, force_first, force_recent, level, branching) & valid
    if (forced.sum(-1) > topk).any():
        raise ValueError("topk is smaller than the number of required distinct blocks")
    identity = valid.sum(-1) <= topk
    return valid, forced, valid & ~forced & ~identity[..., None]


def block_scores(query, source, ids, support, method, scale):
    """Candidate scores summed over the G query heads of a KV head (:48-80).

    query  [R, H, G, D]  (one query token per row)
    source [R, n, H, D]  (the support rows for each query row; rows may share)
    ids    [R, H, W]     candidate ids, -1 for "do not score"
    Returns [R, H, W] in the accumulation dtype.
    """
    rows, heads, width = ids.shape
    acc = np.float64 if query.dtype == np.float64 else np.float32
    n = source.shape[1]
    samples = ids[..., None] * support + np.arange(support)
    valid = (samples >= 0) & (samples < n) & (ids[..., None] >= 0)
    r_idx = np.arange(rows)[:, None, None, None]
    h_idx = np.arange(heads)[None, :, None, None]
    values = source[r_idx, np.clip(samples, 0, n - 1), h_idx].astype(acc)  # [R,H,W,S,D]
    grouped = query.astype(acc)
    products = np.einsum("rhgd,rhwsd->rhgws", grouped, values, optimize=True)
    mask = np.broadcast_to(valid[:, :, None], products.shape)
    sc = acc(scale)
    if method == "pisa":
        logits = np.where(mask, products * sc, -np.inf)
        top = logits.max(-1, keepdims=True)
        top = np.where(np.isfinite(top), top, 0)
        with np.errstate(divide="ignore"):
            score = np.log(np.exp(logits - top).sum(-1)) + top[..., 0]
    else:
        count = np.maximum(mask.sum(-1), 1).astype(acc)
        mean = np.where(mask, products, 0).sum(-1) / count
        score = sc * mean
        if method == "pisa2":
            if support == 2:
                z = np.where(mask, products * sc, 0)
                total = z.sum(-1)
                difference = z[..., 0] - z[..., 1]
                score = np.where(count == 2, acc(0.5) * total + acc(0.125) * difference * difference, total)
            else:
                second = np.where(mask, products * products, 0).sum(-1) / count
                variance = np.maximum(second - mean * mean, 0)
                score = sc * mean + acc(0.5 * scale * scale) * variance
    return score.sum(2).astype(acc)


def leaf_scores(q, k, candidates, block_size, method, positions=None, topk=None, force_first=True,
                force_recent=2, leaf_means=None, dtype="f32"):
    """grouped_leaf_scores (leaf_triton.py:144-232): fp32 scores of arbitrary
    leaf candidates in candidate order, -inf where a slot is not scored.

    Slots with ids outside [0, blocks) are not scored (bucket_kernel,
    grouping_triton.py:34-36).  With ``positions`` [B, T] the level-0 masks of
    leaf_scoreable_mask (leaf_triton.py:23-60 -> score_masks,
    top_k_pyramid_triton.py:105-122) also drop ids past the position, forced
    ids and, for pisa / pisa2, rows whose valid ids all fit in ``topk``.
    Scores are block_scores (top_k_pyramid_torch.py:48-80) over the C raw keys
    (pisa, pisa2; scale D^-0.5) or over the leaf mean (pisa1; scale 1).
    """
    batch, tokens, q_heads, dim = q.shape
    heads, length = k.shape[2], k.shape[1]
    groups = q_heads // heads
    blocks = -(-length // block_size)
    ids = candidates.astype(np.int64)
    in_range = (ids >= 0) & (ids < blocks)
    if positions is None:
        scoreable = in_range
    else:
        pos = np.broadcast_to(np.asarray(positions, np.int64), (batch, tokens))
        pos = np.broadcast_to(pos[..., None], (batch, tokens, heads))
        valid = in_range & (ids * block_size <= pos[..., None])
        forced = force_mask(np.where(in_range, ids, -1), pos, block_size, force_first, force_recent) & valid
        scoreable = valid & ~forced
        if method != "pisa1":
            scoreable &= (valid.sum(-1) > topk)[..., None]
    acc = np.float64 if q.dtype == np.float64 else np.float32
    out = np.full(ids.shape, -np.inf, acc)
    if method == "pisa1":
        means = mean_pool(k, block_size, dtype) if leaf_means is None else leaf_means
        source, support, sc = means, 1, 1.0
    else:
        source, support, sc = k, block_size, dim ** -0.5
    for b in range(batch):
        query = q[b].reshape(tokens, heads, groups, dim)
        src = np.broadcast_to(source[b][None], (tokens,) + source[b].shape)
        score = block_scores(query, src, np.where(scoreable[b], ids[b], -1), support, method, sc)
        out[b] = np.where(scoreable[b], score, -np.inf)
    return out


def network_topk(scores, ids, topk, return_scores=False):
    """Descending bitonic network with its compare/exchange tie order (:84-110).

    Pads to a power of two with score -1e9 / id -1.  Equal scores exchange in a
    descending group and stay in an ascending group.
    """
    width = 1 << (scores.shape[-1] - 1).bit_length()
    pad = width - scores.shape[-1]
    if pad:
        scores = np.concatenate(
            [scores, np.full(scores.shape[:-1] + (pad,), NEG_FILL, scores.dtype)], -1)
        ids = np.concatenate([ids, np.full(ids.shape[:-1] + (pad,), -1, ids.dtype)], -1)
    lane = np.arange(width)
    for exponent in range(1, width.bit_length()):
        group = 1 << exponent
        descending = np.ones(width, bool) if group == width else (lane & group) != 0
        for shift in range(exponent - 1, -1, -1):
            distance = 1 << shift
            partner = lane ^ distance
            peer_score, peer_id = scores[..., partner], ids[..., partner]
            left = (lane & distance) == 0
            left_score = np.where(left, scores, peer_score)
            right_score = np.where(left, peer_score, scores)
            exchange = (left_score > right_score) != descending
            scores = np.where(exchange, peer_score, scores)
            ids = np.where(exchange, peer_id, ids)
    if return_scores:
        return ids[..., :topk], scores[..., :topk]
    return ids[..., :topk]


def _boundary_gap(scores, topk, floor=1e-6):
    """Relative gap between the K-th and (K+1)-th largest score of each row.

    Rows whose (K+1)-th entry is a fill value (fewer contenders than K) or
    whose K-th entry is forced have no boundary: their gap is +inf.
    """
    if scores.shape[-1] <= topk:
        return np.full(scores.shape[:-1], np.inf)
    ordered = -np.sort(-scores.astype(np.float64), axis=-1)
    kth, nxt = ordered[..., topk - 1], ordered[..., topk]
    real = (nxt > -1e8) & (kth < 1e8)
    gap = np.abs(kth - nxt) / np.maximum(np.abs(kth), floor)
    return np.where(real, gap, np.inf)


def pyramid_select(q, k, method, block_size, topk, positions, force_first, force_recent,
                   levels, geometry=None, branching=2, chunk=16, trace=None):
    """Coarse-to-fine descent for every query row (top_k_pyramid_torch.py:137-177).

    q [B, T, Hq, D]; k [B, N, H, D]; positions [B, T] int64; levels list of
    [B, n_l, H, D] arrays.  Returns int64 ids [B, T, H, topk] in network-rank
    order, -1 padded.  ``trace`` (a dict) receives the leaf-level candidate ids
    and scores for tie-aware comparisons: trace["leaf_ids"], trace["leaf_scores"].
    """
    if method not in METHODS:
        raise ValueError("method must be pisa1, pisa2 or pisa")
    batch, length, q_heads, dim = q.shape
    heads = k.shape[2]
    groups = q_heads // heads
    top, first_width = geometry or routing_geometry(levels[0].shape[1], topk, branching)
    # A one-node local pyramid remains that node at additional common levels (:145-147).
    levels = list(levels) + [levels[-1]] * max(0, top + 1 - len(levels))
    scale = dim ** -0.5
    acc = np.float64 if q.dtype == np.float64 else np.float32
    out = np.empty((batch, length, heads, topk), np.int64)
    leaf_ids_all, leaf_scores_all, gaps_all = [], [], []
    for b in range(batch):
        for start in range(0, length, chunk):
            stop = min(start + chunk, length)
            rows = stop - start
            position = np.broadcast_to(positions[b, start:stop, None], (rows, heads))
            query = q[b, start:stop].reshape(rows, heads, groups, dim)
            ids = np.broadcast_to(np.arange(first_width, dtype=np.int64), (rows, heads, first_width)).copy()
            for level in range(top, -1, -1):
                total = levels[level].shape[1]
                ids = np.where(ids >= total, -1, ids)
                valid, forced, scoreable = routing_masks(
                    ids, position, block_size, topk, force_first, force_recent, level, branching)
                if method == "pisa1":
                    scoreable = valid & ~forced
                    source, support, sc = levels[level][b], 1, 1.0
                else:
                    if level == 0:
                        source, support = k[b], block_size
                    else:
                        source, support = levels[level - 1][b], branching
                    sc = scale
                scores = np.zeros(ids.shape, acc)
                if scoreable.any():
                    src = np.broadcast_to(source[None], (rows,) + source.shape)
                    scores = block_scores(query, src, np.where(scoreable, ids, -1), support, method, sc)
                scores = np.where(scoreable, scores, 0)
                scores = np.where(valid, scores, NEG_FILL)
                scores = np.where(forced, POS_FILL, scores).astype(acc)
                if trace is not None:
                    gap = _boundary_gap(scores, topk)
                    gaps = gap if level == top else np.minimum(gaps, gap)
                    if level == 0:
                        leaf_ids_all.append(ids.copy())
                        leaf_scores_all.append(scores.copy())
                        gaps_all.append(gaps)
                ids = network_topk(scores, ids, topk)
                if level:
                    children = ids[..., None] * branching + np.arange(branching)
                    children = np.where(ids[..., None] < 0, -1, children)
                    ids = children.reshape(rows, heads, topk * branching)
            ids = np.where((ids < 0) | (ids * block_size > position[..., None]), -1, ids)
            out[b, start:stop] = ids
    if trace is not None:
        trace["leaf_ids"] = np.concatenate(leaf_ids_all, 0).reshape(batch, length, heads, -1)
        trace["leaf_scores"] = np.concatenate(leaf_scores_all, 0).reshape(batch, length, heads, -1)
        trace["min_gap"] = np.concatenate(gaps_all, 0).reshape(batch, length, heads)
    return out


def select_blocks(q, k, method="pisa", block_size=64, topk=8, query_offset=None,
                  force_first=True, force_recent=2, dtype="f32", branching=2, trace=None,
                  positions=None):
    """``select_blocks(..., backend="torch")`` without packing (top_k_pyramid.py:11-122)."""
    if block_size < 1 or topk < 1 or force_recent < 0:
        raise ValueError("positive block_size/topk and nonnegative force_recent required")
    if force_recent == 0:
        raise ValueError("causal pyramid routing requires force_recent >= 1")
    if positions is None:
        positions = query_positions(q.shape[0], q.shape[1], k.shape[1], query_offset)
    levels = build_pyramid(k, block_size, dtype, branching=branching)
    return pyramid_select(q, k, method, block_size, topk, positions, force_first,
                          force_recent, levels, branching=branching, trace=trace)


# ----------------------------------------------------------------------------
# flat BSA routing (pisa/pisa/ops/flash_sparse_attn/bsa/bsa_torch.py)
# ----------------------------------------------------------------------------

def _merge(scores, ids, stage, descending):
    """One bitonic merge of runs of 2**stage through XOR partners (bsa_torch.py:9-27).

    ``descending=None`` makes run r descend when bit ``stage`` of its lanes is
    set; otherwise every run goes the given way.  A pair exchanges when
    (lower score > upper score) differs from the run's direction, so equal
    scores exchange in descending runs and stay in ascending ones.
    """
    lane = np.arange(scores.shape[-1])
    direction = (lane & (1 << stage)) != 0 if descending is None else np.full(lane.shape, descending)
    for exponent in range(stage - 1, -1, -1):
        distance = 1 << exponent
        partner = lane ^ distance
        lower = lane & ~distance
        upper = lower | distance
        exchange = (scores[..., lower] > scores[..., upper]) != direction
        scores = np.where(exchange, scores[..., partner], scores)
        ids = np.where(exchange, ids[..., partner], ids)
    return scores, ids


def streaming_topk(scores, ids, topk, tile_size):
    """Best ``topk`` ids by tiles of ``tile_size`` (bsa_torch.py:30-60).

    Each tile is sorted into alternating runs, merged ascending against the
    retained best half of the earlier tiles, then merged descending; tiles
    without a valid id leave the retained list alone.  Ids come out in
    network-rank order.
    """
    if topk < 1 or tile_size < 2 * topk or tile_size & (tile_size - 1):
        raise ValueError("tile_size must be a power of two and at least 2 * topk")
    stages = tile_size.bit_length() - 1
    half = tile_size // 2
    retained_scores = np.full(scores.shape[:-1] + (tile_size,), -1, scores.dtype)
    retained_ids = np.zeros(ids.shape[:-1] + (tile_size,), ids.dtype)
    for start in range(0, scores.shape[-1], tile_size):
        values = scores[..., start:start + tile_size]
        indices = ids[..., start:start + tile_size]
        active = (indices >= 0).any(-1, keepdims=True)
        pad = tile_size - values.shape[-1]
        if pad:
            values = np.concatenate([values, np.zeros(values.shape[:-1] + (pad,), values.dtype)], -1)
            indices = np.concatenate([indices, np.full(indices.shape[:-1] + (pad,), -1, indices.dtype)], -1)
        for stage in range(1, stages):
            values, indices = _merge(values, indices, stage, None)
        if start:
            values, indices = _merge(values, indices, stages, False)
            values = np.concatenate([retained_scores[..., :half], values[..., half:]], -1)
            indices = np.concatenate([retained_ids[..., :half], indices[..., half:]], -1)
        values, indices = _merge(values, indices, stages, True)
        retained_scores = np.where(active, values, retained_scores)
        retained_ids = np.where(active, indices, retained_ids)
    return retained_ids[..., :topk]


def bsa_required(positions, block_size, force_first, force_recent):
    """Largest number of distinct required blocks over the rows (bsa_torch.py:88-95)."""
    current = np.asarray(positions) // block_size
    recent = np.minimum(force_recent, current + 1)
    return int((recent + ((current >= force_recent) & bool(force_first))).max())


def bsa_select(q, k, block_size, topk, positions, force_first=True, force_recent=2, dtype="f32",
               chunk=128, trace=None):
    """Flat block routing by summed per-head probabilities (bsa_torch.py:63-106).

    Summaries are the leaf means.  Each query head's logits against the
    complete blocks (``(pos + 1) // C`` of them) give a log-sum-exp
    normaliser; blocks strictly before the current one score
    exp(logit - normaliser), required blocks (first, and the ``force_recent``
    most recent) score 1, and the per-head values are summed over the G heads
    of the KV head.  Ids past the current block are -1.  The query is scaled
    by D**-0.5 in the accumulation type and rounded to its own dtype first.
    Returns int64 ids [B, T, H, topk] in network-rank order.  ``trace`` gets
    ``min_gap``: the relative gap between the K-th and (K+1)-th score per row.
    """
    if bsa_required(positions, block_size, force_first, force_recent) > topk:
        raise ValueError("topk is smaller than the number of required distinct blocks")
    summaries = mean_pool(k, block_size, dtype)
    acc = acc_type(dtype)
    batch, length, q_heads, dim = q.shape
    heads = k.shape[2]
    groups = q_heads // heads
    width = 1 << (max(block_size, 2 * topk) - 1).bit_length()
    count = summaries.shape[1]
    blocks = np.arange(count)
    scale = acc(dim ** -0.5)
    out = np.empty((batch, length, heads, topk), np.int64)
    gaps = np.empty((batch, length, heads))
    for start in range(0, length, chunk):
        stop = min(start + chunk, length)
        query = cast(q[:, start:stop].astype(acc) * scale, dtype).astype(acc)
        query = query.reshape(batch, stop - start, heads, groups, dim)
        logits = np.einsum("bthgd,bmhd->bthgm", query, summaries.astype(acc)).astype(acc)
        position = np.asarray(positions)[:, start:stop, None, None]
        current = position // block_size
        complete = (position + 1) // block_size
        visible = (blocks < complete[..., None])
        masked = np.where(visible, logits, -np.inf)
        peak = masked.max(-1, keepdims=True)
        safe = np.where(np.isfinite(peak), peak, 0)
        with np.errstate(divide="ignore"):
            normalizer = (safe + np.log(np.exp(masked - safe).sum(-1, keepdims=True, dtype=acc))).astype(acc)
        normalizer = np.where(complete[..., None] > 0, normalizer, acc(0))
        forced = np.zeros(current.shape + (count,), bool)
        if force_first:
            forced |= blocks == 0
        for recent in range(force_recent):
            forced |= (current[..., None] >= recent) & (blocks == current[..., None] - recent)
        valid = blocks <= current[..., None]
        candidate = np.where(blocks < current[..., None], logits, -np.inf)
        with np.errstate(over="ignore"):
            probabilities = np.exp(candidate - normalizer).astype(acc)
        probabilities = np.where(forced, acc(1), probabilities)
        scores = probabilities.sum(-2, dtype=acc)
        ids = np.where(valid[..., 0, :], blocks, -1)
        ids = np.broadcast_to(ids, scores.shape).astype(np.int64)
        out[:, start:stop] = streaming_topk(scores, ids, topk, width)
        if trace is not None:
            gaps[:, start:stop] = _boundary_gap(scores, topk)
    if trace is not None:
        trace["min_gap"] = gaps
    return out


# ----------------------------------------------------------------------------
# selected-block attention (sparse_attn_torch.py:6-35)
# ----------------------------------------------------------------------------

def _gather_tokens(indices, block_size, k_len, positions, causal):
    offsets = np.arange(block_size)
    tokens = (indices[..., None] * block_size + offsets).reshape(*indices.shape[:-1], -1)
    valid = (tokens >= 0) & (tokens < k_len)
    if causal:
        valid &= tokens <= positions[:, :, None, None]
    return np.clip(tokens, 0, k_len - 1), valid


def sparse_attention(q, k, v, indices, block_size, scale=None, positions=None, causal=True,
                     chunk=32):
    """Attention over selected blocks with a shared softmax.

    Returns (out [B,T,Hq,Dv] float32/64, lse [B,T,Hq]); rows without a visible
    key give out = 0 and lse = -inf (sparse_attn_torch.py:29-31).
    """
    batch, length, q_heads, dim = q.shape
    heads = k.shape[2]
    groups = q_heads // heads
    scale = dim ** -0.5 if scale is None else scale
    acc = np.float64 if q.dtype == np.float64 else np.float32
    if positions is None:
        positions = query_positions(batch, length, k.shape[1])
    out = np.zeros((batch, length, q_heads, v.shape[-1]), acc)
    lse = np.full((batch, length, q_heads), -np.inf, acc)
    b_idx = np.arange(batch)[:, None, None, None]
    h_idx = np.arange(heads)[None, None, :, None]
    for start in range(0, length, chunk):
        stop = min(start + chunk, length)
        ids = np.asarray(indices[:, start:stop], np.int64)
        tokens, valid = _gather_tokens(ids, block_size, k.shape[1], positions[:, start:stop], causal)
        keys = k[b_idx, tokens, h_idx].astype(acc)      # [B,t,H,S,D]
        values = v[b_idx, tokens, h_idx].astype(acc)
        query = q[:, start:stop].astype(acc).reshape(batch, stop - start, heads, groups, dim)
        logits = np.einsum("bthgd,bthsd->bthgs", query, keys, optimize=True) * acc(scale)
        mask = valid[..., None, :]
        masked = np.where(mask, logits, -np.inf)
        top = masked.max(-1, keepdims=True)
        any_valid = np.isfinite(top)
        top = np.where(any_valid, top, 0)
        ex = np.where(mask, np.exp(masked - top), 0)
        denom = ex.sum(-1, keepdims=True)
        prob = np.where(any_valid, ex / np.where(denom > 0, denom, 1), 0)
        res = np.einsum("bthgs,bthsv->bthgv", prob, values, optimize=True)
        out[:, start:stop] = res.reshape(batch, stop - start, q_heads, -1)
        with np.errstate(divide="ignore"):
            row_lse = np.where(any_valid[..., 0], np.log(np.where(denom[..., 0] > 0, denom[..., 0], 1)) + top[..., 0], -np.inf)
        lse[:, start:stop] = row_lse.reshape(batch, stop - start, q_heads)
    return out, lse


def sparse_attention_backward(q, k, v, indices, block_size, dout, scale=None, positions=None,
                              causal=True, chunk=32):
    """Gradients of ``sum(out * dout)`` for :func:`sparse_attention`.

    The analytic softmax gradient; duplicated block ids contribute once per
    occurrence, exactly as the reference's gather/autograd does.
    """
    batch, length, q_heads, dim = q.shape
    heads, k_len = k.shape[2], k.shape[1]
    groups = q_heads // heads
    scale = dim ** -0.5 if scale is None else scale
    acc = np.float64 if q.dtype == np.float64 else np.float32
    if positions is None:
        positions = query_positions(batch, length, k_len)
    dq = np.zeros(q.shape, acc)
    dk = np.zeros(k.shape, acc)
    dv = np.zeros(v.shape, acc)
    b_idx = np.arange(batch)[:, None, None, None]
    h_idx = np.arange(heads)[None, None, :, None]
    for start in range(0, length, chunk):
        stop = min(start + chunk, length)
        t = stop - start
        ids = np.asarray(indices[:, start:stop], np.int64)
        tokens, valid = _gather_tokens(ids, block_size, k_len, positions[:, start:stop], causal)
        keys = k[b_idx, tokens, h_idx].astype(acc)
        values = v[b_idx, tokens, h_idx].astype(acc)
        query = q[:, start:stop].astype(acc).reshape(batch, t, heads, groups, dim)
        grad = dout[:, start:stop].astype(acc).reshape(batch, t, heads, groups, -1)
        logits = np.einsum("bthgd,bthsd->bthgs", query, keys, optimize=True) * acc(scale)
        mask = valid[..., None, :]
        masked = np.where(mask, logits, -np.inf)
        top = masked.max(-1, keepdims=True)
        any_valid = np.isfinite(top)
        top = np.where(any_valid, top, 0)
        ex = np.where(mask, np.exp(masked - top), 0)
        denom = ex.sum(-1, keepdims=True)
        prob = np.where(any_valid, ex / np.where(denom > 0, denom, 1), 0)
        dprob = np.einsum("bthgv,bthsv->bthgs", grad, values, optimize=True)
        dvals = np.einsum("bthgs,bthgv->bthsv", prob, grad, optimize=True)
        dlogit = prob * (dprob - (prob * dprob).sum(-1, keepdims=True))
        dquery = np.einsum("bthgs,bthsd->bthgd", dlogit, keys, optimize=True) * acc(scale)
        dkeys = np.einsum("bthgs,bthgd->bthsd", dlogit, query, optimize=True) * acc(scale)
        dq[:, start:stop] = dquery.reshape(batch, t, q_heads, dim)
        bb = np.broadcast_to(b_idx, tokens.shape)
        hh = np.broadcast_to(h_idx, tokens.shape)
        np.add.at(dk, (bb, tokens, hh), np.where(valid[..., None], dkeys, 0))
        np.add.at(dv, (bb, tokens, hh), np.where(valid[..., None], dvals, 0))
    return dq, dk, dv


# ----------------------------------------------------------------------------
# comparison helpers used by the parity tests
# ----------------------------------------------------------------------------

def compare_selection(got, expected, min_gap, rel_tol=1e-3):
    """Tie-aware comparison of [..., K] id sets against the oracle's selection.

    ``min_gap`` is the oracle trace's smallest relative K-boundary gap over all
    levels of each row's descent.  A row may differ from ``expected`` only if
    that gap is within ``rel_tol`` (a near-tie that ordinary float
    re-association can flip).  Ids are compared as sets.
    Returns (n_rows, n_exact, n_tie_explained, bad_row_indices).
    """
    k = got.shape[-1]
    got = np.sort(np.asarray(got).reshape(-1, k), -1)
    expected = np.sort(np.asarray(expected).reshape(-1, k), -1)
    gap = np.asarray(min_gap).reshape(-1)
    same = (got == expected).all(-1)
    tie = ~same & (gap <= rel_tol)
    bad = np.nonzero(~same & ~tie)[0]
    return got.shape[0], int(same.sum()), int(tie.sum()), bad
