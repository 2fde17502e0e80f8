"""Block selection, mean pooling and pyramids on the CUDA library.

Drop-in mirrors of the reference operators (paths relative to the
Aphelios-Tang/NlogN_PISA project):
  select_blocks / top_k_pyramid_fn -> pisa/pisa/ops/flash_sparse_attn/top_k_pyramid/top_k_pyramid.py:11-122
  routing_geometry                 -> top_k_pyramid_torch.py:124-133
  mean_pool / build_pyramid        -> pisa/pisa/ops/compress/mean_pooling/mean_pooling.py:8-52
  bsa_fn (select_blocks "bsa")     -> pisa/pisa/ops/flash_sparse_attn/bsa/bsa.py:9-52, bsa_torch.py:63-106
Same argument names, defaults and ValueError contract; every computation runs
in libpisa_b200 (no Triton, no CPU fallback).  ``branching`` (default 2, the
reference's only value) additionally allows a 4-ary pyramid.
"""

from __future__ import annotations

import torch

from . import _lib
from .layout import check_level_sizes, full_level_sizes, level_sizes
from .validation import packed_queries, query_positions, require_cuda, validate_qkv


def routing_geometry(blocks, topk, branching=2):
    """(top, first_width): levels descended and the first network width."""
    top = 0
    while blocks > topk:
        parent = -(-blocks // branching)
        if parent < topk or parent == blocks:
            break
        blocks = parent
        top += 1
    return top, max(16, 1 << (max(blocks, topk) - 1).bit_length())


def _rows16(t):
    """t itself when its rows are 16-byte aligned with a unit last stride, else a contiguous copy."""
    vec = 16 // t.element_size()
    ok = (t.stride(-1) == 1 and t.data_ptr() % 16 == 0
          and all(s % vec == 0 for s in t.stride()[:-1]) and t.shape[-1] % vec == 0)
    return t if ok else t.contiguous()


_c_array = _lib.int64_array


def mean_pool(keys, size, *, backend="auto", fp32_accumulation=False):
    """Mean over the valid tokens of each ``size`` block (tail divides by its count).

    Accumulates in fp32 for every input (the reference's torch path does; its
    Triton path does so when ``fp32_accumulation``), forward only.
    """
    if size < 1:
        raise ValueError("pool size must be positive")
    if backend not in ("auto", "torch", "triton", "cuda"):
        raise ValueError("pooling backend must be auto, torch, or triton")
    require_cuda(keys)
    if keys.ndim != 4 or not keys.numel():
        raise ValueError("pooling requires a positive size and nonempty [B,N,H,D] input")
    if torch.is_grad_enabled() and keys.requires_grad:
        raise ValueError("CUDA pooling does not support gradients")
    code = _lib.dtype_code(keys)
    keys = _rows16(keys)
    batch, length, heads, dim = keys.shape
    blocks = -(-length // size)
    out = torch.empty((batch, blocks, heads, dim), device=keys.device, dtype=keys.dtype)
    with torch.cuda.device(keys.device):
        _lib.check(_lib.lib().pisa_mean_pool(
            _lib.ptr(keys), code, batch, length, heads, dim, *keys.stride()[:3], size,
            _lib.ptr(out), _lib.stream_of(keys.device)))
    return out


def build_pyramid(keys, block_size, *, backend="auto", max_level=None, branching=2):
    """Leaf means first, then pools of ``branching`` up to the root or ``max_level``.

    All levels share one storage allocation; the returned tensors are views.
    """
    if max_level is not None and (type(max_level) is not int or max_level < 0):
        raise ValueError("max_level must be a nonnegative integer or None")
    if block_size < 1:
        raise ValueError("pool size must be positive")
    if backend not in ("auto", "torch", "triton", "cuda"):
        raise ValueError("pooling backend must be auto, torch, or triton")
    require_cuda(keys)
    if keys.ndim != 4 or not keys.numel():
        raise ValueError("pooling requires a positive size and nonempty [B,N,H,D] input")
    if torch.is_grad_enabled() and keys.requires_grad:
        raise ValueError("CUDA pooling does not support gradients")
    code = _lib.dtype_code(keys)
    keys = _rows16(keys)
    batch, length, heads, dim = keys.shape
    sizes = full_level_sizes(-(-length // block_size), branching)
    if max_level is not None:
        sizes = sizes[:max_level + 1]
    offsets = [0]
    for s in sizes[:-1]:
        offsets.append(offsets[-1] + s)
    total = offsets[-1] + sizes[-1]
    storage = torch.empty((batch, total, heads, dim), device=keys.device, dtype=keys.dtype)
    with torch.cuda.device(keys.device):
        _lib.check(_lib.lib().pisa_build_pyramid(
            _lib.ptr(keys), code, batch, length, heads, dim, *keys.stride()[:3], block_size,
            branching, len(sizes), _lib.ptr(storage), storage.stride(0), _c_array(offsets),
            _lib.stream_of(keys.device)))
    return [storage[:, o:o + s] for o, s in zip(offsets, sizes)]


@torch.no_grad()
def select_blocks(q, k, method="pisa", block_size=64, topk=8, cu_seqlens=None, query_offset=None,
                  force_first=True, force_recent=2, backend="auto", pyramid=None, leaf_tile=4,
                  routing_schedule="auto", branching=2):
    """Return block ids [B,Tq,Hkv,K] int64 in network-rank order, padded by -1.

    Arguments as the reference's select_blocks.  Ids are document-relative
    under ``cu_seqlens``; slot order follows the comparison network; required
    blocks (first, and the ``force_recent`` most recent) count toward K.
    """
    validate_qkv(q, k)
    if method not in ("bsa", "pisa1", "pisa2", "pisa"):
        raise ValueError("method must be bsa, pisa1, pisa2 or pisa")
    if backend not in ("torch", "triton", "auto", "cuda"):
        raise ValueError("backend must be torch, triton or auto")
    if leaf_tile not in (1, 2, 4):
        raise ValueError("leaf_tile must be 1, 2 or 4")
    if routing_schedule not in ("auto", "grouped", "fused"):
        raise ValueError("routing_schedule must be auto, grouped or fused")
    if block_size < 1 or topk < 1 or force_recent < 0:
        raise ValueError("positive block_size/topk and nonnegative force_recent required")
    if method != "bsa" and force_recent == 0:
        raise ValueError("causal pyramid routing requires force_recent >= 1")
    if method == "bsa":
        return bsa_fn(q, k, block_size, topk, cu_seqlens=cu_seqlens, query_offset=query_offset,
                      force_first=force_first, force_recent=force_recent, backend=backend)
    if branching not in (2, 4):
        raise ValueError("branching must be 2 or 4")
    if routing_schedule == "auto":
        grouped = method != "pisa1" and (q.shape[1] == k.shape[1] or (cu_seqlens is None and q.shape[1] > 1))
        routing_schedule = "grouped" if grouped else "fused"
        if grouped:
            leaf_tile = 4
    if cu_seqlens is not None:
        segments = list(packed_queries(q, k, cu_seqlens, query_offset))
        blocks = max((ke - ks + block_size - 1) // block_size for _, _, ks, ke, _ in segments)
        geometry = routing_geometry(blocks, topk, branching) if routing_schedule == "fused" else None
        pieces = [
            _select_unpacked(q[:, qs:qe], k[:, ks:ke], method, block_size, topk, offset, force_first,
                             force_recent, None, leaf_tile, routing_schedule, geometry, branching)
            for qs, qe, ks, ke, offset in segments
        ]
        return torch.cat(pieces, 1)
    return _select_unpacked(q, k, method, block_size, topk, query_offset, force_first, force_recent,
                            pyramid, leaf_tile, routing_schedule, None, branching)


def _pyramid_tables(pyramid, k, block_size, top, branching):
    """(storage, batch_stride, offsets, sizes) for a caller-supplied pyramid, or Nones.

    The level sizes must be those of ``k``'s keys for this block size and
    branching (a binary pyramid queried with branching 4, or a pyramid of
    other keys, raises ValueError instead of routing over the wrong tree).
    """
    if pyramid is None:
        return None, 0, None, None
    if hasattr(pyramid, "storage"):
        storage = pyramid.storage
        sizes = [int(x) for x in pyramid.level_sizes]
        starts = getattr(pyramid, "starts", None)
        offsets = list(starts) if starts is not None else [int(x) for x in pyramid.offsets.tolist()]
        if len(offsets) < len(sizes):
            raise ValueError("pyramid offsets must cover every level")
        _check_summary(storage, k)
        check_level_sizes(sizes, k.shape[1], block_size, branching, top + 1)
        return _rows16_storage(storage), storage.stride(0), offsets[:len(sizes)], sizes
    levels = list(pyramid.levels if hasattr(pyramid, "levels") else pyramid)
    if not levels:
        raise ValueError("pyramid has no levels")
    for level in levels:
        _check_summary(level, k)
    sizes = [x.shape[1] for x in levels]
    check_level_sizes(sizes, k.shape[1], block_size, branching, top + 1)
    levels = levels + [levels[-1]] * max(0, top + 1 - len(levels))
    summary = torch.cat(levels, dim=1).contiguous()
    sizes = [x.shape[1] for x in levels]
    offsets = [0]
    for s in sizes[:-1]:
        offsets.append(offsets[-1] + s)
    return summary, summary.stride(0), offsets, sizes


def _rows16_storage(storage):
    if (storage.stride(-1) != 1 or storage.stride(-2) != storage.shape[-1]
            or storage.stride(1) != storage.shape[-1] * storage.shape[-2]):
        raise ValueError("pyramid storage must be contiguous per node ([B, total, H, D])")
    return storage


def _check_summary(t, k):
    if (t.ndim != 4 or t.shape[0] != k.shape[0] or t.shape[2:] != k.shape[2:] or t.dtype != k.dtype
            or t.device != k.device):
        raise ValueError("pyramid levels must be [B, nodes, Hkv, D] tensors like the keys")


def _select_unpacked(q, k, method, block_size, topk, query_offset, force_first, force_recent,
                     pyramid, leaf_tile, routing_schedule, geometry, branching):
    require_cuda(q, k)
    code = _lib.dtype_code(q)
    if topk & (topk - 1) or block_size & (block_size - 1) or not 8 <= topk <= 64 or block_size < 16:
        raise ValueError("GPU routing requires power-of-two block_size >= 16 and topk in {8,16,32,64}")
    blocks = -(-k.shape[1] // block_size)
    if topk < min(blocks, force_recent + int(force_first)):
        raise ValueError("topk cannot hold all required blocks")
    positions, offset = query_positions(q, k, query_offset)
    top, first_width = geometry or routing_geometry(blocks, topk, branching)
    q = _rows16(q)
    k = _rows16(k)
    batch, tokens, q_heads, dim = q.shape
    heads, length = k.shape[2], k.shape[1]
    summary, summary_sb, offsets, sizes = _pyramid_tables(pyramid, k, block_size, top, branching)
    schedule = _lib.SCHEDULES[routing_schedule]
    library = _lib.lib()
    ws_bytes = library.pisa_select_workspace_bytes(
        batch, tokens, q_heads, heads, dim, length, code, _lib.METHODS[method], block_size, branching,
        topk, top, first_width, schedule, 1 if summary is None else 0)
    workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    out = torch.empty((batch, tokens, heads, topk), dtype=torch.int64, device=q.device)
    with torch.cuda.device(q.device):
        _lib.check(library.pisa_select_blocks(
            _lib.ptr(q), *q.stride()[:3], _lib.ptr(k), *k.stride()[:3],
            _lib.ptr(summary), summary_sb,
            _c_array(offsets) if offsets else None, _c_array(sizes) if sizes else None,
            len(sizes) if sizes else 0, _lib.ptr(positions), offset, code, batch, tokens, q_heads,
            heads, dim, length, _lib.METHODS[method], block_size, branching, topk,
            int(bool(force_first)), force_recent, top, first_width, schedule, _lib.ptr(out),
            _lib.ptr(workspace), ws_bytes, _lib.stream_of(q.device)))
    if _lib.status_checks():
        _lib.check_workspace(workspace, q.device)
    return out


@torch.no_grad()
def grouped_leaf_scores(q, k, candidates, block_size, method, tile_size=4, *, positions=None, topk=None,
                        force_first=True, force_recent=2, leaf_means=None, num_warps=None,
                        num_stages=None):
    """FP32 leaf scores [B,Tq,Hkv,W] in the order of ``candidates`` (-inf where unscored).

    Arguments as the reference's grouped_leaf_scores.  ``tile_size``,
    ``num_warps`` and ``num_stages`` are accepted for compatibility (the
    bucketed tensor-core scorer packs 128/G requests per tile whatever they
    are).  With ``positions`` ([B,Tq] or broadcastable int64), ids past the
    query's position, forced ids and rows whose valid ids all fit in
    ``topk`` are not scored.
    """
    validate_qkv(q, k)
    require_cuda(q, k)
    if q.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError("grouped leaf scoring supports FP16, BF16 and FP32")
    if method not in ("pisa1", "pisa2", "pisa") or tile_size not in (1, 2, 4):
        raise ValueError("expected method pisa1/pisa2/pisa and tile_size 1/2/4")
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    if candidates.ndim != 4 or candidates.shape[:3] != (*q.shape[:2], k.shape[2]):
        raise ValueError("candidates must have shape [B,Tq,Hkv,W]")
    if candidates.dtype not in (torch.int32, torch.int64) or candidates.device != q.device:
        raise ValueError("candidates must use an integer dtype on the query device")
    if positions is not None:
        if method != "pisa1" and topk is None:
            raise ValueError("topk is required with positions for pisa and pisa2")
        positions = torch.broadcast_to(positions.to(device=q.device, dtype=torch.int64),
                                       q.shape[:2]).contiguous()
    code = _lib.dtype_code(q)
    q, k = _rows16(q), _rows16(k)
    candidates = candidates.contiguous()
    batch, tokens, q_heads, dim = q.shape
    heads, length, width = k.shape[2], k.shape[1], candidates.shape[-1]
    means_sb = 0
    if leaf_means is not None and method == "pisa1":
        blocks = -(-length // block_size)
        if (leaf_means.shape[0] != batch or leaf_means.shape[1] < blocks or leaf_means.shape[2:] != k.shape[2:]
                or leaf_means.dtype != q.dtype or leaf_means.device != q.device):
            raise ValueError("leaf_means must be [B, blocks, Hkv, D] like the keys")
        if leaf_means.stride(-1) != 1 or leaf_means.stride(-2) != dim or leaf_means.stride(1) != heads * dim:
            leaf_means = leaf_means.contiguous()
        means_sb = leaf_means.stride(0)
    else:
        leaf_means = None
    library = _lib.lib()
    ws_bytes = library.pisa_leaf_scores_workspace_bytes(batch, tokens, q_heads, heads, dim, length, width, code,
                                                        _lib.METHODS[method], block_size, int(leaf_means is not None))
    workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    out = torch.empty(candidates.shape, dtype=torch.float32, device=q.device)
    with torch.cuda.device(q.device):
        _lib.check(library.pisa_leaf_scores(
            _lib.ptr(q), *q.stride()[:3], _lib.ptr(k), *k.stride()[:3], _lib.ptr(leaf_means), means_sb,
            _lib.ptr(candidates), candidates.element_size(), _lib.ptr(positions), code, batch, tokens,
            q_heads, heads, dim, length, width, _lib.METHODS[method], block_size,
            -1 if topk is None else int(topk), int(bool(force_first)), int(force_recent), _lib.ptr(out),
            _lib.ptr(workspace), ws_bytes, _lib.stream_of(q.device)))
    if _lib.status_checks():
        _lib.check_workspace(workspace, q.device)
    return out


top_k_pyramid_fn = select_blocks


@torch.no_grad()
def bsa_fn(q, k, block_size=64, topk=8, *, cu_seqlens=None, query_offset=None, force_first=True,
           force_recent=2, backend="auto"):
    """Flat BSA block ids [B,Tq,Hkv,K] int64 in network-rank order, -1 padded.

    Arguments as the reference's bsa_fn.  Every complete block is scored by
    the softmax probability of its leaf mean under each query head, summed
    over the KV head's query heads; required blocks (first, and the
    ``force_recent`` most recent) score 1 per head.  Results follow the
    reference's torch semantics (bsa_torch.py:63-106) on the CUDA library for
    every backend name; packed documents are selected one by one with
    document-relative ids.
    """
    validate_qkv(q, k)
    if backend not in ("torch", "triton", "auto", "cuda"):
        raise ValueError("backend must be torch, triton or auto")
    if block_size < 1 or topk < 1 or force_recent < 0:
        raise ValueError("positive block_size/topk and nonnegative force_recent required")
    if cu_seqlens is not None:
        segments = list(packed_queries(q, k, cu_seqlens, query_offset))
        return torch.cat([_bsa_unpacked(q[:, qs:qe], k[:, ks:ke], block_size, topk, offset, force_first,
                                        force_recent) for qs, qe, ks, ke, offset in segments], dim=1)
    return _bsa_unpacked(q, k, block_size, topk, query_offset, force_first, force_recent)


def bsa_required_blocks(last_position, block_size, force_first, force_recent):
    """Distinct required blocks of the row at ``last_position`` (the most of any row)."""
    current = last_position // block_size
    return min(force_recent, current + 1) + int(bool(force_first) and current >= force_recent)


def _bsa_unpacked(q, k, block_size, topk, query_offset, force_first, force_recent):
    require_cuda(q, k)
    code = _lib.dtype_code(q)
    positions, offset = query_positions(q, k, query_offset)
    last = offset + q.shape[1] - 1 if positions is None else int(positions.max())
    if bsa_required_blocks(last, block_size, force_first, force_recent) > topk:
        raise ValueError("topk is smaller than the number of required distinct blocks")
    q, k = _rows16(q), _rows16(k)
    batch, tokens, q_heads, dim = q.shape
    heads, length = k.shape[2], k.shape[1]
    library = _lib.lib()
    ws_bytes = library.pisa_bsa_workspace_bytes(batch, length, heads, dim, code, block_size, 0)
    workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    out = torch.empty((batch, tokens, heads, topk), dtype=torch.int64, device=q.device)
    with torch.cuda.device(q.device):
        _lib.check(library.pisa_bsa_select(
            _lib.ptr(q), *q.stride()[:3], _lib.ptr(k), *k.stride()[:3], None, 0, _lib.ptr(positions), offset,
            code, batch, tokens, q_heads, heads, dim, length, block_size, topk, int(bool(force_first)),
            int(force_recent), _lib.ptr(out), _lib.ptr(workspace), ws_bytes, _lib.stream_of(q.device)))
    return out


@torch.no_grad()
def decode_select_attend(q, k, v, pyramid, method="pisa", block_size=64, topk=8, query_offset=None,
                         force_first=True, force_recent=2, scale=None, branching=2, return_lse=False):
    """One decode step in one launch: the block selection of
    ``select_blocks(..., routing_schedule="fused", pyramid=pyramid)`` and the
    attention of ``sparse_attention`` over those blocks (causal at each
    query's position), fused per (token, KV head).

    Returns ``(out [B,Tq,Hq,Dv], ids [B,Tq,Hkv,K])`` (and the fp32 lse when
    ``return_lse``).  ``pyramid`` is the cache's pyramid (a PyramidCache-like
    object or a list of levels) of ``k``.  Inference only, like the
    reference's decode attention (sparse_attn_fla.py:34-37).
    """
    validate_qkv(q, k)
    require_cuda(q, k, v)
    if method not in ("pisa1", "pisa2", "pisa"):
        raise ValueError("method must be pisa1, pisa2 or pisa")
    if block_size < 1 or topk < 1 or force_recent < 1:
        raise ValueError("positive block_size/topk and force_recent >= 1 required")
    if branching not in (2, 4):
        raise ValueError("branching must be 2 or 4")
    if topk & (topk - 1) or block_size & (block_size - 1) or not 8 <= topk <= 64 or block_size < 16:
        raise ValueError("GPU routing requires power-of-two block_size >= 16 and topk in {8,16,32,64}")
    if v.shape[:3] != k.shape[:3] or v.dtype != k.dtype or v.device != k.device:
        raise ValueError("values must be [B, N, Hkv, Dv] like the keys")
    if pyramid is None:
        raise ValueError("the fused decode step needs the key pyramid (a PyramidCache)")
    code = _lib.dtype_code(q)
    blocks = -(-k.shape[1] // block_size)
    if topk < min(blocks, force_recent + int(force_first)):
        raise ValueError("topk cannot hold all required blocks")
    positions, offset = query_positions(q, k, query_offset)
    top, first_width = routing_geometry(blocks, topk, branching)
    q, k, v = _rows16(q), _rows16(k), _rows16(v)
    batch, tokens, q_heads, dim = q.shape
    heads, length, dim_v = k.shape[2], k.shape[1], v.shape[-1]
    summary, summary_sb, offsets, sizes = _pyramid_tables(pyramid, k, block_size, top, branching)
    scale = dim ** -0.5 if scale is None else float(scale)
    ids = torch.empty((batch, tokens, heads, topk), dtype=torch.int64, device=q.device)
    out = torch.empty((batch, tokens, q_heads, dim_v), dtype=q.dtype, device=q.device)
    lse = torch.empty((batch, tokens, q_heads), dtype=torch.float32, device=q.device)
    with torch.cuda.device(q.device):
        _lib.check(_lib.lib().pisa_decode_select_attend(
            _lib.ptr(q), *q.stride()[:3], _lib.ptr(k), *k.stride()[:3], _lib.ptr(v), *v.stride()[:3],
            _lib.ptr(summary), summary_sb, _c_array(offsets), _c_array(sizes), len(sizes),
            _lib.ptr(positions), offset, code, batch, tokens, q_heads, heads, dim, dim_v, length,
            _lib.METHODS[method], block_size, branching, topk, int(bool(force_first)), force_recent, top,
            first_width, scale, _lib.ptr(ids), _lib.ptr(out), _lib.ptr(lse), _lib.stream_of(q.device)))
    return (out, ids, lse) if return_lse else (out, ids)
