"""Shape and sequence-boundary contracts of the public operators.

These restate the reference's argument contract (pisa/pisa/utils/validation.py)
so that callers get the same ValueError behaviour:
  * sequence_slices   -> validation.py:8-18
  * validate_qkv      -> validation.py:21-35
  * query_positions   -> validation.py:38-56
  * packed_queries    -> validation.py:59-81
"""

from __future__ import annotations

import torch


def sequence_slices(cu_seqlens, length):
    """[(start, end)] document ranges from cumulative lengths (one host read)."""
    if cu_seqlens is None:
        return [(0, length)]
    if cu_seqlens.ndim != 1 or cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise ValueError("cu_seqlens must be a one-dimensional integer tensor")
    bounds = [int(x) for x in cu_seqlens.detach().cpu().tolist()]
    if len(bounds) < 2 or bounds[0] != 0 or bounds[-1] != length:
        raise ValueError("cu_seqlens must start at zero and end at the key length")
    pairs = list(zip(bounds[:-1], bounds[1:]))
    if any(a >= b for a, b in pairs):
        raise ValueError("packed sequences must be nonempty and strictly ordered")
    return pairs


def validate_qkv(q, k, v=None):
    """q [B,Tq,Hq,D], k/v [B,N,H,D] with Hq a multiple of H, same dtype/device."""
    if q.ndim != 4 or k.ndim != 4:
        raise ValueError("q and k must have shape [batch, tokens, heads, head_dim]")
    if q.shape[0] != k.shape[0] or q.shape[-1] != k.shape[-1]:
        raise ValueError("q and k must share batch size and head dimension")
    if min(*q.shape, *k.shape) <= 0 or q.shape[2] % k.shape[2]:
        raise ValueError("nonempty tensors and a whole number of query heads per KV head are required")
    if q.device != k.device or q.dtype != k.dtype or not q.is_floating_point():
        raise ValueError("q and k must share a floating dtype and device")
    if v is not None and (v.ndim != 4 or v.shape[:3] != k.shape[:3] or v.device != k.device
                          or v.dtype != k.dtype):
        raise ValueError("v must share k's batch, length, heads, dtype and device")


def query_positions(q, k, query_offset=None):
    """Absolute positions of the queries.

    Returns (positions, offset): for a scalar (or default) offset, positions is
    None and offset the int -- the kernels then use offset + token without a
    device tensor or host sync.  Tensor offsets give an int64 [B, Tq] device
    tensor, bounds-checked on the host as the reference does.
    """
    if query_offset is None or isinstance(query_offset, int):
        offset = k.shape[1] - q.shape[1] if query_offset is None else int(query_offset)
        if offset < 0 or offset + q.shape[1] > k.shape[1]:
            raise ValueError("queries must refer to positions within their key sequence")
        return None, offset
    offset = torch.as_tensor(query_offset, device=q.device, dtype=torch.long)
    if offset.ndim > 1 or offset.numel() not in (1, q.shape[0]):
        raise ValueError("query_offset must be a scalar or one offset per batch element")
    positions = offset.reshape(-1, 1) + torch.arange(q.shape[1], device=q.device)
    positions = positions.expand(q.shape[0], -1).contiguous()
    if bool((positions < 0).any()) or bool((positions >= k.shape[1]).any()):
        raise ValueError("queries must refer to positions within their key sequence")
    return positions, 0


def packed_queries(q, k, cu_seqlens, query_offset=None):
    """Yield (q_start, q_end, k_start, k_end, local_offset) per packed document."""
    if q.shape[0] != 1:
        raise ValueError("packed inputs require batch size one")
    segments = sequence_slices(cu_seqlens, k.shape[1])
    if q.shape[1] == k.shape[1]:
        if query_offset is not None and bool(torch.as_tensor(query_offset).ne(0).any()):
            raise ValueError("packed prefill has local query_offset zero")
        for start, end in segments:
            yield start, end, start, end, 0
    elif q.shape[1] == len(segments):
        offsets = None if query_offset is None else torch.as_tensor(query_offset).reshape(-1)
        if offsets is not None and offsets.numel() not in (1, len(segments)):
            raise ValueError("packed decode needs a scalar or one offset per document")
        for index, (start, end) in enumerate(segments):
            offset = end - start - 1 if offsets is None else int(offsets[min(index, offsets.numel() - 1)])
            yield index, index + 1, start, end, offset
    else:
        raise ValueError("packed inputs support full prefill or one decode query per document")


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("nlogn_pisa_b200 runs on CUDA tensors only; there is no CPU path")
