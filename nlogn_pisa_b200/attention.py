"""Attention over selected key blocks (forward + backward) on the CUDA library.

Drop-in mirror of sparse_attention / sparse_attn_fn
(pisa/pisa/ops/flash_sparse_attn/sparse_attn/sparse_attn.py:10-61) with the
semantics of its torch path (sparse_attn_torch.py:6-35): one softmax over the
union of the selected blocks' keys, causal inside blocks, rows without a
visible key give 0.  Differentiable in q, k and v through
pisa_sparse_attn_fwd / pisa_sparse_attn_bwd.
"""

from __future__ import annotations

import torch

from . import _lib
from .validation import packed_queries, query_positions, require_cuda, validate_qkv


def _rows16(t):
    vec = 16 // t.element_size()
    ok = (t.stride(-1) == 1 and t.data_ptr() % 16 == 0
          and all(s % vec == 0 for s in t.stride()[:-1]) and t.shape[-1] % vec == 0)
    return t if ok else t.contiguous()


def attention_forward(q, k, v, indices, block_size, scale, positions, offset, causal):
    """(out [B,Tq,Hq,Dv] q.dtype, lse [B,Tq,Hq] fp32) through pisa_sparse_attn_fwd."""
    code = _lib.dtype_code(q)
    q, k, v = _rows16(q), _rows16(k), _rows16(v)
    indices = indices.contiguous()
    batch, tokens, q_heads, dim = q.shape
    heads, length, dim_v = k.shape[2], k.shape[1], v.shape[-1]
    out = torch.empty((batch, tokens, q_heads, dim_v), dtype=q.dtype, device=q.device)
    lse = torch.empty((batch, tokens, q_heads), dtype=torch.float32, device=q.device)
    library = _lib.lib()
    ws_bytes = library.pisa_sparse_attn_fwd_workspace_bytes(
        batch, tokens, q_heads, heads, dim, dim_v, length, indices.shape[-1], block_size, code)
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
    with torch.cuda.device(q.device):
        _lib.check(library.pisa_sparse_attn_fwd(
            _lib.ptr(q), *q.stride()[:3], _lib.ptr(k), *k.stride()[:3], _lib.ptr(v), *v.stride()[:3],
            _lib.ptr(indices), indices.element_size(), _lib.ptr(positions), offset, code, batch,
            tokens, q_heads, heads, dim, dim_v, length, indices.shape[-1], block_size, float(scale),
            int(bool(causal)), _lib.ptr(out), _lib.ptr(lse), _lib.ptr(workspace), ws_bytes,
            _lib.stream_of(q.device)))
    if _lib.status_checks():
        _lib.check_workspace(workspace, q.device)
    return out, lse


def attention_backward(q, k, v, out, dout, lse, indices, block_size, scale, positions, offset, causal):
    code = _lib.dtype_code(q)
    q, k, v, out, dout = (x.contiguous() for x in (q, k, v, out, dout))
    indices = indices.contiguous()
    batch, tokens, q_heads, dim = q.shape
    heads, length, dim_v = k.shape[2], k.shape[1], v.shape[-1]
    library = _lib.lib()
    # the tensor-core backward when the shapes allow it, else the gather kernels
    ws = library.pisa_sparse_attn_bwd_tc_workspace_bytes(batch, tokens, q_heads, heads, dim, dim_v, length,
                                                         indices.shape[-1], block_size, code)
    tensor_core = ws > 0
    if not tensor_core:
        ws = library.pisa_sparse_attn_bwd_workspace_bytes(batch, tokens, q_heads, heads, dim, dim_v, length)
    workspace = torch.empty(ws, dtype=torch.uint8, device=q.device)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    with torch.cuda.device(q.device):
        _lib.check(library.pisa_sparse_attn_bwd(
            _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), _lib.ptr(dout), _lib.ptr(lse),
            _lib.ptr(indices), indices.element_size(), _lib.ptr(positions), offset, code, batch,
            tokens, q_heads, heads, dim, dim_v, length, indices.shape[-1], block_size, float(scale),
            int(bool(causal)), _lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv), _lib.ptr(workspace), ws,
            _lib.stream_of(q.device)))
    if tensor_core and _lib.status_checks():
        _lib.check_workspace(workspace, q.device)
    return dq, dk, dv


class SparseAttentionFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, indices, block_size, scale, positions, offset, causal):
        out, lse = attention_forward(q, k, v, indices, block_size, scale, positions, offset, causal)
        ctx.save_for_backward(q, k, v, out, lse, indices, positions)
        ctx.args = (block_size, scale, offset, causal)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse, indices, positions = ctx.saved_tensors
        block_size, scale, offset, causal = ctx.args
        dq, dk, dv = attention_backward(q, k, v, out, dout, lse, indices, block_size, scale,
                                        positions, offset, causal)
        return dq, dk, dv, None, None, None, None, None, None


def sparse_attention(q, k, v, indices, block_size=64, scale=None, cu_seqlens=None, query_offset=None,
                     backend="auto", causal=True):
    """Attention over the selected blocks ``indices`` [B,Tq,Hkv,S] (int32 or int64)."""
    validate_qkv(q, k, v)
    if indices.ndim != 4 or indices.shape[:3] != (*q.shape[:2], k.shape[2]):
        raise ValueError("indices must have shape [B,Tq,Hkv,K]")
    if indices.dtype not in (torch.int32, torch.int64) or indices.device != q.device:
        raise ValueError("indices must be integers on the query device")
    if block_size < 1 or backend not in ("torch", "auto", "triton", "fla", "cuda"):
        raise ValueError("invalid block_size or attention backend")
    require_cuda(q, k, v)
    _lib.dtype_code(q)
    scale = k.shape[-1] ** -0.5 if scale is None else scale
    if cu_seqlens is not None:
        outputs = [
            sparse_attention(q[:, qs:qe], k[:, ks:ke], v[:, ks:ke], indices[:, qs:qe], block_size,
                             scale, query_offset=offset, backend=backend, causal=causal)
            for qs, qe, ks, ke, offset in packed_queries(q, k, cu_seqlens, query_offset)
        ]
        return torch.cat(outputs, 1)
    positions, offset = query_positions(q, k, query_offset)
    return SparseAttentionFunction.apply(q, k, v, indices, block_size, scale, positions, offset, causal)


sparse_attn_fn = sparse_attention
