"""Tensor-core attention backward against the oracle and the gather backward.

The tensor-core path (fp16/bf16, block size 64, head_dim 64) runs when the
caller passes pisa_sparse_attn_bwd_tc_workspace_bytes(...) bytes; the
per-query gather kernels run with the smaller workspace.  Both are checked
against the oracle's analytic gradient of the masked softmax
(sparse_attn_torch.py:6-35 under autograd) on arbitrary ids: -1, duplicates,
blocks past the causal edge, a tail block (N % 64 != 0), query offsets.
"""

import numpy as np
import pytest
import torch

import pisa_oracle as O

pytestmark = pytest.mark.gpu


def _run_backward(q, k, v, ids, C, offset, causal, tensor_core):
    from nlogn_pisa_b200 import _lib
    from nlogn_pisa_b200.attention import attention_forward
    from nlogn_pisa_b200.validation import query_positions

    positions, off = query_positions(q, k, offset)
    scale = q.shape[-1] ** -0.5
    out, lse = attention_forward(q, k, v, ids, C, scale, positions, off, causal)
    g = torch.Generator(device=q.device).manual_seed(99)
    dout = torch.randn(out.shape, generator=g, device=q.device).to(q.dtype)
    lib = _lib.lib()
    B, T, Hq, D = q.shape
    H, N, Dv = k.shape[2], k.shape[1], v.shape[-1]
    code = _lib.dtype_code(q)
    tc_bytes = lib.pisa_sparse_attn_bwd_tc_workspace_bytes(B, T, Hq, H, D, Dv, N, ids.shape[-1], C, code)
    if tensor_core:
        assert tc_bytes > 0
        ws_bytes = tc_bytes
    else:
        ws_bytes = lib.pisa_sparse_attn_bwd_workspace_bytes(B, T, Hq, H, D, Dv, N)
        assert ws_bytes < tc_bytes
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    _lib.check(lib.pisa_sparse_attn_bwd(
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), _lib.ptr(dout), _lib.ptr(lse), _lib.ptr(ids),
        ids.element_size(), _lib.ptr(positions), off, code, B, T, Hq, H, D, Dv, N, ids.shape[-1], C, float(scale),
        int(causal), _lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv), _lib.ptr(ws), ws_bytes, _lib.stream_of(q.device)))
    if tensor_core:
        _lib.check_workspace(ws, q.device)
    return (dq, dk, dv), dout


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [
    # B, T, N, Hq, H, S, causal, offset
    (1, 1500, 1500, 4, 1, 8, True, None),
    (2, 700, 1000, 8, 2, 12, True, 300),
    (1, 900, 900, 16, 16, 16, False, None),
    (1, 1200, 1337, 2, 2, 6, True, 137),
])
def test_tensor_core_backward_matches_oracle(cuda_device, dtype, shape):
    B, T, N, Hq, H, S, causal, offset = shape
    C, D = 64, 64
    g = torch.Generator().manual_seed(sum(shape[:6]))
    q = torch.randn(B, T, Hq, D, generator=g).to(dtype).cuda()
    k = torch.randn(B, N, H, D, generator=g).to(dtype).cuda()
    v = torch.randn(B, N, H, D, generator=g).to(dtype).cuda()
    blocks = -(-N // C)
    ids = torch.randint(-1, blocks + 1, (B, T, H, S), generator=g)
    ids[..., 1] = ids[..., 0]                     # duplicates count twice
    ids = ids.cuda()
    (dq, dk, dv), dout = _run_backward(q, k, v, ids, C, offset, causal, tensor_core=True)
    pos = O.query_positions(B, T, N, offset)
    want = O.sparse_attention_backward(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                                       ids.cpu().numpy(), C, dout.float().cpu().numpy(), positions=pos,
                                       causal=causal)
    for got, ref, name in zip((dq, dk, dv), want, ("dq", "dk", "dv")):
        np.testing.assert_allclose(got.float().cpu().numpy(), ref, rtol=1e-2, atol=3e-2, err_msg=name)
    # and against the gather backward on the same inputs
    (gq, gk, gv), _ = _run_backward(q, k, v, ids, C, offset, causal, tensor_core=False)
    for a, b, name in zip((dq, dk, dv), (gq, gk, gv), ("dq", "dk", "dv")):
        torch.testing.assert_close(a.float(), b.float(), rtol=1e-2, atol=3e-2, msg=name)


def test_autograd_takes_tensor_core_backward(cuda_device):
    """sparse_attention's autograd at the training shape family (G=1, D=64, C=64)."""
    import nlogn_pisa_b200 as P

    g = torch.Generator(device=cuda_device).manual_seed(8)
    B, N, H, D, C, K = 2, 2048, 4, 64, 64, 16
    q = torch.randn(B, N, H, D, generator=g, device=cuda_device).to(torch.bfloat16).requires_grad_(True)
    k = torch.randn(B, N, H, D, generator=g, device=cuda_device).to(torch.bfloat16).requires_grad_(True)
    v = torch.randn(B, N, H, D, generator=g, device=cuda_device).to(torch.bfloat16).requires_grad_(True)
    ids = P.select_blocks(q.detach(), k.detach(), method="pisa2", block_size=C, topk=K, force_recent=1)
    out = P.sparse_attention(q, k, v, ids, block_size=C)
    dout = torch.randn(out.shape, generator=g, device=cuda_device).to(torch.bfloat16)
    out.backward(dout)
    want = O.sparse_attention_backward(q.detach().float().cpu().numpy(), k.detach().float().cpu().numpy(),
                                       v.detach().float().cpu().numpy(), ids.cpu().numpy(), C,
                                       dout.float().cpu().numpy(), positions=O.query_positions(B, N, N))
    for got, ref, name in zip((q.grad, k.grad, v.grad), want, ("dq", "dk", "dv")):
        np.testing.assert_allclose(got.float().cpu().numpy(), ref, rtol=1e-2, atol=3e-2, err_msg=name)
