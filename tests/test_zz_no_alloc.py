"""The no-allocation backward entry point, checked against the regular one.

pisa_sparse_attn_bwd_noalloc serves callers that cannot allocate device
memory (a host runtime bound to the C ABI that owns only the tensors it
passes, or a framework with a fixed device-memory plan): it keeps its dK/dV
accumulators in a fixed 32 MiB array inside the library instead of a caller
workspace.  This file runs last so that a stop-at-first-failure run has
already run every other test.
"""

import ctypes

import pytest
import torch

from nlogn_pisa_b200 import _lib
from nlogn_pisa_b200.attention import attention_backward, attention_forward

# gradient tolerance of the attention tests (bf16 inputs, fp32 accumulation)
ATOL = 3e-2


def _noalloc_backward(q, k, v, out, dout, lse, ids, block_size, scale):
    lib = _lib.lib()
    B, T, Hq, D = q.shape
    H, N, Dv = k.shape[2], k.shape[1], v.shape[-1]
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    torch.cuda.synchronize(q.device)
    free0, allocated0 = torch.cuda.mem_get_info(q.device)[0], torch.cuda.memory_allocated(q.device)
    with torch.cuda.device(q.device):
        rc = lib.pisa_sparse_attn_bwd_noalloc(
            _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), _lib.ptr(dout), _lib.ptr(lse), _lib.ptr(ids),
            ids.element_size(), None, 0, _lib.dtype_code(q), B, T, Hq, H, D, Dv, N, ids.shape[-1], block_size,
            float(scale), 1, _lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv), _lib.stream_of(q.device))
        _lib.check(rc)
        torch.cuda.synchronize(q.device)
    # device memory (the process-wide free count and torch's allocator) is
    # unchanged across the call, apart from the one-time set-up of a first call
    memory = (torch.cuda.mem_get_info(q.device)[0] - free0, torch.cuda.memory_allocated(q.device) - allocated0)
    return (dq, dk, dv), memory


@pytest.mark.gpu
def test_noalloc_backward_matches_workspace_backward(cuda_device):
    torch.manual_seed(7)
    B, N, Hq, H, D, C, S = 2, 700, 8, 2, 64, 32, 8
    dt = torch.bfloat16
    q = torch.randn(B, N, Hq, D, device=cuda_device).to(dt)
    k = torch.randn(B, N, H, D, device=cuda_device).to(dt)
    v = torch.randn(B, N, H, D, device=cuda_device).to(dt)
    dout = torch.randn(B, N, Hq, D, device=cuda_device).to(dt)
    # causal block choices: each row picks S distinct blocks at or before its own
    pos = torch.arange(N, device=cuda_device)
    scores = torch.rand(B, N, H, (N + C - 1) // C, device=cuda_device)
    scores = scores.masked_fill(torch.arange(scores.shape[-1], device=cuda_device) * C > pos[None, :, None, None], -1.0)
    ids = scores.topk(S, dim=-1).indices
    ids = torch.where(torch.gather(scores, -1, ids) < 0, torch.full_like(ids, -1), ids).contiguous()
    scale = D ** -0.5
    out, lse = attention_forward(q, k, v, ids, C, scale, None, 0, True)
    ref = attention_backward(q, k, v, out, dout, lse, ids, C, scale, None, 0, True)
    # two calls in a row: the second sees the first call's leftovers in the shared array
    for call in range(2):
        got, memory = _noalloc_backward(q, k, v, out, dout, lse, ids, C, scale)
        if call == 1:
            assert memory == (0, 0), memory
        for name, g, r in zip(("dq", "dk", "dv"), got, ref):
            assert torch.isfinite(g.float()).all(), name
            torch.testing.assert_close(g.float(), r.float(), atol=ATOL, rtol=0, msg=name)


@pytest.mark.gpu
def test_noalloc_backward_rejects_shapes_above_its_scratch(cuda_device):
    lib = _lib.lib()
    cap = lib.pisa_sparse_attn_bwd_noalloc_max_bytes()
    assert cap == 32 << 20
    # N*H*(D+Dv)*4 bytes above the cap: refused before any device work
    N = cap // (4 * 8 * 256) + 64
    rc = lib.pisa_sparse_attn_bwd_noalloc(None, None, None, None, None, None, None, 8, None, 0, _lib.BF16,
                                          1, 1, 32, 8, 128, 128, N, 32, 64, 0.1, 1, None, None, None,
                                          ctypes.c_void_p(0))
    assert rc == _lib.ERR_UNSUPPORTED
    assert "scratch" in lib.pisa_last_error().decode()
    # the limit is pisa_sparse_attn_bwd_workspace_bytes <= the scratch size, exactly
    per_token = lib.pisa_sparse_attn_bwd_workspace_bytes(1, 1, 32, 8, 128, 128, 1024) // 1024
    fits = cap // per_token
    assert lib.pisa_sparse_attn_bwd_workspace_bytes(1, 1, 32, 8, 128, 128, fits) <= cap
    assert lib.pisa_sparse_attn_bwd_workspace_bytes(1, 1, 32, 8, 128, 128, fits + 1) > cap
    rc = lib.pisa_sparse_attn_bwd_noalloc(None, None, None, None, None, None, None, 8, None, 0, _lib.BF16,
                                          1, 1, 32, 8, 128, 128, fits + 1, 32, 64, 0.1, 1, None, None, None,
                                          ctypes.c_void_p(0))
    assert rc == _lib.ERR_UNSUPPORTED
