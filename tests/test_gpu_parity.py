"""CUDA path against the reference's golden outputs and the numpy oracle."""

import numpy as np
import pytest
import torch

import pisa_oracle as O
from golden_cases import CASES, load, np_inputs, offset_arg

pytestmark = pytest.mark.gpu

GPU_CASES = [n for n, c in CASES.items() if c["dtype"] != "f64"]
# the GPU routing envelope (top_k_pyramid_triton.py:329-332): topk in {8,16,32,64}
SELECT_CASES = [n for n in GPU_CASES if CASES[n]["K"] >= 8]


def _cuda(*tensors):
    return [t.cuda() for t in tensors]


def _positions(case):
    return O.query_positions(case["B"], case["T"], case["N"], case.get("offset"))


def _trace(case, q, k, method, branching=2):
    trace = {}
    levels = O.build_pyramid(k, case["C"], case["dtype"], branching=branching)
    ids = O.pyramid_select(q, k, method, case["C"], case["K"], _positions(case), case["ff"], case["fr"],
                           levels, branching=branching, trace=trace)
    return ids, trace


def _check_ids(got, want, trace, min_exact=1.0):
    rows, exact, tie, bad = O.compare_selection(got, want, trace["min_gap"])
    assert len(bad) == 0, f"{len(bad)} rows differ beyond near-ties, e.g. rows {bad[:5]}"
    assert exact >= min_exact * rows, (exact, tie, rows)
    return exact, tie, rows


@pytest.mark.parametrize("schedule", ["grouped", "fused"])
@pytest.mark.parametrize("name", SELECT_CASES)
def test_selection_matches_reference(cuda_device, name, schedule):
    import nlogn_pisa_b200 as P

    case, rec, (q, k, v, dout), (qn, kn, vn, _) = np_inputs(name)
    qc, kc = _cuda(q, k)
    for method in case["methods"]:
        got = P.select_blocks(qc, kc, method=method, block_size=case["C"], topk=case["K"],
                              query_offset=offset_arg(case), force_first=case["ff"],
                              force_recent=case["fr"], routing_schedule=schedule)
        assert got.dtype == torch.int64 and got.shape == rec[f"ids_{method}"].shape
        _, trace = _trace(case, qn, kn, method)
        min_exact = 0.99 if name == "config1" else 1.0
        _check_ids(got.cpu().numpy(), rec[f"ids_{method}"].astype(np.int64), trace, min_exact)


def test_selection_outside_gpu_envelope_raises(cuda_device):
    """topk 4 / f64 are outside the GPU routing envelope: ValueError, as the reference's GPU path."""
    import nlogn_pisa_b200 as P

    case, rec, (q, k, v, dout), _ = np_inputs("tail_f32")
    qc, kc = _cuda(q, k)
    with pytest.raises(ValueError, match="topk"):
        P.select_blocks(qc, kc, block_size=case["C"], topk=case["K"], force_recent=1)
    with pytest.raises(ValueError):
        P.select_blocks(qc.double(), kc.double(), block_size=16, topk=8, force_recent=1)


@pytest.mark.parametrize("name", SELECT_CASES)
def test_network_order_matches_reference(cuda_device, name):
    """Slot order (network rank) is reproduced, not only the id sets."""
    import nlogn_pisa_b200 as P

    case, rec, (q, k, v, dout), _ = np_inputs(name)
    qc, kc = _cuda(q, k)
    method = case["methods"][0]
    got = P.select_blocks(qc, kc, method=method, block_size=case["C"], topk=case["K"],
                          query_offset=offset_arg(case), force_first=case["ff"],
                          force_recent=case["fr"]).cpu().numpy()
    want = rec[f"ids_{method}"].astype(np.int64)
    same_rows = (got == want).all(-1).mean()
    assert same_rows >= (0.99 if name == "config1" else 1.0), same_rows


@pytest.mark.parametrize("name", GPU_CASES)
def test_attention_matches_reference(cuda_device, name):
    import nlogn_pisa_b200 as P

    case, rec, (q, k, v, dout), (qn, kn, vn, dn) = np_inputs(name)
    ids = torch.from_numpy(rec[f"ids_{case['methods'][0]}"].astype(np.int64))
    qc, kc, vc, ic = _cuda(q, k, v, ids)
    out = P.sparse_attention(qc, kc, vc, ic, block_size=case["C"], query_offset=offset_arg(case))
    step = int(rec["out_rows_step"])
    tol = 2e-2 if case["dtype"] == "bf16" else 1e-5
    np.testing.assert_allclose(out.float().cpu().numpy()[:, ::step], rec["out"], rtol=0, atol=tol)
    # lse against the oracle's restatement
    from nlogn_pisa_b200.attention import attention_forward

    positions, offset = None, None
    from nlogn_pisa_b200.validation import query_positions
    positions, offset = query_positions(qc, kc, offset_arg(case))
    _, lse = attention_forward(qc, kc, vc, ic, case["C"], case["D"] ** -0.5, positions, offset, True)
    _, lse_ref = O.sparse_attention(qn, kn, vn, ids.numpy(), case["C"], positions=_positions(case))
    lse = lse.cpu().numpy()
    assert (np.isinf(lse) == np.isinf(lse_ref)).all()
    fin = np.isfinite(lse_ref)
    np.testing.assert_allclose(lse[fin], lse_ref[fin], rtol=0, atol=1e-4 if case["dtype"] == "bf16" else 1e-5)


@pytest.mark.parametrize("name", [n for n in GPU_CASES if CASES[n]["grads"]])
def test_attention_grads_match_oracle(cuda_device, name):
    import nlogn_pisa_b200 as P

    case, rec, (q, k, v, dout), (qn, kn, vn, dn) = np_inputs(name)
    ids = torch.from_numpy(rec[f"ids_{case['methods'][0]}"].astype(np.int64))
    qc, kc, vc, ic, dc = _cuda(q, k, v, ids, dout)
    qc.requires_grad_(True), kc.requires_grad_(True), vc.requires_grad_(True)
    out = P.sparse_attention(qc, kc, vc, ic, block_size=case["C"], query_offset=offset_arg(case))
    out.backward(dc)
    dq, dk, dv = O.sparse_attention_backward(qn, kn, vn, ids.numpy(), case["C"], dn,
                                             positions=_positions(case))
    if case["dtype"] == "bf16":
        tol = dict(rtol=1e-2, atol=2e-2)
    else:
        tol = dict(rtol=1e-4, atol=1e-4)
    for got, want, key in ((qc.grad, dq, "dq"), (kc.grad, dk, "dk"), (vc.grad, dv, "dv")):
        np.testing.assert_allclose(got.float().cpu().numpy(), want, err_msg=key, **tol)


def test_pyramid_matches_reference(cuda_device):
    import nlogn_pisa_b200 as P

    rec = load("pyramid")
    g = torch.Generator().manual_seed(11)
    keys = torch.randn(2, 1000, 3, 40, generator=g)
    for tag, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        levels = P.build_pyramid(keys.to(dt).cuda(), 16)
        want = [rec[f"{tag}_level{i}"] for i in range(len(levels))]
        assert f"{tag}_level{len(levels)}" not in rec
        for got, exp in zip(levels, want):
            got = got.float().cpu().numpy()
            if tag == "bf16":
                np.testing.assert_array_equal(got, exp)
            else:
                np.testing.assert_allclose(got, exp, rtol=1e-6, atol=1e-6)
        pooled = P.mean_pool(keys.to(dt).cuda(), 7)
        np.testing.assert_allclose(pooled.float().cpu().numpy(),
                                   O.mean_pool(O.cast(keys.numpy(), tag), 7, tag), rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("dtype,branching,n,heads,dim,block", [
    (torch.bfloat16, 4, 32768, 8, 128, 64),   # the 32K benchmark keys (16-leaf groups, two local levels)
    (torch.bfloat16, 2, 5000, 3, 64, 32),     # binary, ragged tail at every level
    (torch.float16, 4, 3333, 2, 256, 16),     # wide rows
    (torch.float32, 4, 2100, 4, 128, 64),     # fp32 rows (32 columns of 16 bytes)
    (torch.bfloat16, 4, 700, 5, 40, 64),      # 5 columns per row: a partial lane of leaves
])
def test_pyramid_two_pass_build_matches_oracle(cuda_device, dtype, branching, n, heads, dim, block):
    """Every level bit-exact against the oracle's rounding chain, keys strided in batch and tokens."""
    import nlogn_pisa_b200 as P

    g = torch.Generator().manual_seed(n + dim)
    big = torch.randn(2, n + 5, heads + 1, dim, generator=g).to(dtype).cuda()
    keys = big[:, 3:3 + n, 1:]                 # a view: batch, token and head strides of the parent
    assert not keys.is_contiguous()
    tag = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[dtype]
    want = O.build_pyramid(keys.cpu().float().numpy(), block, tag, branching=branching)
    got = P.build_pyramid(keys, block, branching=branching)
    assert len(got) == len(want)
    for level, (a, b) in enumerate(zip(got, want)):
        np.testing.assert_array_equal(a.float().cpu().numpy(), b, err_msg=f"level {level}")
    pooled = P.mean_pool(keys, block)
    np.testing.assert_array_equal(pooled.float().cpu().numpy(), want[0])


def test_strided_keys_and_pyramid_cache(cuda_device):
    """Decode through a PyramidCache (strided key views, incremental pyramid)."""
    import nlogn_pisa_b200 as P

    g = torch.Generator().manual_seed(21)
    B, N, H, G, D, C, K = 2, 700, 2, 4, 64, 32, 8
    keys = torch.randn(B, N + 3, H, D, generator=g).to(torch.bfloat16)
    q = torch.randn(B, 3, H * G, D, generator=g).to(torch.bfloat16)
    cache = P.PyramidCache.from_keys(keys[:, :N].cuda(), block_size=C)
    for step in range(3):
        cache.append(keys[:, N + step:N + step + 1].cuda())
        length = N + step + 1
        kn = O.cast(keys[:, :length].float().numpy(), "bf16")
        levels = O.build_pyramid(kn, C, "bf16")
        for lv_got, lv_want in zip(cache.levels, levels):
            np.testing.assert_array_equal(lv_got.float().cpu().numpy(), lv_want)
        qs = q[:, step:step + 1].cuda()
        for method in ("pisa", "pisa2", "pisa1"):
            got = P.select_blocks(qs, cache.keys, method=method, block_size=C, topk=K,
                                  query_offset=length - 1, force_recent=1, pyramid=cache,
                                  routing_schedule="fused").cpu().numpy()
            trace = {}
            qn = q[:, step:step + 1].float().numpy()
            pos = O.query_positions(B, 1, length, length - 1)
            want = O.pyramid_select(qn, kn, method, C, K, pos, True, 1, levels, trace=trace)
            _check_ids(got, want, trace)


@pytest.mark.parametrize("branching", [4])
@pytest.mark.parametrize("method", ["pisa", "pisa2", "pisa1"])
def test_branching4_matches_oracle(cuda_device, method, branching):
    """The 4-ary extension against the oracle's generalised restatement."""
    import nlogn_pisa_b200 as P

    g = torch.Generator().manual_seed(31)
    B, N, H, G, D, C, K = 1, 3000, 2, 4, 64, 16, 16
    q = torch.randn(B, N, H * G, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, N, H, D, generator=g).to(torch.bfloat16)
    got = P.select_blocks(q.cuda(), k.cuda(), method=method, block_size=C, topk=K, force_recent=1,
                          branching=branching).cpu().numpy()
    qn, kn = q.float().numpy(), k.float().numpy()
    levels = O.build_pyramid(kn, C, "bf16", branching=branching)
    rows = np.arange(0, N, 7)
    trace = {}
    want = O.pyramid_select(qn[:, rows], kn, method, C, K, O.query_positions(B, N, N)[:, rows], True, 1,
                            levels, branching=branching, trace=trace)
    _check_ids(got[:, rows], want, trace, min_exact=0.99)


def test_sampled_rows_at_32k(cuda_device):
    """The 32K prefill benchmark shape (N=32768, Hq=32, Hkv=8, D=128, C=64, K=32), sampled query rows."""
    import nlogn_pisa_b200 as P

    g = torch.Generator().manual_seed(0)
    B, N, Hq, H, D, C, K = 1, 32768, 32, 8, 128, 64, 32
    q = torch.randn(B, N, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, N, H, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, N, H, D, generator=g).to(torch.bfloat16)
    qc, kc, vc = _cuda(q, k, v)
    ids = P.select_blocks(qc, kc, method="pisa", block_size=C, topk=K, force_recent=1)
    out = P.sparse_attention(qc, kc, vc, ids, block_size=C)
    rows = np.array([0, 1, 63, 64, 2047, 2048, 4095, 9000, 16383, 20000, 32766, 32767])
    qn, kn, vn = q.float().numpy(), k.float().numpy(), v.float().numpy()
    levels = O.build_pyramid(kn, C, "bf16")
    trace = {}
    pos = np.broadcast_to(rows[None], (1, len(rows)))
    want = O.pyramid_select(qn[:, rows], kn, "pisa", C, K, pos, True, 1, levels, trace=trace)
    got = ids.cpu().numpy()[:, rows]
    _check_ids(got, want, trace, min_exact=0.95)
    ref_out, _ = O.sparse_attention(qn[:, rows], kn, vn, got, C, positions=pos)
    np.testing.assert_allclose(out.float().cpu().numpy()[:, rows], ref_out, rtol=0, atol=2e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [
    # B, T, N, Hq, H, D, C, S, causal, offset
    (1, 1500, 1500, 8, 2, 64, 64, 8, True, None),
    (2, 700, 1000, 4, 1, 128, 32, 12, True, 300),
    (1, 900, 900, 16, 1, 64, 16, 16, False, None),
    (1, 1200, 1337, 2, 2, 128, 128, 6, True, 137),
])
def test_tensor_core_attention_matches_oracle(cuda_device, dtype, shape):
    """Bucketed tensor-core attention on arbitrary indices: -1, duplicates, blocks past
    the causal edge, tails (N % C != 0), query offsets, non-causal."""
    import nlogn_pisa_b200 as P
    from nlogn_pisa_b200 import _lib

    B, T, N, Hq, H, D, C, S, causal, offset = shape
    g = torch.Generator().manual_seed(sum(shape[:8]))
    q = torch.randn(B, T, Hq, D, generator=g).to(dtype)
    k = torch.randn(B, N, H, D, generator=g).to(dtype)
    v = torch.randn(B, N, H, D, generator=g).to(dtype)
    blocks = -(-N // C)
    ids = torch.randint(-1, blocks + 1, (B, T, H, S), generator=g)
    ids[..., 1] = ids[..., 0]                     # duplicates count twice
    code = _lib.DTYPES[dtype]
    assert _lib.lib().pisa_sparse_attn_fwd_workspace_bytes(B, T, Hq, H, D, D, N, S, C, code) > 0
    out = P.sparse_attention(q.cuda(), k.cuda(), v.cuda(), ids.cuda(), block_size=C,
                             query_offset=offset, causal=causal)
    pos = O.query_positions(B, T, N, offset)
    want, _ = O.sparse_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), ids.numpy(), C,
                                 positions=pos, causal=causal)
    np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=0, atol=2e-2)


def test_packed_documents_match_per_document_oracle(cuda_device):
    """Packed varlen batch (cu_seqlens): block ids are document-relative and
    each document is selected and attended on its own, as the reference does
    (validation.py:59-81, top_k_pyramid.py:73-86, sparse_attn.py:29-55)."""
    import nlogn_pisa_b200 as P

    g = torch.Generator().manual_seed(41)
    lengths = [300, 517, 129]
    Hq, H, D, C, K = 8, 2, 64, 16, 8
    total = sum(lengths)
    q = torch.randn(1, total, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(1, total, H, D, generator=g).to(torch.bfloat16)
    v = torch.randn(1, total, H, D, generator=g).to(torch.bfloat16)
    cu = torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int64)
    qc, kc, vc = _cuda(q, k, v)
    ids = P.select_blocks(qc, kc, method="pisa", block_size=C, topk=K, cu_seqlens=cu.cuda(), force_recent=1)
    out = P.sparse_attention(qc, kc, vc, ids, block_size=C, cu_seqlens=cu.cuda()).float().cpu().numpy()
    ids = ids.cpu().numpy()
    start = 0
    for n in lengths:
        qd, kd, vd = (x[:, start:start + n].float().numpy() for x in (q, k, v))
        levels = O.build_pyramid(kd, C, "bf16")
        trace = {}
        pos = O.query_positions(1, n, n)
        want = O.pyramid_select(qd, kd, "pisa", C, K, pos, True, 1, levels, trace=trace)
        _check_ids(ids[:, start:start + n], want, trace)
        ref, _ = O.sparse_attention(qd, kd, vd, ids[:, start:start + n], C, positions=pos)
        np.testing.assert_allclose(out[:, start:start + n], ref, atol=2e-2, rtol=0)
        start += n


def test_batched_decode_step_matches_oracle(cuda_device):
    """A decode step for many sequences (Tq=1, fused schedule request, which
    runs the grouped tile pipeline from 256 rows on) against the oracle, then
    attention over the selected blocks."""
    import nlogn_pisa_b200 as P

    g = torch.Generator().manual_seed(43)
    B, N, Hq, H, D, C, K = 48, 3000, 32, 8, 128, 64, 16
    q = torch.randn(B, 1, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, N, H, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, N, H, D, generator=g).to(torch.bfloat16)
    qc, kc, vc = _cuda(q, k, v)
    ids = P.select_blocks(qc, kc, method="pisa", block_size=C, topk=K, query_offset=N - 1, force_recent=1,
                          routing_schedule="fused", branching=4)
    out = P.sparse_attention(qc, kc, vc, ids, block_size=C, query_offset=N - 1).float().cpu().numpy()
    ids = ids.cpu().numpy()
    qn, kn, vn = (x.float().numpy() for x in (q, k, v))
    levels = O.build_pyramid(kn, C, "bf16", branching=4)
    pos = O.query_positions(B, 1, N, N - 1)
    trace = {}
    want = O.pyramid_select(qn, kn, "pisa", C, K, pos, True, 1, levels, branching=4, trace=trace)
    _check_ids(ids, want, trace)
    ref, _ = O.sparse_attention(qn, kn, vn, ids, C, positions=pos)
    np.testing.assert_allclose(out, ref, atol=2e-2, rtol=0)


def test_tensor_core_attention_many_tiles_per_cta_poisoned_workspace(cuda_device):
    """Enough tiles that every CTA of the persistent tile kernel runs two tile
    groups (K/V buffers replaced mid-pipeline), on a workspace filled with NaN
    bytes so that a partial read before it is written cannot go unnoticed."""
    from nlogn_pisa_b200 import _lib

    B, T, N, Hq, H, D, C, S = 1, 2000, 2000, 16, 16, 64, 64, 16
    g = torch.Generator().manual_seed(5)
    q = torch.randn(B, T, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, N, H, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, N, H, D, generator=g).to(torch.bfloat16)
    blocks = -(-N // C)
    ids = torch.randint(-1, blocks + 1, (B, T, H, S), generator=g)
    ids[..., 1] = ids[..., 0]
    lib = _lib.lib()
    code = _lib.BF16
    wsb = lib.pisa_sparse_attn_fwd_workspace_bytes(B, T, Hq, H, D, D, N, S, C, code)
    assert wsb > 0
    qc, kc, vc, ic = (x.to(cuda_device) for x in (q, k, v, ids))
    for _ in range(2):
        ws = torch.full((wsb,), 0xFF, dtype=torch.uint8, device=cuda_device)
        out = torch.empty((B, T, Hq, D), dtype=torch.bfloat16, device=cuda_device)
        lse = torch.empty((B, T, Hq), dtype=torch.float32, device=cuda_device)
        _lib.check(lib.pisa_sparse_attn_fwd(
            _lib.ptr(qc), *qc.stride()[:3], _lib.ptr(kc), *kc.stride()[:3], _lib.ptr(vc), *vc.stride()[:3],
            _lib.ptr(ic), 8, None, 0, code, B, T, Hq, H, D, D, N, S, C, float(D ** -0.5), 0, _lib.ptr(out),
            _lib.ptr(lse), _lib.ptr(ws), wsb, _lib.stream_of(cuda_device)))
        _lib.check_workspace(ws, cuda_device)
        pos = O.query_positions(B, T, N, None)
        want, want_lse = O.sparse_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), ids.numpy(), C,
                                            positions=pos, causal=False)
        np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=0, atol=2e-2)
        np.testing.assert_allclose(lse.cpu().numpy(), want_lse, rtol=0, atol=1e-3)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [
    # B, T, N, Hq, H, D, S, causal, per-batch offsets
    (3, 1, 3000, 32, 8, 128, 32, True, False),   # decode step, 4 query heads per KV head
    (2, 5, 1337, 16, 2, 64, 12, True, True),     # 8 query heads per KV head, ragged tail
    (2, 3, 900, 2, 2, 128, 7, True, False),      # one query head per KV head
    (1, 40, 700, 4, 2, 64, 9, False, False),     # non-causal, two query heads per KV head
])
def test_ring_gather_attention_matches_oracle(cuda_device, dtype, shape):
    """The ring-staged gather (short query runs, block size 64, D in {64, 128},
    1/2/4/8 query heads per KV head) on arbitrary indices: -1, duplicates,
    blocks past the causal edge or past N, per-batch query positions; output
    and log-sum-exp against the oracle."""
    from nlogn_pisa_b200.attention import attention_forward

    B, T, N, Hq, H, D, S, causal, per_batch = shape
    C = 64
    g = torch.Generator().manual_seed(sum(shape[:7]))
    q = torch.randn(B, T, Hq, D, generator=g).to(dtype)
    k = torch.randn(B, N, H, D, generator=g).to(dtype)
    v = torch.randn(B, N, H, D, generator=g).to(dtype)
    blocks = -(-N // C)
    ids = torch.randint(-1, blocks + 1, (B, T, H, S), generator=g)
    ids[..., 1] = ids[..., 0]                     # duplicates count twice
    ids[..., 2] = blocks - 1                      # the ragged last block
    if per_batch:
        offsets = [N - T - 200 * b for b in range(B)]
        pos = O.query_positions(B, T, N, offsets)
        positions = torch.from_numpy(np.ascontiguousarray(pos)).cuda()
    else:
        pos = O.query_positions(B, T, N, N - T)
        positions = None
    out, lse = attention_forward(q.cuda(), k.cuda(), v.cuda(), ids.cuda(), C, D ** -0.5, positions, N - T, causal)
    want, want_lse = O.sparse_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), ids.numpy(), C,
                                        positions=pos, causal=causal)
    np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=0, atol=2e-2)
    np.testing.assert_allclose(lse.cpu().numpy(), want_lse, rtol=0, atol=1e-3)
