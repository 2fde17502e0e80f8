"""Flat BSA selection on the CUDA library against the reference's golden ids and the oracle."""

import numpy as np
import pytest
import torch

import pisa_oracle as O
from golden_cases import BSA_CASES, bsa_case, offset_arg

pytestmark = pytest.mark.gpu


def _oracle(q, k, C, K, positions, ff, fr, dtype):
    trace = {}
    ids = O.bsa_select(q.float().numpy(), k.float().numpy(), C, K, positions, ff, fr, dtype, trace=trace)
    return ids, trace


@pytest.mark.parametrize("name", sorted(BSA_CASES))
def test_bsa_matches_reference(cuda_device, name):
    """Ids equal bsa_fn(backend="torch") of the reference (fixtures), up to near-ties."""
    import nlogn_pisa_b200 as P

    case, rec, (q, k) = bsa_case(name)
    got = P.bsa_fn(q.cuda(), k.cuda(), case["C"], case["K"], query_offset=offset_arg(case),
                   force_first=case["ff"], force_recent=case["fr"])
    assert got.dtype == torch.int64 and got.shape == rec["ids"].shape
    positions = O.query_positions(case["B"], case["T"], case["N"], offset_arg(case))
    _, trace = _oracle(q, k, case["C"], case["K"], positions, case["ff"], case["fr"], case["dtype"])
    want = rec["ids"].astype(np.int64)
    rows, exact, tie, bad = O.compare_selection(got.cpu().numpy(), want, trace["min_gap"])
    assert len(bad) == 0, f"{len(bad)} rows differ beyond near-ties, e.g. rows {bad[:5]}"
    # slot order follows the network: rows with equal sets also match position by position
    same_set = (np.sort(got.cpu().numpy(), -1) == np.sort(want, -1)).all(-1)
    assert (got.cpu().numpy() == want).all(-1)[same_set].all()
    assert exact >= 0.99 * rows


def test_bsa_through_select_blocks_and_packed(cuda_device):
    """select_blocks(method="bsa") dispatches to BSA; packed documents use local ids."""
    import nlogn_pisa_b200 as P

    g = torch.Generator().manual_seed(31)
    q = torch.randn(1, 900, 8, 64, generator=g).to(torch.bfloat16).cuda()
    k = torch.randn(1, 900, 2, 64, generator=g).to(torch.bfloat16).cuda()
    a = P.select_blocks(q, k, method="bsa", block_size=32, topk=8, force_recent=2)
    b = P.bsa_fn(q, k, 32, 8, force_recent=2)
    assert torch.equal(a, b)
    cu = torch.tensor([0, 300, 333, 900], dtype=torch.int32, device="cuda")
    packed = P.select_blocks(q, k, method="bsa", block_size=32, topk=8, force_recent=1, cu_seqlens=cu)
    for s, e in ((0, 300), (300, 333), (333, 900)):
        one = P.bsa_fn(q[:, s:e], k[:, s:e], 32, 8, force_recent=1)
        assert torch.equal(packed[:, s:e], one)


@pytest.mark.parametrize("dtype,hq,hkv,d,C,K", [
    (torch.bfloat16, 32, 8, 128, 64, 32),    # the 32K benchmark geometry
    (torch.float16, 16, 1, 64, 64, 16),      # G = 16: one token per warp
    (torch.bfloat16, 4, 4, 64, 128, 8),      # G = 1, 128-block tiles
    (torch.float32, 6, 2, 32, 32, 16),       # fp32 FMA path, G = 3
])
def test_bsa_sampled_rows_at_scale(cuda_device, dtype, hq, hkv, d, C, K):
    """Every row on the GPU; sampled rows against the oracle (rows are independent given the keys)."""
    import nlogn_pisa_b200 as P

    n = 32768 if d == 128 else 8192
    g = torch.Generator().manual_seed(hq * 7 + d)
    q = torch.randn(1, n, hq, d, generator=g).to(dtype)
    k = torch.randn(1, n, hkv, d, generator=g).to(dtype)
    got = P.bsa_fn(q.cuda(), k.cuda(), C, K, force_recent=1).cpu().numpy()
    rows = np.sort(np.random.default_rng(3).choice(n, 48, replace=False))
    rows[:2] = [0, n - 1]
    tag = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[dtype]
    positions = np.asarray(rows, np.int64)[None]
    want, trace = _oracle(q[:, rows], k, C, K, positions, True, 1, tag)
    got_rows = got[:, rows]
    r, exact, tie, bad = O.compare_selection(got_rows, want, trace["min_gap"])
    assert len(bad) == 0, f"{len(bad)} sampled rows differ beyond near-ties"
    assert exact >= 0.95 * r


def test_bsa_argument_errors(cuda_device):
    import nlogn_pisa_b200 as P

    q = torch.zeros(1, 256, 4, 32, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 256, 4, 32, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="required distinct blocks"):
        P.bsa_fn(q, k, 16, 2, force_recent=3)
    with pytest.raises(ValueError):
        P.bsa_fn(q, k, 16, 8, force_recent=-1)
    with pytest.raises(ValueError):
        P.bsa_fn(q.cpu(), k.cpu(), 16, 8)
