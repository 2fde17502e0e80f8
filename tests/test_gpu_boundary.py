"""GPU checks of the boundary entry points: grouped_leaf_scores, the device
status path of bounded waits, pyramid caches (this library's and the
reference's own object) and the validation of caller pyramids."""

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import pisa_oracle as O
from golden_cases import LEAF_CASES, leaf_case

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("name", sorted(LEAF_CASES))
@pytest.mark.parametrize("method", ["pisa", "pisa1", "pisa2"])
@pytest.mark.parametrize("cand_dtype", [torch.int64, torch.int32])
def test_grouped_leaf_scores_match_reference(cuda_device, name, method, cand_dtype):
    """Scores in candidate order with -inf for ids out of range and, with
    positions, for masked ids (leaf_triton.py:144-232): bf16 pisa/pisa2 run the
    bucketed tensor-core scorer, fp32 and pisa1 the SIMT scorer."""
    import nlogn_pisa_b200 as P

    case, rec, (q, k, cand, positions) = leaf_case(name)
    qc, kc, cc, pc = q.cuda(), k.cuda(), cand.to(cand_dtype).cuda(), positions.cuda()
    for tag, pos in (("plain", None), ("masked", pc)):
        got = P.grouped_leaf_scores(qc, kc, cc, case["C"], method, positions=pos, topk=case["K"],
                                    force_first=case["ff"], force_recent=case["fr"]).cpu().numpy()
        want = rec[f"{method}_{tag}"]
        assert got.dtype == np.float32 and got.shape == want.shape
        assert (np.isinf(got) == np.isinf(want)).all(), (method, tag)
        fin = np.isfinite(want)
        np.testing.assert_allclose(got[fin], want[fin], rtol=1e-4, atol=2e-3, err_msg=f"{method} {tag}")


def test_grouped_leaf_scores_with_leaf_means(cuda_device):
    """pisa1 with caller leaf means (a pyramid level view) equals pooling inside."""
    import nlogn_pisa_b200 as P

    case, rec, (q, k, cand, positions) = leaf_case("leaf_bf16")
    qc, kc, cc = q.cuda(), k.cuda(), cand.cuda()
    cache = P.PyramidCache.from_keys(kc, block_size=case["C"])
    got = P.grouped_leaf_scores(qc, kc, cc, case["C"], "pisa1", leaf_means=cache.levels[0])
    want = P.grouped_leaf_scores(qc, kc, cc, case["C"], "pisa1")
    torch.testing.assert_close(got, want, rtol=0, atol=0)


def test_expired_wait_surfaces_as_runtime_error(cuda_device):
    """A bounded wait on a barrier nothing arrives on records PISA_ERR_TIMEOUT
    in the workspace status word; reading it back raises RuntimeError and the
    context stays usable.  No copy or tensor-core operation is in flight."""
    from nlogn_pisa_b200 import _lib

    lib = _lib.lib()
    ws = torch.empty(256, dtype=torch.uint8, device=cuda_device)
    stream = _lib.stream_of(cuda_device)
    _lib.check(lib.pisa_wait_selftest(1, 1000, _lib.ptr(ws), 256, stream))
    _lib.check_workspace(ws, cuda_device)                       # arrived: OK
    _lib.check(lib.pisa_wait_selftest(0, 2000, _lib.ptr(ws), 256, stream))
    assert lib.pisa_workspace_status(_lib.ptr(ws), stream) == _lib.ERR_TIMEOUT
    with pytest.raises(RuntimeError, match="bounded device-side wait expired"):
        _lib.check_workspace(ws, cuda_device)
    # the context still works, and the next call's clear resets the word
    x = torch.arange(10, device=cuda_device).sum().item()
    assert x == 45
    _lib.check(lib.pisa_wait_selftest(1, 1000, _lib.ptr(ws), 256, stream))
    _lib.check_workspace(ws, cuda_device)


def test_polynomial_exp2_matches_ex2_approx_error(cuda_device):
    """The FMA-pipe 2^x of the leaf epilogue stays within 4e-7 relative of the
    exact value over the inputs the epilogue gives it (x <= 0, down to the
    -125 clamp), the size of ex2.approx.f32's own error."""
    from nlogn_pisa_b200 import _lib

    x = torch.cat([torch.linspace(-125.0, 0.0, 1_000_001), -torch.rand(100_000) * 3,
                   torch.tensor([0.0, -0.5, -0.49999997, -1.5, -124.5, -125.0])]).to(cuda_device)
    poly, mufu = torch.empty_like(x), torch.empty_like(x)
    _lib.check(_lib.lib().pisa_ex2_selftest(_lib.ptr(x), _lib.ptr(poly), _lib.ptr(mufu), x.numel(),
                                            _lib.stream_of(cuda_device)))
    exact = torch.exp2(x.double())
    rel_poly = ((poly.double() - exact).abs() / exact).max().item()
    rel_mufu = ((mufu.double() - exact).abs() / exact).max().item()
    assert rel_poly < 4e-7, rel_poly
    assert rel_poly < 4 * max(rel_mufu, 1e-7), (rel_poly, rel_mufu)
    assert (poly > 0).all()


def test_checked_mode_reads_status_of_real_calls(cuda_device):
    """With status checks on, select_blocks / sparse_attention read their
    status words back (OK on a normal run) and give the same results."""
    import nlogn_pisa_b200 as P

    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, 2048, 8, 64, generator=g).to(torch.bfloat16).cuda()
    k = torch.randn(1, 2048, 2, 64, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(1, 2048, 2, 64, generator=g).to(torch.bfloat16).cuda()
    ids = P.select_blocks(q, k, block_size=64, topk=8, force_recent=1)
    out = P.sparse_attention(q, k, v, ids, block_size=64)
    P.set_status_checks(True)
    try:
        ids2 = P.select_blocks(q, k, block_size=64, topk=8, force_recent=1)
        out2 = P.sparse_attention(q, k, v, ids2, block_size=64)
    finally:
        P.set_status_checks(False)
    assert torch.equal(ids, ids2)
    assert torch.equal(out, out2)


def test_pyramid_cache_regrowth_matches_oracle(cuda_device):
    """Appends that cross several storage regrowths (pages of 16 leaves, 1.5x
    growth) keep every level equal to a fresh pyramid of the keys."""
    import nlogn_pisa_b200 as P

    g = torch.Generator().manual_seed(17)
    B, H, D, C = 2, 2, 64, 16
    keys = torch.randn(B, 1500, H, D, generator=g).to(torch.bfloat16)
    for branching in (2, 4):
        cache = P.PyramidCache(block_size=C, branching=branching)
        done = 0
        for n in (5, 250, 1, 1, 300, 17, 600, 326):
            cache.append(keys[:, done:done + n].cuda())
            done += n
            want = O.build_pyramid(O.cast(keys[:, :done].float().numpy(), "bf16"), C, "bf16",
                                   branching=branching)
            assert len(cache.levels) >= len(want)
            for lv_got, lv_want in zip(cache.levels, want):
                np.testing.assert_array_equal(lv_got.float().cpu().numpy(), lv_want)
            assert cache.offsets.tolist() == list(cache.starts)
            assert cache.lengths.tolist()[:len(want)] == [w.shape[1] for w in want]
        assert torch.equal(cache.keys.cpu(), keys)


def test_caller_pyramid_of_wrong_shape_raises(cuda_device):
    """select_blocks rejects a pyramid that does not belong to the keys or the branching."""
    import nlogn_pisa_b200 as P

    g = torch.Generator().manual_seed(19)
    q = torch.randn(1, 1, 8, 64, generator=g).to(torch.bfloat16).cuda()
    k = torch.randn(1, 3000, 2, 64, generator=g).to(torch.bfloat16).cuda()
    binary = P.PyramidCache.from_keys(k, block_size=32)
    with pytest.raises(ValueError, match="level sizes"):
        P.select_blocks(q, k, block_size=32, topk=8, query_offset=2999, force_recent=1, pyramid=binary,
                        routing_schedule="fused", branching=4)
    with pytest.raises(ValueError, match="level sizes"):
        P.select_blocks(q, k[:, :2000], block_size=32, topk=8, query_offset=1999, force_recent=1,
                        pyramid=binary, routing_schedule="fused")
    with pytest.raises(ValueError, match="level sizes"):
        P.select_blocks(q, k, block_size=32, topk=8, query_offset=2999, force_recent=1,
                        pyramid=binary.levels[:2], routing_schedule="fused", branching=4)


def _reference_pyramid_cache():
    """The reference's own xmixers PyramidCache class from the offline install, or skip."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "xmixers").exists():
        pytest.skip("the reference package is not installed under baseline/_ref")
    if str(ref) not in sys.path:
        sys.path.append(str(ref))
    try:
        from xmixers.utils.attention_cache import PyramidCache
    except Exception as exc:  # its import chain needs only torch; anything else is an environment gap
        pytest.skip(f"reference PyramidCache not importable: {type(exc).__name__}")
    return PyramidCache


def test_reference_pyramid_cache_object_is_a_drop_in(cuda_device):
    """The reference's own PyramidCache object (attention_cache.py:50-140),
    built by its own code on the host and moved to the GPU attribute by
    attribute, drives select_blocks(pyramid=...) to the oracle's ids; read with
    branching 4 it raises ValueError."""
    import nlogn_pisa_b200 as P

    RefCache = _reference_pyramid_cache()
    g = torch.Generator().manual_seed(23)
    B, N, H, G, D, C, K = 2, 1800, 2, 4, 64, 32, 8
    keys = torch.randn(B, N, H, D, generator=g).to(torch.bfloat16)
    q = torch.randn(B, 1, H * G, D, generator=g).to(torch.bfloat16)
    ref = RefCache.from_keys(keys[:, :1000], block_size=C)
    ref.append(keys[:, 1000:])
    ref.storage = ref.storage.cuda()
    ref.offsets, ref.lengths = ref.offsets.cuda(), ref.lengths.cuda()
    ref.tokens.buffer = ref.tokens.buffer.cuda()
    for method in ("pisa", "pisa2", "pisa1"):
        got = P.select_blocks(q.cuda(), ref.keys, method=method, block_size=C, topk=K, query_offset=N - 1,
                              force_recent=1, pyramid=ref, routing_schedule="fused").cpu().numpy()
        kn = O.cast(keys.float().numpy(), "bf16")
        levels = O.build_pyramid(kn, C, "bf16")
        trace = {}
        want = O.pyramid_select(q.float().numpy(), kn, method, C, K, O.query_positions(B, 1, N, N - 1),
                                True, 1, levels, trace=trace)
        rows, exact, tie, bad = O.compare_selection(got, want, trace["min_gap"])
        assert len(bad) == 0 and exact == rows, (method, exact, tie, rows)
    with pytest.raises(ValueError, match="level sizes"):
        P.select_blocks(q.cuda(), ref.keys, block_size=C, topk=K, query_offset=N - 1, force_recent=1,
                        pyramid=ref, routing_schedule="fused", branching=4)
