"""The numpy oracle against golden outputs of the reference's torch path."""

import numpy as np
import pytest

import pisa_oracle as O
from golden_cases import BSA_CASES, CASES, LEAF_CASES, bsa_case, leaf_case, load, np_inputs, offset_arg

SELECT_CASES = [n for n in CASES if n != "config1"]


def positions_for(case):
    off = case.get("offset")
    return O.query_positions(case["B"], case["T"], case["N"], off)


def run_select(case, q, k, method, trace=None):
    levels = O.build_pyramid(k, case["C"], case["dtype"])
    return O.pyramid_select(q, k, method, case["C"], case["K"], positions_for(case), case["ff"],
                            case["fr"], levels, trace=trace)


@pytest.mark.parametrize("name", SELECT_CASES)
def test_selection_matches_reference(name):
    case, rec, _, (q, k, v, dout) = np_inputs(name)
    for method in case["methods"]:
        trace = {}
        got = run_select(case, q, k, method, trace)
        want = rec[f"ids_{method}"].astype(np.int64)
        rows, exact, tie, bad = O.compare_selection(got, want, trace["min_gap"])
        assert len(bad) == 0, (name, method, bad[:5])
        # the small cases are exact, including network order
        assert exact == rows, (name, method, exact, rows, tie)
        np.testing.assert_array_equal(got, want)


def test_config1_selection_matches_reference():
    """The reference's CPU-runnable benchmark case (N=4096, Hq=Hkv=4, D=64, C=64, K=16, first+recent=1, fp32)."""
    case, rec, _, (q, k, v, dout) = np_inputs("config1")
    for method in case["methods"]:
        trace = {}
        got = run_select(case, q, k, method, trace)
        want = rec[f"ids_{method}"].astype(np.int64)
        rows, exact, tie, bad = O.compare_selection(got, want, trace["min_gap"])
        assert len(bad) == 0, (method, bad[:5])
        assert exact + tie == rows
        assert exact >= 0.999 * rows, (method, exact, rows)


@pytest.mark.parametrize("name", list(CASES))
def test_attention_matches_reference(name):
    case, rec, tensors, (q, k, v, dout) = np_inputs(name)
    ids = rec[f"ids_{case['methods'][0]}"].astype(np.int64)
    pos = positions_for(case)
    out, lse = O.sparse_attention(q, k, v, ids, case["C"], positions=pos)
    step = int(rec["out_rows_step"])
    tol = dict(rtol=0, atol=2e-2) if case["dtype"] == "bf16" else dict(rtol=1e-5, atol=1e-5)
    if case["dtype"] == "f64":
        tol = dict(rtol=1e-12, atol=1e-12)
    got = out[:, ::step]
    if case["dtype"] == "bf16":
        got = O.round_bf16(got)
    np.testing.assert_allclose(got, rec["out"], **tol)
    assert np.isfinite(lse[np.isfinite(lse)]).all()
    if "dq" in rec:
        dq, dk, dv = O.sparse_attention_backward(q, k, v, ids, case["C"], dout, positions=pos)
        # The reference's bf16 dK/dV come from autograd's index_put accumulating
        # every gathered contribution in bf16 (sparse_attn_torch.py:17-18), so
        # they carry a few percent of error; the oracle accumulates in fp32.
        gtol = dict(rtol=1e-4, atol=1e-4) if case["dtype"] != "bf16" else dict(rtol=3e-2, atol=3e-2)
        if case["dtype"] == "f64":
            gtol = dict(rtol=1e-10, atol=1e-10)
        for got_g, key in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
            want = rec[key]
            if case["dtype"] == "bf16":
                got_g = O.round_bf16(got_g)
            np.testing.assert_allclose(got_g, want, err_msg=key, **gtol)


def test_pyramid_matches_reference():
    import torch

    rec = load("pyramid")
    g = torch.Generator().manual_seed(11)
    keys = torch.randn(2, 1000, 3, 40, generator=g)
    for tag in ("f32", "bf16"):
        k = O.cast(keys.numpy(), tag)
        levels = O.build_pyramid(k, 16, tag)
        want = [rec[f"{tag}_level{i}"] for i in range(len([x for x in rec if x.startswith(tag + "_level")]))]
        assert len(levels) == len(want)
        for got, exp in zip(levels, want):
            if tag == "bf16":
                np.testing.assert_array_equal(got, exp)
            else:
                np.testing.assert_allclose(got, exp, rtol=1e-6, atol=1e-6)


def test_geometry_examples():
    """Routing geometry values worked out from top_k_pyramid_torch.py:124-133."""
    assert O.routing_geometry(64, 16) == (2, 16)
    assert O.routing_geometry(512, 32) == (4, 32)
    assert O.routing_geometry(2048, 32) == (6, 32)
    assert O.routing_geometry(4096, 32) == (7, 32)
    assert O.routing_geometry(20, 16) == (0, 32)
    assert O.routing_geometry(512, 32, branching=4) == (2, 32)


def test_network_tie_order():
    """Equal scores: the network's compare/exchange order decides (:84-110)."""
    scores = np.array([[1.0, 1.0, 1.0, 1.0, 0.5, 2.0, 1.0, 1.0]], np.float32)
    ids = np.arange(8)[None]
    import torch, sys
    # restated expectation computed by hand-running the network is checked
    # against the fixture-pinned implementation via an independent sort of the
    # selected scores: they must be the top-K values.
    got, sc = O.network_topk(scores, ids, 4, return_scores=True)
    assert sorted(scores[0][got[0]].tolist(), reverse=True) == sc[0].tolist()
    assert sc[0].tolist() == [2.0, 1.0, 1.0, 1.0]


def test_forced_count_raises():
    ids = np.arange(4)[None, None]
    pos = np.array([[255]])
    with pytest.raises(ValueError):
        O.routing_masks(ids, pos, 64, 1, True, 2)


@pytest.mark.parametrize("name", sorted(LEAF_CASES))
@pytest.mark.parametrize("method", ["pisa", "pisa1", "pisa2"])
def test_leaf_scores_match_reference(name, method):
    """grouped_leaf_scores semantics: the reference's block_scores and masks on
    random candidate lists (ids out of range, past the position, forced)."""
    case, rec, (q, k, cand, positions) = leaf_case(name)
    qn, kn = (x.float().numpy() for x in (q, k))
    for tag, pos in (("plain", None), ("masked", positions.numpy())):
        got = O.leaf_scores(qn, kn, cand.numpy(), case["C"], method, positions=pos, topk=case["K"],
                            force_first=case["ff"], force_recent=case["fr"], dtype=case["dtype"])
        want = rec[f"{method}_{tag}"]
        assert (np.isinf(got) == np.isinf(want)).all(), (method, tag)
        fin = np.isfinite(want)
        assert fin.any() and (~fin).any()
        np.testing.assert_allclose(got[fin], want[fin], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", sorted(BSA_CASES))
def test_bsa_selection_matches_reference(name):
    """Flat BSA ids equal the reference's bsa_fn(backend="torch") in network order."""
    case, rec, (q, k) = bsa_case(name)
    dt = case["dtype"]
    as_np = (lambda t: t.double().numpy()) if dt == "f64" else (lambda t: t.float().numpy())
    positions = O.query_positions(case["B"], case["T"], case["N"], offset_arg(case))
    trace = {}
    got = O.bsa_select(as_np(q), as_np(k), case["C"], case["K"], positions, case["ff"], case["fr"], dt,
                       trace=trace)
    want = rec["ids"].astype(np.int64)
    rows, exact, tie, bad = O.compare_selection(got, want, trace["min_gap"])
    assert len(bad) == 0 and exact == rows
    np.testing.assert_array_equal(got, want)


def test_bsa_streaming_network_ties():
    """Streaming top-K keeps the network's tie order on equal scores and -1 padding.

    Known answer from the reference's streaming_topk (bsa_torch.py:30-60) on
    these inputs: [[10, 7, 6, 9], [4, -1, -1, -1]].
    """
    scores = np.array([[1, 1, 1, 1, 0, 0, 2, 2, 1, 1, 3, 0], [0] * 12], np.float32)
    ids = np.broadcast_to(np.arange(12), (2, 12)).copy()
    ids[:, 11] = -1
    ids[1, 5:] = -1
    assert O.streaming_topk(scores, ids, 4, 8).tolist() == [[10, 7, 6, 9], [4, -1, -1, -1]]


def test_bsa_required_blocks_raise():
    q = np.zeros((1, 4, 1, 8), np.float32)
    k = np.zeros((1, 64, 1, 8), np.float32)
    positions = np.array([[60, 61, 62, 63]])
    with pytest.raises(ValueError):
        O.bsa_select(q, k, 8, 2, positions, True, 3)
