"""Load golden fixtures and regenerate their seeded inputs as numpy arrays."""

from pathlib import Path

import numpy as np
import torch

from make_golden import BSA_CASES, CASES, LEAF_CASES, inputs, leaf_inputs, offset_arg  # noqa: F401  (tests/golden on sys.path)

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def np_inputs(name):
    """(case, q, k, v, dout) with arrays in float32/float64 and the torch tensors."""
    case = CASES[name]
    tensors = inputs(case)
    rec = load(name)
    for key, t in zip(("q", "k", "v", "dout"), tensors):
        x = t.to(torch.float64)
        got = np.array([x.sum().item(), x.square().sum().item(), x.abs().max().item()])
        np.testing.assert_allclose(got, rec[f"{key}_sum"], rtol=1e-12, atol=1e-9,
                                   err_msg=f"seeded {key} for {name} drifted from the fixture")
    arrays = [t.to(torch.float64 if t.dtype == torch.float64 else torch.float32).numpy() for t in tensors]
    return case, rec, tensors, arrays


def leaf_case(name):
    """(case, rec, (q, k, cand, positions) torch tensors) for a leaf-score fixture."""
    case = LEAF_CASES[name]
    q, k, cand, positions = leaf_inputs(case)
    rec = load(name)
    for key, t in (("q", q), ("k", k), ("cand", cand), ("positions", positions)):
        x = t.to(torch.float64)
        got = np.array([x.sum().item(), x.square().sum().item(), x.abs().max().item()])
        np.testing.assert_allclose(got, rec[f"{key}_sum"], rtol=1e-12, atol=1e-9,
                                   err_msg=f"seeded {key} for {name} drifted from the fixture")
    return case, rec, (q, k, cand, positions)


def bsa_case(name):
    """(case, rec, (q, k) torch tensors) for a flat BSA selection fixture."""
    case = BSA_CASES[name]
    q, k, _, _ = inputs(case)
    rec = load(name)
    for key, t in (("q", q), ("k", k)):
        x = t.to(torch.float64)
        got = np.array([x.sum().item(), x.square().sum().item(), x.abs().max().item()])
        np.testing.assert_allclose(got, rec[f"{key}_sum"], rtol=1e-12, atol=1e-9,
                                   err_msg=f"seeded {key} for {name} drifted from the fixture")
    return case, rec, (q, k)
