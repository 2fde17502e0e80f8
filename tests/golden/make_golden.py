"""Generate the golden fixtures from the reference's own torch path.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py /path/to/NlogN_PISA

It imports the reference package ``pisa`` from ``<root>/pisa`` and calls
``select_blocks(..., backend="torch")`` (top_k_pyramid.py:11-122),
``sparse_attention(..., backend="torch")`` with autograd
(sparse_attn.py:10-61, sparse_attn_torch.py:6-35) and ``build_pyramid``
(mean_pooling.py:45-52), and the leaf scores of random candidate lists with
the reference's ``block_scores`` / ``routing_masks``
(top_k_pyramid_torch.py:48-80,114-120; the grouped_leaf_scores semantics of
leaf_triton.py:144-232), and the flat BSA selection ``bsa_fn(...,
backend="torch")`` (bsa.py:9-52, bsa_torch.py:63-106).  Inputs are regenerated from their seed by
:func:`inputs` (torch's CPU generator, fp32 normal draws in q, k, v, dout
order, then a cast), so the fixtures hold only outputs plus input checksums.
The reference is not needed to *read* the fixtures.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16, "f64": torch.float64}

# name: shape/parameter dictionary.  ``methods`` lists the selection methods
# recorded; attention (+ gradients when ``grads``) runs on the ids of the
# first method.  ``rows`` subsamples stored attention rows (every n-th token).
CASES = {
    "tail_f32": dict(B=2, N=200, T=200, Hq=4, Hkv=2, D=16, C=16, K=4, ff=True, fr=1,
                     dtype="f32", seed=1, methods=("pisa", "pisa1", "pisa2"), grads=True),
    "bf16_g4": dict(B=1, N=257, T=257, Hq=8, Hkv=2, D=64, C=16, K=8, ff=True, fr=2,
                    dtype="bf16", seed=2, methods=("pisa", "pisa1", "pisa2"), grads=True),
    "noff_g1": dict(B=1, N=700, T=700, Hq=2, Hkv=2, D=32, C=32, K=8, ff=False, fr=3,
                    dtype="f32", seed=3, methods=("pisa", "pisa1", "pisa2"), grads=False),
    "offset_suffix": dict(B=2, N=1000, T=3, offset=600, Hq=4, Hkv=1, D=32, C=32, K=8, ff=True,
                          fr=2, dtype="f32", seed=4, methods=("pisa", "pisa1", "pisa2"), grads=False),
    "batch_offsets": dict(B=2, N=1000, T=2, offset=[500, 998], Hq=4, Hkv=1, D=32, C=32, K=8,
                          ff=True, fr=1, dtype="f32", seed=5, methods=("pisa", "pisa2"), grads=False),
    "decode_bf16": dict(B=3, N=1500, T=1, Hq=8, Hkv=2, D=64, C=32, K=8, ff=True, fr=1,
                        dtype="bf16", seed=6, methods=("pisa", "pisa1", "pisa2"), grads=False),
    "fits": dict(B=1, N=100, T=100, Hq=2, Hkv=1, D=16, C=16, K=8, ff=True, fr=2,
                 dtype="f32", seed=7, methods=("pisa", "pisa1", "pisa2"), grads=True),
    "f64": dict(B=1, N=150, T=150, Hq=2, Hkv=1, D=16, C=16, K=4, ff=True, fr=1,
                dtype="f64", seed=8, methods=("pisa", "pisa2"), grads=True),
    # the reference's own CPU-runnable benchmark case
    "config1": dict(B=1, N=4096, T=4096, Hq=4, Hkv=4, D=64, C=64, K=16, ff=True, fr=1,
                    dtype="f32", seed=0, methods=("pisa", "pisa1", "pisa2"), grads=False, rows=16),
}


def inputs(case):
    """Seeded q, k, v, dout for a case (fp32 normal draws, then a cast)."""
    g = torch.Generator().manual_seed(case["seed"])
    dt = DTYPES[case["dtype"]]
    q = torch.randn(case["B"], case["T"], case["Hq"], case["D"], generator=g).to(dt)
    k = torch.randn(case["B"], case["N"], case["Hkv"], case["D"], generator=g).to(dt)
    v = torch.randn(case["B"], case["N"], case["Hkv"], case["D"], generator=g).to(dt)
    dout = torch.randn(case["B"], case["T"], case["Hq"], case["D"], generator=g).to(dt)
    return q, k, v, dout


def checksum(t):
    x = t.detach().to(torch.float64)
    return np.array([x.sum().item(), x.square().sum().item(), x.abs().max().item()])


def offset_arg(case):
    off = case.get("offset")
    if isinstance(off, list):
        return torch.tensor(off)
    return off


def as_np(t):
    return t.detach().to(torch.float64 if t.dtype == torch.float64 else torch.float32).numpy()


# Leaf scores of arbitrary candidate lists (grouped_leaf_scores semantics),
# computed with the reference's torch scoring and masks.
LEAF_CASES = {
    "leaf_bf16": dict(B=2, T=40, N=300, Hq=8, Hkv=2, D=64, C=16, W=16, K=8, ff=True, fr=2,
                      dtype="bf16", seed=12),
    "leaf_f32": dict(B=1, T=30, N=200, Hq=4, Hkv=4, D=32, C=32, W=10, K=4, ff=False, fr=1,
                     dtype="f32", seed=13),
}


# Flat BSA selection (bsa_fn(..., backend="torch"), bsa.py:9-52 -> bsa_torch.py:63-106)
# on the inputs of :func:`inputs`; ``C < 2K`` cases widen the comparison tile.
BSA_CASES = {
    "bsa_tail_f32": dict(B=2, N=200, T=200, Hq=4, Hkv=2, D=16, C=16, K=4, ff=True, fr=1,
                         dtype="f32", seed=21),
    "bsa_bf16_g4": dict(B=1, N=257, T=257, Hq=8, Hkv=2, D=64, C=16, K=8, ff=True, fr=2,
                        dtype="bf16", seed=22),
    "bsa_wide_tile": dict(B=1, N=700, T=700, Hq=2, Hkv=2, D=32, C=16, K=16, ff=False, fr=3,
                          dtype="f32", seed=23),
    "bsa_bench_g4": dict(B=1, N=2048, T=2048, Hq=16, Hkv=4, D=128, C=64, K=32, ff=True, fr=1,
                         dtype="bf16", seed=24),
    "bsa_decode_bf16": dict(B=3, N=1500, T=1, Hq=8, Hkv=2, D=64, C=32, K=8, ff=True, fr=1,
                            dtype="bf16", seed=25),
    "bsa_offsets": dict(B=2, N=1000, T=3, offset=[500, 997], Hq=4, Hkv=1, D=32, C=32, K=8, ff=True,
                        fr=2, dtype="f32", seed=26),
    "bsa_no_recent": dict(B=1, N=300, T=300, Hq=16, Hkv=1, D=32, C=32, K=8, ff=True, fr=0,
                          dtype="bf16", seed=27),
}


def leaf_inputs(case):
    """Seeded q, k, candidates (distinct ids per row in [-2, blocks + 2)) and positions."""
    g = torch.Generator().manual_seed(case["seed"])
    dt = DTYPES[case["dtype"]]
    q = torch.randn(case["B"], case["T"], case["Hq"], case["D"], generator=g).to(dt)
    k = torch.randn(case["B"], case["N"], case["Hkv"], case["D"], generator=g).to(dt)
    blocks = -(-case["N"] // case["C"])
    rows = case["B"] * case["T"] * case["Hkv"]
    cand = torch.stack([torch.randperm(blocks + 4, generator=g)[:case["W"]] - 2 for _ in range(rows)])
    cand = cand.reshape(case["B"], case["T"], case["Hkv"], case["W"])
    positions = torch.randint(0, case["N"], (case["B"], case["T"]), generator=g)
    return q, k, cand, positions


def leaf_reference(root_modules, q, k, cand, positions, case, method):
    """The reference's block_scores / routing_masks / mean_pool on one case."""
    block_scores, routing_masks, mean_pool = root_modules
    C, K = case["C"], case["K"]
    blocks = -(-case["N"] // C)
    in_range = (cand >= 0) & (cand < blocks)
    ids = torch.where(in_range, cand, -1)
    out = {}
    for masked in (False, True):
        if masked:
            pos = positions[..., None].expand(*cand.shape[:3])
            valid, forced, scoreable = routing_masks(ids, pos, C, K, case["ff"], case["fr"])
            if method == "pisa1":
                scoreable = valid & ~forced
        else:
            scoreable = in_range
        if method == "pisa1":
            source, support, scale = mean_pool(k, C, backend="torch"), 1, 1.0
        else:
            source, support, scale = k, C, case["D"] ** -0.5
        result = torch.full(cand.shape, -torch.inf)
        for b in range(case["B"]):
            src = source[b:b + 1].expand(case["T"], *source.shape[1:])
            sc = block_scores(q[b], src, torch.where(scoreable[b], ids[b], -1), support, method, scale)
            result[b] = torch.where(scoreable[b], sc.float(), -torch.inf)
        out["masked" if masked else "plain"] = result.numpy()
    return out


def main(root, which=None):
    sys.path.insert(0, str(Path(root) / "pisa"))
    from pisa.ops.compress.mean_pooling import build_pyramid, mean_pool
    from pisa.ops.flash_sparse_attn.sparse_attn import sparse_attention
    from pisa.ops.flash_sparse_attn.top_k_pyramid import select_blocks
    from pisa.ops.flash_sparse_attn.top_k_pyramid.top_k_pyramid_torch import block_scores, routing_masks

    from pisa.ops.flash_sparse_attn.bsa import bsa_fn

    torch.set_num_threads(max(1, torch.get_num_threads()))
    for name, case in BSA_CASES.items():
        if which and name not in which:
            continue
        q, k, _, _ = inputs(case)
        ids = bsa_fn(q, k, case["C"], case["K"], query_offset=offset_arg(case), force_first=case["ff"],
                     force_recent=case["fr"], backend="torch")
        rec = {"q_sum": checksum(q), "k_sum": checksum(k), "ids": ids.numpy().astype(np.int16)}
        np.savez_compressed(HERE / f"{name}.npz", **rec)
        print(name, {k: v.shape for k, v in rec.items()})
    for name, case in LEAF_CASES.items():
        if which and name not in which:
            continue
        q, k, cand, positions = leaf_inputs(case)
        rec = {"q_sum": checksum(q), "k_sum": checksum(k), "cand_sum": checksum(cand),
               "positions_sum": checksum(positions)}
        for method in ("pisa", "pisa1", "pisa2"):
            for tag, arr in leaf_reference((block_scores, routing_masks, mean_pool), q, k, cand, positions,
                                           case, method).items():
                rec[f"{method}_{tag}"] = arr
        np.savez_compressed(HERE / f"{name}.npz", **rec)
        print(name, {k: v.shape for k, v in rec.items()})
    if which and not (set(which) & (set(CASES) | {"pyramid"})):
        return
    for name, case in CASES.items():
        if which and name not in which:
            continue
        q, k, v, dout = inputs(case)
        rec = {
            "q_sum": checksum(q), "k_sum": checksum(k), "v_sum": checksum(v), "dout_sum": checksum(dout),
        }
        for method in case["methods"]:
            ids = select_blocks(q, k, method=method, block_size=case["C"], topk=case["K"],
                                query_offset=offset_arg(case), force_first=case["ff"],
                                force_recent=case["fr"], backend="torch")
            rec[f"ids_{method}"] = ids.numpy().astype(np.int16)
        ids = torch.from_numpy(rec[f"ids_{case['methods'][0]}"].astype(np.int64))
        qa, ka, va = (x.clone().requires_grad_(case["grads"]) for x in (q, k, v))
        out = sparse_attention(qa, ka, va, ids, block_size=case["C"], query_offset=offset_arg(case),
                               backend="torch")
        step = case.get("rows", 1)
        rec["out"] = as_np(out)[:, ::step]
        rec["out_rows_step"] = np.array(step)
        if case["grads"]:
            (out.to(torch.float64) * dout.to(torch.float64)).sum().backward()
            rec["dq"], rec["dk"], rec["dv"] = as_np(qa.grad), as_np(ka.grad), as_np(va.grad)
        np.savez_compressed(HERE / f"{name}.npz", **rec)
        print(name, {k: v.shape for k, v in rec.items()})

    if which and "pyramid" not in which:
        return
    # Pyramid levels with a tail block, bf16 and f32 (mean_pooling_torch.py:7-14).
    g = torch.Generator().manual_seed(11)
    keys = torch.randn(2, 1000, 3, 40, generator=g)
    rec = {"keys_sum": checksum(keys)}
    for tag, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        levels = build_pyramid(keys.to(dt), 16, backend="torch")
        for i, level in enumerate(levels):
            rec[f"{tag}_level{i}"] = as_np(level)
    np.savez_compressed(HERE / "pyramid.npz", **rec)
    print("pyramid", len(rec))


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <path of the NlogN_PISA checkout> [fixture names...]")
    main(sys.argv[1], set(sys.argv[2:]) or None)
