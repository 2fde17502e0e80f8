"""Timed CPU runs of the hot path on a bounded sample of a workload's query rows.

TEST INFRASTRUCTURE: used only by bench.py's ``cpu_baseline`` leg and its
``--impl reference`` arm, never by the product path.

Two implementations can be timed:

* ``port``: the numpy oracle (pisa_oracle.py), which restates the reference
  torch path and its branching-b generalisation;
* ``reference``: the reference's own torch CPU path,
  ``select_blocks(..., backend="torch")`` + ``sparse_attention(...,
  backend="torch")`` (pisa/pisa/ops/flash_sparse_attn/top_k_pyramid/
  top_k_pyramid.py:11-122, sparse_attn/sparse_attn.py:10-61), imported from
  the offline install under ``baseline/_ref``.  The reference pyramid is binary
  (mean_pooling.py:45-52), so it runs with branching 2 whatever the
  workload's branching.

Query rows are independent given the keys (validation.py:38-47 offsets), so
each of ``workers`` spawned processes (one thread each; by default one per host
core) times selection + attention on its own ``rows_per_worker`` sampled rows;
the pyramid build (once per sequence) is timed separately and charged pro
rata.  Throughput = sampled rows / the slowest worker's time, in tokens/s,
i.e. an extrapolation of the sample to the whole sequence.  The inputs are
drawn once in the parent and shared through memory-mapped files.
"""

from __future__ import annotations

import os
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"


def reference_available():
    """True when the reference package is installed under baseline/_ref."""
    return (REF / "pisa" / "ops").exists()


def _load(job):
    import numpy as np
    import torch

    arrays = {}
    for name in ("k", "v"):
        raw = np.load(Path(job["dir"]) / f"{name}.npy", mmap_mode="r")
        arrays[name] = torch.from_numpy(np.ascontiguousarray(raw)).view(torch.bfloat16 if job["bf16"] else torch.float32)
    q = torch.from_numpy(np.load(Path(job["dir"]) / "q_rows.npy")[job["slice"][0]:job["slice"][1]])
    arrays["q"] = q.view(torch.bfloat16) if job["bf16"] else q
    return arrays


def _worker(job):
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = "1"
    import sys
    import warnings

    import numpy as np
    import torch

    warnings.filterwarnings("ignore")
    torch.set_num_threads(1)
    sys.path.insert(0, str(ROOT))
    from nlogn_pisa_b200.workloads import Workload

    w = Workload(**job["workload"])
    x = _load(job)
    rows = np.asarray(job["rows"])
    if job["impl"] == "reference":
        sys.path.insert(0, str(REF))
        from pisa.ops import select_blocks, sparse_attention
        from pisa.ops.compress.mean_pooling.mean_pooling import build_pyramid

        k, v = x["k"][None], x["v"][None]
        t0 = time.perf_counter()
        levels = build_pyramid(k, w.block_size, backend="torch")
        pyramid_s = time.perf_counter() - t0
        t0 = time.perf_counter()
        for i, r in enumerate(rows):
            q = x["q"][i:i + 1][None]
            ids = select_blocks(q, k, method=w.method, block_size=w.block_size, topk=w.topk,
                                query_offset=int(r), force_first=w.force_first,
                                force_recent=w.force_recent, backend="torch", pyramid=levels)
            sparse_attention(q, k, v, ids, block_size=w.block_size, query_offset=int(r), backend="torch")
        return len(rows), time.perf_counter() - t0, pyramid_s
    sys.path.insert(0, str(ROOT / "oracle"))
    import pisa_oracle as O

    kn, vn = (x[n].float().numpy()[None] for n in ("k", "v"))
    qn = x["q"].float().numpy()[None]
    t0 = time.perf_counter()
    levels = O.build_pyramid(kn, w.block_size, w.dtype, branching=w.branching)
    pyramid_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    for start in range(0, len(rows), 8):
        sel = rows[start:start + 8]
        pos = sel[None]
        ids = O.pyramid_select(qn[:, start:start + 8], kn, w.method, w.block_size, w.topk, pos, w.force_first,
                               w.force_recent, levels, branching=w.branching)
        O.sparse_attention(qn[:, start:start + 8], kn, vn, ids, w.block_size, positions=pos)
    return len(rows), time.perf_counter() - t0, pyramid_s


def time_sample(workload, rows_per_worker=24, workers=None, seed=1234, impl="port", repeats=1):
    """Return a cpu_baseline dict for the bench JSON line (batch 0 of the workload).

    With ``repeats`` > 1 the same sample is timed that many times on one
    process pool and the dict carries every repeat's value in ``values``
    (``value`` is the median)."""
    import multiprocessing as mp
    from dataclasses import replace

    import numpy as np
    import torch

    import sys
    sys.path.insert(0, str(ROOT))
    from nlogn_pisa_b200.workloads import make_inputs

    if impl == "reference":
        if not reference_available():
            raise RuntimeError("the reference package is not installed under baseline/_ref")
        workload = replace(workload, branching=2)
    workers = workers or os.cpu_count() or 1
    rng = np.random.default_rng(seed)
    tokens = workload.tokens
    q, k, v = make_inputs(workload, "cpu")
    bf16 = q.dtype == torch.bfloat16
    rows = [sorted(rng.integers(0, tokens, rows_per_worker).tolist()) for _ in range(workers)]
    flat = np.concatenate([np.asarray(r) for r in rows])
    as_np = (lambda t: t.contiguous().view(torch.int16).numpy()) if bf16 else (lambda t: t.contiguous().numpy())
    with tempfile.TemporaryDirectory(prefix="pisa_cpu_") as tmp:
        np.save(Path(tmp) / "k.npy", as_np(k[0]))
        np.save(Path(tmp) / "v.npy", as_np(v[0]))
        np.save(Path(tmp) / "q_rows.npy", as_np(q[0, torch.from_numpy(flat)]))
        del q, k, v
        jobs = [{"workload": workload.as_dict(), "rows": rows[i], "impl": impl, "dir": tmp, "bf16": bf16,
                 "slice": (i * rows_per_worker, (i + 1) * rows_per_worker)} for i in range(workers)]
        ctx = mp.get_context("spawn")
        with ctx.Pool(workers) as pool:
            results = pool.map(_worker, jobs * repeats, chunksize=1)
    values, seconds_all = [], []
    for r in range(repeats):
        part = results[r * workers:(r + 1) * workers]
        n_rows = sum(x[0] for x in part)
        pyramid_s = max(x[2] for x in part)
        # each worker's row time plus its pro-rata share of one pyramid build
        seconds = max(x[1] + pyramid_s * x[0] / tokens for x in part)
        values.append(n_rows / seconds)
        seconds_all.append(seconds)
    order = sorted(range(repeats), key=lambda i: values[i])
    mid = order[repeats // 2]
    seconds = seconds_all[mid]
    what = ("reference torch path select_blocks + sparse_attention (backend='torch', baseline/_ref; "
            "binary pyramid, the reference's only branching)" if impl == "reference"
            else "numpy oracle selection + attention")
    return {
        "value": values[mid],
        "values": values,
        "unit": "tokens/s",
        "cores": workers,
        "kind": "reference" if impl == "reference" else "port",
        "sample": (f"{n_rows} random query rows of {workload.name} ({what}; {workers} processes x 1 thread "
                   f"on {os.cpu_count()} host cores; pyramid build {pyramid_s:.2f}s charged pro rata); "
                   f"tokens/s extrapolated from the sampled rows to the {tokens}-token sequence"),
        "seconds": seconds,
        "rows_sampled": n_rows,
    }
