"""Timed CPU run of the oracle on a bounded sample of a workload's query rows.

TEST INFRASTRUCTURE: used only by bench.py's ``cpu_baseline`` leg and its
``--impl reference`` arm, never by the product path.

Query rows are independent given the keys (validation.py:38-47 offsets), so
the oracle's selection + attention is timed on ``rows_per_worker`` sampled
rows in each of ``workers`` spawned processes (one BLAS thread each); the
pyramid build (once per sequence) is timed separately and charged pro rata.
Throughput = sampled rows / max worker time, in tokens/s.
"""

from __future__ import annotations

import os
import time


def _worker(job):
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
    os.environ.setdefault("MKL_NUM_THREADS", "1")
    import sys
    from pathlib import Path

    import numpy as np
    import torch

    torch.set_num_threads(1)
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "oracle"))
    import pisa_oracle as O
    from nlogn_pisa_b200.workloads import Workload, make_inputs

    w = Workload(**job["workload"])
    q, k, v = make_inputs(w, "cpu")
    qn, kn, vn = (x.float().numpy() for x in (q, k, v))
    del q, k, v
    t0 = time.perf_counter()
    levels = O.build_pyramid(kn, w.block_size, w.dtype, branching=w.branching)
    pyramid_s = time.perf_counter() - t0
    rows = np.asarray(job["rows"])
    t0 = time.perf_counter()
    for start in range(0, len(rows), 8):
        sel = rows[start:start + 8]
        pos = np.broadcast_to(sel[None], (w.batch, len(sel)))
        ids = O.pyramid_select(qn[:, sel], kn, w.method, w.block_size, w.topk, pos, w.force_first,
                               w.force_recent, levels, branching=w.branching)
        O.sparse_attention(qn[:, sel], kn, vn, ids, w.block_size, positions=pos)
    return len(rows), time.perf_counter() - t0, pyramid_s


def time_sample(workload, rows_per_worker=24, workers=None, seed=1234):
    """Return a cpu_baseline dict for the bench JSON line."""
    import multiprocessing as mp

    import numpy as np

    workers = workers or min(16, os.cpu_count() or 1)
    rng = np.random.default_rng(seed)
    tokens = workload.tokens
    jobs = [{"workload": workload.as_dict(),
             "rows": sorted(rng.integers(0, tokens, rows_per_worker).tolist())} for _ in range(workers)]
    ctx = mp.get_context("spawn")
    with ctx.Pool(workers) as pool:
        results = pool.map(_worker, jobs)
    n_rows = sum(r[0] for r in results)
    pyramid_s = max(r[2] for r in results)
    # each worker's row time plus its pro-rata share of one pyramid build
    per_worker = [r[1] + pyramid_s * r[0] / tokens for r in results]
    seconds = max(per_worker)
    return {
        "value": n_rows * workload.batch / seconds,
        "unit": "tokens/s",
        "cores": workers,
        "kind": "port",
        "sample": (f"{n_rows} random query rows of {workload.name} (numpy oracle selection + attention, "
                   f"{workers} processes x 1 thread, pyramid build {pyramid_s:.2f}s charged pro rata)"),
        "seconds": seconds,
    }
