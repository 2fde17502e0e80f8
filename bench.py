#!/usr/bin/env python
"""Benchmark of the PISA hot path: pyramid -> block selection -> selected attention.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload prefill32k] [--impl ours|reference]

One step = one causal prefill of one synthetic sequence per GPU (the 32K
benchmark configuration by default: B=1, N=32768, Hq=32, Hkv=8, D=128, block 64, branching
4, top-K 32, forced first + current block, LSE scoring, bf16): key pyramid,
coarse-to-fine routing with leaf scoring and top-K, then attention over the
selected blocks.  Multi-GPU runs (torchrun) give each rank its own sequence
(weak scaling, no collective on the data path).  Prints one JSON line on rank 0.

The reference arm (--impl reference) times the CPU restatement of the
reference algorithm on a bounded sample of query rows on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import re
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--workload", default="prefill32k")
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-rows", type=int, default=16, help="sampled rows per CPU worker (cpu_baseline leg)")
    p.add_argument("--ref-rows", type=int, default=48, help="sampled rows per CPU worker (reference arm)")
    p.add_argument("--no-decode", action="store_true", help="skip the 128K-KV decode measurement")
    p.add_argument("--no-extra", action="store_true", help="skip the binary-pyramid and 256K lines")
    p.add_argument("--only", choices=("decode", "training"),
                   help="run one configuration alone and print its JSON object (profiling runs)")
    p.add_argument("--decode-batch", type=int, default=64, help="sequences of the decode configuration")
    p.add_argument("--decode-kv", type=int, default=131072, help="KV-cache tokens of the decode configuration")
    p.add_argument("--train-tokens", type=int, default=16384, help="tokens per sequence of the training configuration")
    p.add_argument("--triton-comparator", action="store_true",
                   help="time the reference's own Triton selection (baseline/_ref) beside ours on this GPU "
                        "and print that comparison as one JSON line instead of the benchmark")
    return p.parse_args()


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock, power and clock-event reasons of one GPU, read through NVML
    every 10 ms by a background thread while the timed region runs."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, device):
        self.device = device
        self.rows = []
        self.error = None
        self.thread = None
        self.stop_flag = threading.Event()

    def _handle(self, nvml):
        import torch

        props = torch.cuda.get_device_properties(self.device)
        bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        return nvml.nvmlDeviceGetHandleByPciBusId(bus)

    def start(self):
        try:
            import pynvml as nvml

            nvml.nvmlInit()
            handle = self._handle(nvml)
            self.max_mhz = nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM)
            masks = [(name, getattr(nvml, attr)) for name, attr in self.REASONS if hasattr(nvml, attr)]
        except Exception as exc:  # NVML missing or device not found: report, do not fail the bench
            self.error = f"nvml unavailable: {type(exc).__name__}"
            return

        def loop():
            while not self.stop_flag.is_set():
                try:
                    sm = nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM)
                    reasons = nvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                    power = nvml.nvmlDeviceGetPowerUsage(handle) / 1000.0
                except Exception as exc:
                    self.error = f"nvml read failed: {type(exc).__name__}"
                    return
                self.rows.append((sm, power, [name for name, bit in masks if reasons & bit]))
                time.sleep(0.01)

        self.thread = threading.Thread(target=loop, daemon=True)
        self.thread.start()

    def stop(self):
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join(timeout=5)
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.error or "no samples"]}
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": float(self.max_mhz),
                "reasons": sorted({n for r in self.rows for n in r[2]}), "samples": len(self.rows),
                "power_w_max": max(r[1] for r in self.rows)}


def decode_bench(args, device, world, peaks_hbm):
    """The decode benchmark configuration: one decode step for 64 sequences with a 131072-token
    KV cache (Hq=32, Hkv=8, D=128, block 64, branching 4, top-K 32, forced
    first + current block).  The pyramid is built once (a PyramidCache keeps it
    between steps); a step is the fused-schedule selection plus attention over
    the selected blocks.  Returns the JSON object reported under "decode"."""
    import torch
    import torch.distributed as dist
    from nlogn_pisa_b200 import _lib
    from nlogn_pisa_b200.selection import _c_array, level_sizes, routing_geometry  # noqa: F401

    Bd, N, Hq, H, D, C, K, br = args.decode_batch, args.decode_kv, 32, 8, 128, 64, 32, 4
    lib = _lib.lib()
    gen = torch.Generator(device=device).manual_seed(3)
    dt = torch.bfloat16
    k = torch.randn((Bd, N, H, D), generator=gen, device=device, dtype=dt)
    v = torch.randn((Bd, N, H, D), generator=gen, device=device, dtype=dt)
    q = torch.randn((Bd, 1, Hq, D), generator=gen, device=device, dtype=dt)
    code = _lib.dtype_code(q)
    sptr = _lib.stream_of(device)
    stream = torch.cuda.current_stream(device)
    leaves = N // C
    top, first_width = routing_geometry(leaves, K, br)
    sizes = level_sizes(leaves, br, top + 1)
    offsets = [sum(sizes[:i]) for i in range(len(sizes))]
    storage = torch.empty((Bd, sum(sizes), H, D), dtype=dt, device=device)
    _lib.check(lib.pisa_build_pyramid(_lib.ptr(k), code, Bd, N, H, D, *k.stride()[:3], C, br, len(sizes),
                                      _lib.ptr(storage), storage.stride(0), _c_array(offsets), sptr))
    method = _lib.METHODS["pisa"]
    fused = _lib.SCHEDULES[os.environ.get("PISA_BENCH_DECODE_SCHEDULE", "fused")]
    ws_bytes = lib.pisa_select_workspace_bytes(Bd, 1, Hq, H, D, N, code, method, C, br, K, top, first_width, fused, 0)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=device)
    ids = torch.empty((Bd, 1, H, K), dtype=torch.int64, device=device)
    out = torch.empty((Bd, 1, Hq, D), dtype=dt, device=device)
    lse = torch.empty((Bd, 1, Hq), dtype=torch.float32, device=device)

    def select():
        _lib.check(lib.pisa_select_blocks(
            _lib.ptr(q), *q.stride()[:3], _lib.ptr(k), *k.stride()[:3], _lib.ptr(storage), storage.stride(0),
            _c_array(offsets), _c_array(sizes), len(sizes), None, N - 1, code, Bd, 1, Hq, H, D, N, method, C, br,
            K, 1, 1, top, first_width, fused, _lib.ptr(ids), _lib.ptr(ws), ws_bytes, sptr))

    def attend():
        _lib.check(lib.pisa_sparse_attn_fwd(
            _lib.ptr(q), *q.stride()[:3], _lib.ptr(k), *k.stride()[:3], _lib.ptr(v), *v.stride()[:3],
            _lib.ptr(ids), 8, None, N - 1, code, Bd, 1, Hq, H, D, D, N, K, C, float(D ** -0.5), 1,
            _lib.ptr(out), _lib.ptr(lse), None, 0, sptr))

    for _ in range(max(args.warmup, 3)):
        select()
        attend()
    torch.cuda.synchronize()
    steps = max(args.steps, 5)
    for name in _lib.KERNELS:
        _lib.kernel_time(name)
    _lib.kernel_timing(True)
    launches0 = lib.pisa_launch_count()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    for e in ev:
        e[0].record(stream)
        select()
        e[1].record(stream)
        attend()
        e[2].record(stream)
    torch.cuda.synchronize()
    _lib.kernel_timing(False)
    launches = (lib.pisa_launch_count() - launches0) / steps
    leaf_ms, _ = _lib.kernel_time("leaf_tiles")
    other_us = {name: 1000.0 * _lib.kernel_time(name)[0] / steps for name in ("router", "leaf_final", "dense_level")}
    ms = max_over_ranks([sum(e[0].elapsed_time(e[2]) for e in ev) / steps,
                         sum(e[0].elapsed_time(e[1]) for e in ev) / steps,
                         sum(e[1].elapsed_time(e[2]) for e in ev) / steps], device, world)
    step_us, select_us, attend_us = (x * 1000.0 for x in ms)
    # bytes a step must move: the coarse child summaries, the keys of the b*K
    # leaf candidates (leaf scoring), keys and values of the K selected blocks
    # (attention), the queries and outputs
    summaries = sum(sizes[1:]) * br * D * 2 if top > 0 else 0
    per_head = summaries + br * K * C * D * 2 + 2 * K * C * D * 2
    step_bytes = Bd * H * per_head + 2 * Bd * Hq * D * 2
    achieved = step_bytes / (step_us * 1e-6) / 1e9

    # the same step as one fused launch (pisa_decode_select_attend): selection
    # and attention per (sequence, KV head) in one CTA
    ids_f = torch.empty_like(ids)
    out_f = torch.empty_like(out)

    def fused_step():
        _lib.check(lib.pisa_decode_select_attend(
            _lib.ptr(q), *q.stride()[:3], _lib.ptr(k), *k.stride()[:3], _lib.ptr(v), *v.stride()[:3],
            _lib.ptr(storage), storage.stride(0), _c_array(offsets), _c_array(sizes), len(sizes), None, N - 1,
            code, Bd, 1, Hq, H, D, D, N, method, C, br, K, 1, 1, top, first_width, float(D ** -0.5),
            _lib.ptr(ids_f), _lib.ptr(out_f), None, sptr))

    for _ in range(max(args.warmup, 3)):
        fused_step()
    torch.cuda.synchronize()
    launches0 = lib.pisa_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fused_step()
    e1.record(stream)
    torch.cuda.synchronize()
    fused_launches = (lib.pisa_launch_count() - launches0) / steps
    fused_us = max_over_ranks([e0.elapsed_time(e1) / steps], device, world)[0] * 1000.0
    same = (torch.sort(ids_f, -1).values == torch.sort(ids, -1).values).all(-1).float().mean().item()
    fused_achieved = step_bytes / (fused_us * 1e-6) / 1e9
    del k, v, storage
    return {"workload": f"decode{N // 1024}k", "batch": Bd, "kv_tokens": N, "q_heads": Hq, "kv_heads": H, "head_dim": D,
            "fused_kernel": {"us_per_step": fused_us, "us_per_token": fused_us / Bd, "launches_per_step": fused_launches,
                             "rows_with_same_ids_as_two_step_path": same,
                             "roofline": {"bound": "hbm", "achieved": fused_achieved, "unit": "GB/s",
                                          "peak": peaks_hbm, "frac": fused_achieved / peaks_hbm}},
            "block_size": C, "branching": br, "topk": K,
            "schedule": os.environ.get("PISA_BENCH_DECODE_SCHEDULE", "fused"),
            "us_per_step": step_us, "us_per_token": step_us / Bd, "steps": steps,
            "select_us": select_us, "attention_us": attend_us, "leaf_tiles_us": 1000.0 * leaf_ms / steps,
            "router_us": other_us["router"], "leaf_final_us": other_us["leaf_final"],
            "launches_per_step": launches,
            "roofline": {"bound": "hbm", "algorithmic_bytes_per_step": step_bytes, "achieved": achieved,
                         "unit": "GB/s", "peak": peaks_hbm, "frac": achieved / peaks_hbm},
            "l2": "inputs (34 GB of keys and values) far larger than L2"}


def profiled_traffic(kernel, workload):
    """DRAM bytes (read + write) per launch of `kernel` on `workload` from the
    committed ncu summaries: a line `traffic <kernel> <workload>: <bytes>`."""
    pattern = re.compile(rf"^traffic {kernel} {workload}: (\d+)", re.M)
    for path in sorted((ROOT / "profiles").glob("*.md")):
        m = pattern.search(path.read_text())
        if m:
            return int(m.group(1))
    return None


# ---------------------------------------------------------------------------
# the reference arm: CPU restatement on a bounded sample
# ---------------------------------------------------------------------------
def max_over_ranks(values, device, world):
    """Element-wise max of per-rank timings over all ranks: the slowest rank
    sets a multi-GPU step.  One all-reduce (MAX) when world > 1."""
    import torch

    t = torch.tensor([float(x) for x in values], device=device, dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def arm_config(w, world):
    """The `config` object of both arms' JSON lines."""
    return {
        "workload": w.name, "batch_per_gpu": w.batch, "tokens": w.tokens, "q_heads": w.q_heads,
        "kv_heads": w.kv_heads, "head_dim": w.head_dim, "block_size": w.block_size, "branching": w.branching,
        "topk": w.topk, "method": w.method, "forced": "first + current block", "schedule": "grouped",
        "l2": "flushed between timed steps (256 MiB write outside the events)",
        "parallelism": f"dp{world} (one sequence per GPU, no collective)",
    }


def run_reference(args, workload):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    sys.path.insert(0, str(ROOT / "oracle"))
    from cpu_sample import reference_available, time_sample

    # The reference's own CPU implementation of the path (its torch backend,
    # from the offline install under baseline/_ref) when present, else the
    # oracle port of it.  One process pool on all host cores; warm-up and
    # timed repeats of the same bounded sample of query rows.
    impl = "reference" if reference_available() else "port"
    repeats = max(1, args.steps) + max(0, args.warmup)
    base = time_sample(workload, rows_per_worker=args.ref_rows, impl=impl, repeats=repeats)
    timed = base["values"][max(0, args.warmup):]
    value = statistics.median(timed)
    line = {
        "impl": "reference",
        "metric": "prefill tokens/s (select+attend)",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * workload.tokens / value,
        "extrapolated": True,
        "step": (f"one step = {base['rows_sampled']} sampled query rows timed on {base['cores']} host processes, "
                 f"extrapolated to the {workload.tokens}-token sequence; ms_per_step is that extrapolation, "
                 f"sample wall time {1000.0 * base['seconds']:.0f} ms"),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": workload.dtype,
        "data": "synthetic",
        "config": arm_config(workload, int(os.environ.get("WORLD_SIZE", "1")))
        | ({"branching": 2, "branching_note": "the reference implements only a binary pyramid"}
           if base["kind"] == "reference" else {}),
        "cpu_baseline": {k: base[k] for k in ("unit", "cores", "kind", "sample")} | {"value": value},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def prefill_measure(w, device, rank, steps, warmup, world, kernel_timing=True, sample_clocks=None,
                    heads=None, seed=None):
    """Time the pyramid -> selection -> attention step of workload `w` through
    the C ABI with inputs resident in HBM.  Returns per-stage device times
    (max over ranks), per-kernel device times and the step's algorithmic work.
    `heads` = (kv_slice, q_slice) runs one KV-head group of the sequence."""
    import torch

    from nlogn_pisa_b200 import _lib
    from nlogn_pisa_b200.selection import _c_array, level_sizes, routing_geometry  # noqa: F401
    from nlogn_pisa_b200.workloads import make_inputs

    q, k, v = make_inputs(w, device, seed=w.seed + rank if seed is None else seed)
    if heads is not None:
        kv, qh = heads
        q, k, v = q[:, :, qh].contiguous(), k[:, :, kv].contiguous(), v[:, :, kv].contiguous()
    B, N, Hq, H, D = w.batch, w.tokens, q.shape[2], k.shape[2], w.head_dim
    G, C, K, br = Hq // H, w.block_size, w.topk, w.branching
    code = _lib.dtype_code(q)
    lib = _lib.lib()
    stream = torch.cuda.current_stream(device)
    sptr = _lib.stream_of(device)
    leaves = -(-N // C)
    top, first_width = routing_geometry(leaves, K, br)
    sizes = level_sizes(leaves, br, top + 1)
    offsets = [sum(sizes[:i]) for i in range(len(sizes))]
    storage = torch.empty((B, sum(sizes), H, D), dtype=q.dtype, device=device)
    ids = torch.empty((B, N, H, K), dtype=torch.int64, device=device)
    out = torch.empty((B, N, Hq, D), dtype=q.dtype, device=device)
    lse = torch.empty((B, N, Hq), dtype=torch.float32, device=device)
    method = _lib.METHODS[w.method]
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
    sel_ws_bytes = lib.pisa_select_workspace_bytes(B, N, Hq, H, D, N, code, method, C, br, K, top,
                                                   first_width, _lib.SCHEDULES["grouped"], 0)
    sel_ws = torch.empty(max(sel_ws_bytes, 1), dtype=torch.uint8, device=device)
    attn_ws_bytes = lib.pisa_sparse_attn_fwd_workspace_bytes(B, N, Hq, H, D, D, N, K, C, code)
    attn_ws = torch.empty(max(attn_ws_bytes, 1), dtype=torch.uint8, device=device)

    def pyramid():
        _lib.check(lib.pisa_build_pyramid(
            _lib.ptr(k), code, B, N, H, D, *k.stride()[:3], C, br, len(sizes), _lib.ptr(storage),
            storage.stride(0), _c_array(offsets), sptr))

    def select():
        _lib.check(lib.pisa_select_blocks(
            _lib.ptr(q), *q.stride()[:3], _lib.ptr(k), *k.stride()[:3], _lib.ptr(storage),
            storage.stride(0), _c_array(offsets), _c_array(sizes), len(sizes), None, 0, code, B, N,
            Hq, H, D, N, method, C, br, K, int(w.force_first), w.force_recent, top, first_width,
            _lib.SCHEDULES["grouped"], _lib.ptr(ids), _lib.ptr(sel_ws), sel_ws_bytes, sptr))

    def attend():
        _lib.check(lib.pisa_sparse_attn_fwd(
            _lib.ptr(q), *q.stride()[:3], _lib.ptr(k), *k.stride()[:3], _lib.ptr(v), *v.stride()[:3],
            _lib.ptr(ids), 8, None, 0, code, B, N, Hq, H, D, D, N, K, C, float(D ** -0.5), 1,
            _lib.ptr(out), _lib.ptr(lse), _lib.ptr(attn_ws), attn_ws_bytes, sptr))

    stages = (("pyramid", pyramid), ("select", select), ("attention", attend))
    for _ in range(max(warmup, 3)):
        for _, fn in stages:
            fn()
    torch.cuda.synchronize()
    _lib.check(lib.pisa_workspace_status(_lib.ptr(sel_ws), sptr))
    if attn_ws_bytes:
        _lib.check(lib.pisa_workspace_status(_lib.ptr(attn_ws), sptr))

    # algorithmic work of one step (outside the timed region), from the actual selections
    pos = torch.arange(N, device=device)
    valid_ids = (ids >= 0) & (ids * C <= pos[None, :, None, None])
    key_count = torch.clamp(torch.minimum(pos[None, :, None, None] + 1, torch.full_like(ids, N)) - ids * C, 0, C)
    attn_keys = torch.where(valid_ids, key_count, 0).sum().item()
    leaf = pos // C
    cand = torch.full_like(leaf, br * K)
    forced = 1 + (leaf > 0).long()          # first block + current block (force_recent = 1)
    invalid = (br - 1) - (leaf % br)        # siblings of the current leaf past the causal edge
    scored = torch.where(leaf + 1 > K, cand - forced - invalid, 0)
    es = q.element_size()
    plan = lib.pisa_select_level_plan(B, N, Hq, H, D, N, code, method, C, br, K, top, first_width,
                                      _lib.SCHEDULES["grouped"])
    dense_lv = [lv for lv in range(1, top + 1) if (plan >> lv) & 1]           # levels scored densely
    dense_nodes = sum(sizes[lv] for lv in dense_lv)                          # dense scores per row
    # the descent's own coarse work per row: every scored level's candidates x their children
    coarse_cols = sum((first_width if lv == top else br * K) * br for lv in range(1, top + 1) if sizes[lv] > K)
    work = {
        "attn_flops": attn_keys * G * 4 * D,
        "leaf_flops": scored.sum().item() * H * B * 2 * D * G * C,
        "pyramid_bytes": (B * N * H * D + B * sum(sizes) * H * D) * es,
        # combine: read every visible request's G partial rows, write the output
        "combine_bytes": valid_ids.sum().item() * G * (D * es + 8) + B * N * Hq * D * es,
        # router: read the dense coarse scores, write the leaf candidates (int32) and masks (u8)
        "router_bytes": B * N * H * (dense_nodes * 4 + br * K * 5),
        # dense coarse levels: children of every node of those levels, G query rows of D
        "dense_flops": B * N * H * G * 2 * D * sum(sizes[lv - 1] for lv in dense_lv),
        # the descent's algorithmic coarse work (candidate children per scored level)
        "coarse_flops": B * N * H * G * 2 * D * coarse_cols,
        # final top-K: read candidates, masks and scores of the b*K leaf slots, write K int64 ids
        "final_bytes": B * N * H * (br * K * 9 + K * 8),
        "selected_flops": attn_keys * G * 4 * D,
    }
    del valid_ids, key_count

    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    for name in _lib.KERNELS:
        _lib.kernel_time(name)            # drop warm-up records
    if kernel_timing:
        _lib.kernel_timing(True)
    launches0 = lib.pisa_launch_count()
    if sample_clocks:
        sample_clocks.start()
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(len(stages) + 1)] for _ in range(steps)]
    for step in range(steps):
        flush.zero_()
        ev = events[step]
        ev[0].record(stream)
        for i, (_, fn) in enumerate(stages):
            fn()
            ev[i + 1].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clock_info = sample_clocks.stop() if sample_clocks else None
    launches = lib.pisa_launch_count() - launches0
    _lib.kernel_timing(False)
    kernel_ms = {name: _lib.kernel_time(name) for name in _lib.KERNELS}
    stage_ms = [sum(ev[i].elapsed_time(ev[i + 1]) for ev in events) / steps for i in range(len(stages))]
    step_ms = sum(ev[0].elapsed_time(ev[-1]) for ev in events) / steps
    times = max_over_ranks([step_ms] + stage_ms, device, world)
    kt = max_over_ranks([kernel_ms[n][0] for n in _lib.KERNELS], device, world)
    _lib.check(lib.pisa_workspace_status(_lib.ptr(sel_ws), sptr))
    if attn_ws_bytes:
        _lib.check(lib.pisa_workspace_status(_lib.ptr(attn_ws), sptr))
    return {
        "tensors": (q, k, v), "step_ms": times[0], "stage_ms": dict(zip((s for s, _ in stages), times[1:])),
        "kernel_ms": {n: (ms, kernel_ms[n][1]) for n, ms in zip(_lib.KERNELS, kt)},
        "launches": launches, "work": work, "clocks": clock_info, "steps": steps,
        "value": world * B * N / (times[0] / 1000.0),
    }


def kernel_report(m, hbm, tensor):
    """Per-kernel roofline entries: algorithmic work per step over device time per step."""
    w = m["work"]
    table = {
        "leaf_tiles": ("leaf_tc_kernel", "tensor", w["leaf_flops"] / 1e12, tensor, "TFLOP/s"),
        "attn_tiles": ("attn_tc_kernel", "tensor", w["attn_flops"] / 1e12, tensor, "TFLOP/s"),
        "attn_combine": ("attn_combine_kernel", "hbm", w["combine_bytes"] / 1e9, hbm, "GB/s"),
        "pyramid": ("pyramid kernels", "hbm", w["pyramid_bytes"] / 1e9, hbm, "GB/s"),
        "dense_level": ("dense_level_kernel", "tensor", w["dense_flops"] / 1e12, tensor, "TFLOP/s"),
        "router": ("route_warp_kernel", "hbm", w["router_bytes"] / 1e9, hbm, "GB/s"),
        "leaf_final": ("leaf_final_kernel", "hbm", w["final_bytes"] / 1e9, hbm, "GB/s"),
    }
    report = {}
    for name, (ms_total, count) in m["kernel_ms"].items():
        if count == 0:
            continue
        kname, bound, amount, peak, unit = table[name]
        per_step_ms = ms_total / m["steps"]
        achieved = amount / (per_step_ms / 1000.0)
        report[name] = {"kernel": kname, "bound": bound, "ms_per_step": per_step_ms,
                        "launches_per_step": count / m["steps"], "ms_per_launch": ms_total / count,
                        "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak}
    return report


def stage_report(m, hbm, tensor):
    w = m["work"]
    work = {"pyramid": ("hbm", w["pyramid_bytes"] / 1e9, hbm, "GB/s"),
            "select": ("tensor", (w["leaf_flops"] + w["coarse_flops"]) / 1e12, tensor, "TFLOP/s"),
            "attention": ("tensor", w["attn_flops"] / 1e12, tensor, "TFLOP/s")}
    out = {}
    for name, ms in m["stage_ms"].items():
        bound, amount, peak, unit = work[name]
        achieved = amount / (ms / 1000.0)
        out[name] = {"ms": ms, "bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                     "frac": achieved / peak}
    return out


E2E_CUTS = (1 / 16, 1 / 4, 1 / 2, 3 / 4, 15 / 16)


def e2e_prefill(w, tensors, device, world, steps, cuts=E2E_CUTS):
    """The same step end to end through the public API with pinned host buffers,
    as an incremental prefill: token chunks of the sequence are copied in on
    one stream while earlier chunks are selected and attended on the compute
    stream (select_blocks / sparse_attention with query_offset on the key
    prefix, which gives the same result as one call over the whole sequence),
    and each chunk's output is copied back on a third stream."""
    import torch

    import nlogn_pisa_b200 as P

    q, k, v = tensors
    B, N, C, K, br = w.batch, w.tokens, w.block_size, w.topk, w.branching
    stream = torch.cuda.current_stream(device)
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    hout = torch.empty((B, N, w.q_heads, w.head_dim), dtype=q.dtype, pin_memory=True)
    dq, dk, dv = (torch.empty_like(x) for x in (q, k, v))
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    # short first and last chunks (the copy in of the first and the copy out
    # of the last are not overlapped with compute), long chunks between
    cuts = sorted({0, N} | {min(N, int(N * f) // C * C) for f in cuts})
    bounds = [(a, b) for a, b in zip(cuts[:-1], cuts[1:]) if b > a]
    ev_in = [torch.cuda.Event() for _ in bounds]
    ev_out = [torch.cuda.Event() for _ in bounds]

    def e2e_step():
        s_in.wait_stream(stream)          # the device copies of the last step are free
        with torch.cuda.stream(s_in):
            for (a, b), ev in zip(bounds, ev_in):
                for dst, src in ((dk, hk), (dv, hv), (dq, hq)):
                    dst[:, a:b].copy_(src[:, a:b], non_blocking=True)
                ev.record(s_in)
        for (a, b), ei, eo in zip(bounds, ev_in, ev_out):
            stream.wait_event(ei)
            sel = P.select_blocks(dq[:, a:b], dk[:, :b], method=w.method, block_size=C, topk=K,
                                  query_offset=a, force_first=w.force_first, force_recent=w.force_recent,
                                  branching=br)
            o = P.sparse_attention(dq[:, a:b], dk[:, :b], dv[:, :b], sel, block_size=C, query_offset=a)
            eo.record(stream)
            s_out.wait_event(eo)
            o.record_stream(s_out)
            with torch.cuda.stream(s_out):
                hout[:, a:b].copy_(o, non_blocking=True)
        stream.wait_stream(s_out)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(steps):
        e2e_step()
    e_end.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks([e_start.elapsed_time(e_end) / steps], device, world)[0]
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv))
    d2h = hout.numel() * hout.element_size()
    return {"value": world * B * N / (e2e_ms / 1000.0), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
            "mode": f"incremental prefill in token chunks {[b - a for a, b in bounds]} through select_blocks / "
                    "sparse_attention; host-to-device, compute and device-to-host on three streams"}


def long_context_bench(device, world, rank, hbm, tensor, steps=3):
    """The 262144-token configuration split over the ranks of this run, both ways
    (nlogn_pisa_b200/sharding.py):
      kv_heads  each rank runs its group of Hkv/world KV heads (and their query
                heads) of the one sequence; no collective;
      sequence  each rank owns 1/world of the query rows and of the keys/values,
                pools its leaf blocks, all-gathers leaf means, keys and values
                over NCCL and rebuilds the upper levels locally (world > 1).
    value = the sequence's tokens / the slowest rank's device time per step."""
    import torch
    import torch.distributed as dist

    import nlogn_pisa_b200 as P
    from nlogn_pisa_b200.sharding import head_groups, sequence_shards, sequence_sharded_prefill
    from nlogn_pisa_b200.workloads import WORKLOADS, make_inputs

    w = WORKLOADS["prefill256k"]
    out = {"workload": w.name, "tokens": w.tokens, "ranks": world}
    kv, qh = head_groups(w.q_heads, w.kv_heads, rank, world)
    m = prefill_measure(w, device, rank, steps, 3, world, heads=(kv, qh), seed=w.seed)
    m["tensors"] = None
    torch.cuda.empty_cache()
    out["kv_heads"] = {"value": w.tokens / (m["step_ms"] / 1000.0), "unit": "tokens/s", "ms_per_step": m["step_ms"],
                       "kv_heads_per_rank": kv.stop - kv.start, "scaling": "strong", "collective": "none",
                       "stages": stage_report(m, hbm, tensor)}
    if world > 1:
        q, k, v = make_inputs(w, device, seed=w.seed)
        shards = sequence_shards(w.tokens, w.block_size, world)
        a, b = shards[rank]
        ql, kl, vl = (x[:, a:b].contiguous() for x in (q, k, v))
        del q, k, v
        torch.cuda.empty_cache()
        stream = torch.cuda.current_stream(device)

        def step():
            return sequence_sharded_prefill(ql, kl, vl, shards, rank, method=w.method, block_size=w.block_size,
                                            topk=w.topk, force_first=w.force_first, force_recent=w.force_recent,
                                            branching=w.branching)

        for _ in range(2):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks([e0.elapsed_time(e1) / steps], device, world)[0]
        out["sequence"] = {"value": w.tokens / (ms / 1000.0), "unit": "tokens/s", "ms_per_step": ms,
                           "tokens_per_rank": b - a, "scaling": "strong",
                           "collective": "NCCL all-gather of leaf means, keys and values; upper levels rebuilt locally",
                           "api": "public Python API (select_blocks / sparse_attention with pyramid=)"}
        del ql, kl, vl
        torch.cuda.empty_cache()
    return out


def training_bench(device, world, rank, tensor, steps=5, warmup=3, batch=4, tokens=16384):
    """The training configuration: fwd + bwd + AdamW step of one random-init
    LLaMA-style block (d_model 1024, Hq = Hkv = 16, D = 64, SwiGLU 2816,
    RMSNorm, RoPE 1e4, pisa2, block 64, branching 4, top-K 16) on `batch`
    sequences of `tokens` uniform random token ids per GPU, bf16 autocast with
    fp32 master weights, data-parallel over the run's ranks (DDP: NCCL
    all-reduce of the gradients inside the timed step).  Loss: mean square of
    the block's normalised output.  value = tokens of all ranks / step time
    (max over ranks)."""
    import torch
    import torch.distributed as dist

    from nlogn_pisa_b200.model import BlockConfig, DecoderBlock

    cfg = BlockConfig()
    torch.manual_seed(1234)
    model = DecoderBlock(cfg).to(device)
    if world > 1:
        model = torch.nn.parallel.DistributedDataParallel(model, device_ids=[device.index])
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)
    g = torch.Generator(device=device).manual_seed(4321 + rank)
    ids = torch.randint(0, cfg.vocab_size, (batch, tokens), generator=g, device=device)
    stream = torch.cuda.current_stream(device)

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            h = model(ids)
            loss = h.float().square().mean()
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        loss = step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks([e0.elapsed_time(e1) / steps], device, world)[0]
    # the attention layer alone (selection + attention fwd + bwd) on this shape
    import nlogn_pisa_b200 as P

    Hq, D = cfg.num_attention_heads, cfg.head_dim
    q = torch.randn(batch, tokens, Hq, D, device=device, dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(batch, tokens, cfg.num_key_value_heads, D, device=device, dtype=torch.bfloat16,
                    requires_grad=True)
    v = torch.randn_like(k, requires_grad=True)
    dout = torch.randn(batch, tokens, Hq, D, device=device, dtype=torch.bfloat16)
    ids_sel = P.select_blocks(q.detach(), k.detach(), method=cfg.attention_method, block_size=cfg.block_size,
                              topk=cfg.topk, force_recent=cfg.force_recent, branching=cfg.branching)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    for i in range(warmup + steps):
        if i == warmup:
            ev[0].record(stream)
        P.select_blocks(q.detach(), k.detach(), method=cfg.attention_method, block_size=cfg.block_size,
                        topk=cfg.topk, force_recent=cfg.force_recent, branching=cfg.branching)
        if i == warmup:
            ev[1].record(stream)
        out = P.sparse_attention(q, k, v, ids_sel, block_size=cfg.block_size)
        if i == warmup:
            ev[2].record(stream)
        out.backward(dout)
        if i == warmup:
            ev[3].record(stream)
        q.grad = k.grad = v.grad = None
    torch.cuda.synchronize()
    sel_ms, fwd_ms, bwd_ms = (ev[j].elapsed_time(ev[j + 1]) for j in range(3))
    pos = torch.arange(tokens, device=device)
    valid = (ids_sel >= 0) & (ids_sel * cfg.block_size <= pos[None, :, None, None])
    keys = torch.clamp(pos[None, :, None, None] + 1 - ids_sel * cfg.block_size, 0, cfg.block_size)
    fwd_flops = torch.where(valid, keys, 0).sum().item() * 4 * D * (Hq // cfg.num_key_value_heads)
    bwd_flops = 2.5 * fwd_flops
    return {"workload": f"train_block{tokens // 1024}k", "value": world * batch * tokens / (ms / 1000.0), "unit": "tokens/s",
            "ms_per_step": ms, "steps": steps, "batch_per_gpu": batch, "tokens": tokens, "loss": float(loss.detach()),
            "parallelism": f"dp{world} (DDP, NCCL all-reduce of gradients)" if world > 1 else "dp1",
            "scaling": "weak", "model": "1 LLaMA-style block: d 1024, Hq=Hkv=16, D 64, SwiGLU 2816, RMSNorm, "
                                          "RoPE 1e4 (fraction 0.5), pisa2, block 64, branching 4, top-K 16",
            "attention_layer": {"select_ms": sel_ms, "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
                                "fwd_frac": fwd_flops / 1e12 / (fwd_ms / 1000.0) / tensor,
                                "bwd_frac": bwd_flops / 1e12 / (bwd_ms / 1000.0) / tensor,
                                "bwd_flops_rule": "2.5 x the forward's selected FLOPs"}}


def compact_line(w, m, hbm, tensor):
    """A secondary workload's measurement: throughput, stages and kernels."""
    return {"workload": w.name, "tokens": w.tokens, "branching": w.branching, "topk": w.topk,
            "value": m["value"], "unit": "tokens/s", "ms_per_step": m["step_ms"], "steps": m["steps"],
            "stages": stage_report(m, hbm, tensor), "kernels": kernel_report(m, hbm, tensor)}


# ---------------------------------------------------------------------------
# same-box GPU comparator: the reference's Triton selection
# ---------------------------------------------------------------------------
# (name, tokens, kv heads, head dim, topk, force_recent): the selection
# benchmark geometry of the reference (pisa/benchmarks/flash_sparse_attn/
# top_k_pyramid/benchmark.py:84-95: B=1, Hq=32, Hkv=2, D=64, block 64, K=8,
# first + previous + current block forced, seed 2024) and the 32K prefill
# configuration with the reference's binary pyramid.
COMPARATOR_CASES = (
    ("selection_bench", 65536, 2, 64, 8, 2),
    ("selection_bench", 131072, 2, 64, 8, 2),
    ("selection_bench", 262144, 2, 64, 8, 2),
    ("prefill32k_b2", 32768, 8, 128, 32, 1),
)


def _device_ms(fn, steps, warmup, flush):
    """Median CUDA-event milliseconds of fn() over `steps` calls, L2 flushed before each."""
    import torch

    for _ in range(warmup):
        fn()
    times = []
    for _ in range(steps):
        flush.zero_()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        end.synchronize()
        times.append(start.elapsed_time(end))
    return statistics.median(times)


def bsa_bench(device, steps=5):
    """Selection time of the flat BSA comparator (bsa_fn, the reference's
    baseline routing, bsa_torch.py:63-106) beside PISA routing on the same
    32K prefill inputs and GPU: the reference README's PISA-over-BSA ratio,
    measured on this library's own kernels."""
    import torch

    import nlogn_pisa_b200 as P
    from nlogn_pisa_b200.workloads import WORKLOADS, make_inputs

    w = WORKLOADS["prefill32k"]
    q, k, _ = make_inputs(w, device, seed=w.seed)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    opts = dict(block_size=w.block_size, topk=w.topk, force_first=True, force_recent=1)
    bsa_ms = _device_ms(lambda: P.bsa_fn(q, k, **opts), steps, 3, flush)
    pisa_ms = {f"b{br}": _device_ms(lambda: P.select_blocks(q, k, method="pisa", branching=br, **opts),
                                    steps, 3, flush) for br in (2, 4)}
    blocks = -(-w.tokens // w.block_size)
    # two passes of q . mean over the visible blocks of every (token, query head)
    flops = 2 * 2 * w.head_dim * w.q_heads * w.batch * sum(min(blocks, (t // w.block_size) + 1)
                                                            for t in range(w.tokens))
    out = {"workload": w.name, "tokens": w.tokens, "topk": w.topk, "block_size": w.block_size,
           "bsa_select_ms": bsa_ms, "pisa_select_ms": pisa_ms,
           "bsa_over_pisa_b2": bsa_ms / pisa_ms["b2"], "bsa_over_pisa_b4": bsa_ms / pisa_ms["b4"],
           "bsa_score_tflops": flops / 1e12 / (bsa_ms / 1000.0),
           "timing": f"median of {steps} CUDA-event samples, 256 MiB L2 flush before each; each call "
                     "includes its own leaf-mean or pyramid build"}
    del q, k, flush
    torch.cuda.empty_cache()
    return out


def triton_comparator(args):
    """Selection time (fresh pyramid + prefill routing) of the reference's own
    Triton path, select_blocks(..., backend="triton", routing_schedule=
    "grouped", leaf_tile=4) from the offline install under baseline/_ref
    (top_k_pyramid.py:11-122 -> top_k_pyramid_triton.py:311-447), beside this
    library's select_blocks on the same inputs and GPU, and its BSA
    selection (bsa_fn, backend="triton") at the selection-benchmark geometry.
    The agreement is the fraction of (token, KV head) rows whose id sets are
    equal; the Triton path and the torch path may differ in the last score
    bits (top_k_pyramid.py:44-45)."""
    import torch

    ref_root = ROOT / "baseline" / "_ref"
    if not (ref_root / "pisa" / "ops").exists():
        print(json.dumps({"comparator": "reference triton selection",
                          "unavailable": "the reference package is not installed under baseline/_ref"}))
        return 0
    sys.path.insert(0, str(ref_root))
    import nlogn_pisa_b200 as P

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    try:
        from pisa.ops.flash_sparse_attn.bsa import bsa_fn
        from pisa.ops.flash_sparse_attn.top_k_pyramid import top_k_pyramid_fn
    except Exception as exc:
        print(json.dumps({"comparator": "reference triton selection",
                          "unavailable": f"reference import failed: {type(exc).__name__}: {exc}"}))
        return 0
    rows = []
    for name, n, hkv, d, topk, recent in COMPARATOR_CASES:
        torch.manual_seed(2024)
        q = torch.randn(1, n, 32, d, device=device, dtype=torch.bfloat16)
        k = torch.randn(1, n, hkv, d, device=device, dtype=torch.bfloat16)
        opts = dict(method="pisa", block_size=64, topk=topk, force_first=True, force_recent=recent,
                    routing_schedule="grouped", leaf_tile=4)
        row = {"case": name, "tokens": n, "q_heads": 32, "kv_heads": hkv, "head_dim": d, "topk": topk,
               "force_recent": recent, "branching": 2}
        ours = lambda: P.select_blocks(q, k, backend="cuda", branching=2, **opts)  # noqa: E731
        ref = lambda: top_k_pyramid_fn(q, k, backend="triton", **opts)  # noqa: E731
        row["ours_ms"] = _device_ms(ours, args.steps, max(args.warmup, 3), flush)
        try:
            row["triton_ms"] = _device_ms(ref, args.steps, max(args.warmup, 3), flush)
            a = ours().sort(-1).values
            b = ref().to(torch.int64).sort(-1).values
            row["rows_equal"] = float((a == b).all(-1).float().mean())
            row["triton_over_ours"] = row["triton_ms"] / row["ours_ms"]
        except Exception as exc:
            row["triton_error"] = f"{type(exc).__name__}: {str(exc)[:200]}"
        if name == "selection_bench":
            row["bsa_ours_ms"] = _device_ms(lambda: P.bsa_fn(q, k, block_size=64, topk=topk, force_recent=recent),
                                            args.steps, max(args.warmup, 3), flush)
            try:
                row["bsa_triton_ms"] = _device_ms(lambda: bsa_fn(q, k, block_size=64, topk=topk, backend="triton"),
                                                  args.steps, max(args.warmup, 3), flush)
            except Exception as exc:
                row["bsa_error"] = f"{type(exc).__name__}: {str(exc)[:200]}"
                # the FLA prefill route of bsa_fn needs another fla-core release than the
                # box's; the reference's own Triton BSA kernel (bsa_triton.py:86-114) is
                # its general GPU path
                try:
                    from pisa.ops.flash_sparse_attn.bsa.bsa_triton import select_bsa

                    pos = torch.arange(n, device=device).expand(1, n).contiguous()
                    row["bsa_triton_ms"] = _device_ms(lambda: select_bsa(q, k, 64, topk, pos, True, recent),
                                                      args.steps, max(args.warmup, 3), flush)
                    row["bsa_triton_path"] = "bsa_triton.select_bsa"
                    got = P.bsa_fn(q, k, block_size=64, topk=topk, force_recent=recent).sort(-1).values
                    want = select_bsa(q, k, 64, topk, pos, True, recent).sort(-1).values
                    row["bsa_rows_equal"] = float((got == want).all(-1).float().mean())
                except Exception as exc2:
                    row["bsa_error2"] = f"{type(exc2).__name__}: {str(exc2)[:200]}"
        rows.append(row)
        del q, k
        torch.cuda.empty_cache()
    import triton

    print(json.dumps({"comparator": "reference triton selection (same GPU, same inputs)",
                      "gpu": torch.cuda.get_device_name(device), "triton": triton.__version__,
                      "timing": f"median of {args.steps} CUDA-event samples, 256 MiB L2 flush before each",
                      "cases": rows}), flush=True)
    return 0


def main():
    args = parse_args()
    from nlogn_pisa_b200.workloads import WORKLOADS

    if args.triton_comparator:
        return triton_comparator(args)
    workload = WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference(args, workload)

    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    from nlogn_pisa_b200 import _lib

    peaks = {}
    peaks_file = ROOT / "MEASURED_PEAKS.json"
    if peaks_file.exists():
        peaks = json.loads(peaks_file.read_text())
    hbm = peaks.get("hbm_gbs", 6650.0)
    tensor = peaks.get("bf16_tflops", 1590.0)
    src = "measured" if peaks else "fallback"

    if args.only == "decode":
        print(json.dumps(decode_bench(args, device, world, hbm)), flush=True)
        return 0
    if args.only == "training":
        print(json.dumps(training_bench(device, world, rank, tensor, steps=args.steps, tokens=args.train_tokens)),
              flush=True)
        return 0
    w = workload
    clocks = ClockSampler(local)
    m = prefill_measure(w, device, rank, args.steps, args.warmup, world, sample_clocks=clocks)
    e2e = e2e_prefill(w, m["tensors"], device, world, args.steps)
    m["tensors"] = None
    torch.cuda.empty_cache()
    kernels = kernel_report(m, hbm, tensor)
    dominant = max((n for n in kernels if n in ("leaf_tiles", "attn_tiles", "attn_combine")),
                   key=lambda n: kernels[n]["ms_per_step"])
    dom = kernels[dominant]

    extra = {}
    if world == 1 and not args.no_extra:
        for name, steps in (("prefill32k_b2", 5),):
            if name == w.name:
                continue
            mx = prefill_measure(WORKLOADS[name], device, rank, steps, 3, world)
            mx["tensors"] = None
            extra[name] = compact_line(WORKLOADS[name], mx, hbm, tensor)
            torch.cuda.empty_cache()
    bsa = None if (args.no_extra or world > 1) else bsa_bench(device)
    long_ctx = None if args.no_extra else long_context_bench(device, world, rank, hbm, tensor)
    training = None if args.no_extra else training_bench(device, world, rank, tensor)
    torch.cuda.empty_cache()
    decode = None if args.no_decode else decode_bench(args, device, world, hbm)

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            sys.path.insert(0, str(ROOT / "oracle"))
            from cpu_sample import time_sample

            cpu = time_sample(w, rows_per_worker=args.cpu_rows)
            for key in ("seconds", "values", "rows_sampled"):
                cpu.pop(key, None)
        line = {
            "metric": "prefill tokens/s (select+attend)",
            "value": m["value"],
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(args.warmup, 3),
            "ms_per_step": m["step_ms"],
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": w.dtype,
            "data": "synthetic",
            "config": arm_config(w, world),
            "roofline": {"kernel": dom["kernel"], "bound": dom["bound"], "achieved": dom["achieved"],
                         "peak": dom["peak"], "unit": dom["unit"], "frac": dom["frac"],
                         "traffic": profiled_traffic(dominant, w.name),
                         "peak_source": f"{src} (burst)", "ms_per_launch": dom["ms_per_launch"],
                         "launches_per_step": dom["launches_per_step"],
                         "work_per_launch": dom["achieved"] * dom["ms_per_launch"] / 1000.0,
                         "timing": "CUDA events around each launch on its stream, timed steps only"},
            "kernels": kernels,
            "stages": stage_report(m, hbm, tensor),
            "select_attend_tensor_frac": (m["work"]["leaf_flops"] + m["work"]["attn_flops"])
            / 1e12 / (m["step_ms"] / 1000.0) / tensor,
            "workloads": extra,
            "bsa": bsa,
            "long_context": long_ctx,
            "training": training,
            "decode": decode,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": m["launches"],
            "clocks": m["clocks"],
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
