"""Seeded synthetic inputs with the shapes of the benchmark configurations.

No public dataset is involved: every configuration is synthetic.  q, k, v are
drawn from N(0, 1) in that order with one seeded generator, in fp32, then cast
to the compute dtype.  The long-context configuration adds a per-block mean
offset N(0, 0.5^2) to the keys so block summaries carry signal.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    tokens: int
    q_heads: int
    kv_heads: int
    head_dim: int
    block_size: int
    topk: int
    branching: int
    force_first: bool
    force_recent: int
    method: str
    dtype: str
    seed: int = 0
    key_block_offset_std: float = 0.0

    def as_dict(self):
        return asdict(self)

    @property
    def torch_dtype(self):
        return {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[self.dtype]


WORKLOADS = {
    # 32K causal prefill, GQA 4:1 (the headline benchmark)
    "prefill32k": Workload("prefill32k", 1, 32768, 32, 8, 128, 64, 32, 4, True, 1, "pisa", "bf16"),
    # the same with the reference's binary pyramid
    "prefill32k_b2": Workload("prefill32k_b2", 1, 32768, 32, 8, 128, 64, 32, 2, True, 1, "pisa", "bf16"),
    # smaller cases of the 32K benchmark for profiler captures (inputs still larger than L2);
    # 16K is the smallest length at which the coarse level is scored densely and routed by warps
    "prefill8k": Workload("prefill8k", 1, 8192, 32, 8, 128, 64, 32, 4, True, 1, "pisa", "bf16"),
    "prefill16k": Workload("prefill16k", 1, 16384, 32, 8, 128, 64, 32, 4, True, 1, "pisa", "bf16"),
    # a smaller case of the 256K configuration for profiler captures: three
    # dense coarse levels as at 256K, 1024 leaves
    "prefill64k": Workload("prefill64k", 1, 65536, 32, 8, 128, 64, 32, 4, True, 1, "pisa", "bf16",
                           key_block_offset_std=0.5),
    # 256K causal prefill with informative block means
    "prefill256k": Workload("prefill256k", 1, 262144, 32, 8, 128, 64, 32, 4, True, 1, "pisa", "bf16",
                            key_block_offset_std=0.5),
    # the reference's CPU-runnable case
    "config1": Workload("config1", 1, 4096, 4, 4, 64, 64, 16, 4, True, 1, "pisa", "f32"),
}


def make_inputs(w: Workload, device="cpu", seed=None):
    """(q, k, v) for a workload, drawn on ``device`` with a seeded generator."""
    gen = torch.Generator(device=device).manual_seed(w.seed if seed is None else seed)
    shape_q = (w.batch, w.tokens, w.q_heads, w.head_dim)
    shape_kv = (w.batch, w.tokens, w.kv_heads, w.head_dim)
    q = torch.randn(shape_q, generator=gen, device=device)
    k = torch.randn(shape_kv, generator=gen, device=device)
    v = torch.randn(shape_kv, generator=gen, device=device)
    if w.key_block_offset_std:
        blocks = -(-w.tokens // w.block_size)
        offset = torch.randn((w.batch, blocks, w.kv_heads, w.head_dim), generator=gen, device=device)
        offset = offset * w.key_block_offset_std
        k = k + offset.repeat_interleave(w.block_size, dim=1)[:, : w.tokens]
    dt = w.torch_dtype
    return q.to(dt), k.to(dt), v.to(dt)
