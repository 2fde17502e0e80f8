"""A LLaMA-style decoder block around the PISA token mixer, for training runs.

The block of the reference's xmixers LLaMA models
(xmixers/xmixers/models/transformer/llama/modeling_llama.py): pre-norm
RMSNorm -> PyramidSparseAttention -> residual, RMSNorm -> SwiGLU FFN ->
residual.  Norms, projections and the FFN are ordinary torch operations (GEMMs
on cuBLAS); the selection and the attention forward/backward run in this
library.  Used by the benchmark's training configuration (one block,
data-parallel over the GPUs of a node).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn
import torch.nn.functional as F

from .mixer import PyramidSparseAttention


@dataclass
class BlockConfig:
    """The PisaConfig fields the block and its mixer read (xmixers/xmixers/pisa_config.py:8-46)."""

    vocab_size: int = 50257
    hidden_size: int = 1024
    intermediate_size: int = 2816
    num_attention_heads: int = 16
    num_key_value_heads: int = 16
    head_dim: int = 64
    attention_method: str = "pisa2"
    block_size: int = 64
    topk: int = 16
    branching: int = 4
    prefill_routing: str | None = "auto"
    leaf_tile: int = 4
    force_first: bool = True
    force_recent: int = 1
    rope_theta: float = 10000.0
    rope_fraction: float = 0.5
    rope_position_mode: str = "document"
    rms_norm_eps: float = 1e-5
    bias: bool = False
    init_std: float = 0.02


class RMSNorm(nn.Module):
    def __init__(self, dim, eps):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        y = x.float()
        y = y * torch.rsqrt(y.square().mean(-1, keepdim=True) + self.eps)
        return (y * self.weight.float()).to(x.dtype)


class SwiGLU(nn.Module):
    def __init__(self, hidden, inner, bias):
        super().__init__()
        self.gate = nn.Linear(hidden, inner, bias=bias)
        self.up = nn.Linear(hidden, inner, bias=bias)
        self.down = nn.Linear(inner, hidden, bias=bias)

    def forward(self, x):
        return self.down(F.silu(self.gate(x)) * self.up(x))


class DecoderBlock(nn.Module):
    """Embedding -> one pre-norm block -> final norm; returns the hidden states."""

    def __init__(self, cfg: BlockConfig):
        super().__init__()
        self.embed = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.norm1 = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.attn = PyramidSparseAttention(cfg)
        self.norm2 = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.ffn = SwiGLU(cfg.hidden_size, cfg.intermediate_size, cfg.bias)
        self.norm_out = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, std=cfg.init_std)

    def forward(self, tokens):
        x = self.embed(tokens)
        a, _ = self.attn(self.norm1(x))
        x = x + a
        x = x + self.ffn(self.norm2(x))
        return self.norm_out(x)
