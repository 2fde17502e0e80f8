"""The PISA token mixer of the xmixers LLaMA models, on this library.

Mirror of PyramidSparseAttention
(xmixers/xmixers/modules/token_mixers/vanilla_attention/pyramid_sparse_attention.py:71-222):
q/k/v projections, split-half rotary encoding of q and k (pisa_rotary), block
selection and attention over the selected blocks (select_blocks /
sparse_attention), the output projection, and the decode cache (PyramidCache
for keys, TensorCache for values) with the same dictionary layout.  The
config is duck-typed: any object with the PisaConfig field names
(xmixers/xmixers/pisa_config.py:8-46) works.  Only the PISA selection methods
(pisa, pisa1, pisa2) are served; full attention and NSA are other layers.
"""

from __future__ import annotations

import torch
from torch import nn

from . import _lib
from .attention import sparse_attention
from .cache import PyramidCache, TensorCache
from .selection import select_blocks


def rotary_frequencies(head_dim, base, fraction):
    """Per-pair frequencies base^(-2i/D) for the first int(D/2 * fraction) pairs,
    0 for the rest (the xmixers RotaryEmbedding, lrpe.py:20-27 with type 3)."""
    theta = base ** (-2 / head_dim * torch.arange(head_dim // 2, dtype=torch.int64)).float()
    theta[int(head_dim // 2 * fraction):] = 0
    return theta


def token_positions(length, device, cu_seqlens=None, offset=0):
    """[1, length] positions; under cu_seqlens each document restarts at 0
    (pyramid_sparse_attention.py:6-11)."""
    positions = torch.arange(length, device=device)[None] + offset
    if cu_seqlens is not None:
        for begin, end in zip(cu_seqlens[:-1].tolist(), cu_seqlens[1:].tolist()):
            positions[:, begin:end] -= begin
    return positions


def _rotary(x, frequency, positions):
    out = torch.empty_like(x)
    pos = positions.to(device=x.device, dtype=torch.int64).contiguous()
    pos_sb = 0 if pos.shape[0] == 1 else pos.stride(0)
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().pisa_rotary(
            _lib.ptr(x), *x.stride()[:3], _lib.ptr(out), *out.stride()[:3], _lib.ptr(pos), pos_sb, 0,
            _lib.ptr(frequency), _lib.dtype_code(x), *x.shape, _lib.stream_of(x.device)))
    return out


class _Rotary(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, frequency, positions):
        ctx.save_for_backward(frequency, positions)
        return _rotary(x.contiguous() if x.stride(-1) != 1 else x, frequency, positions)

    @staticmethod
    def backward(ctx, dout):
        frequency, positions = ctx.saved_tensors
        # the transpose of a rotation by a is the rotation by -a
        return _rotary(dout.contiguous(), -frequency, positions), None, None


class RotaryEmbedding(nn.Module):
    def __init__(self, head_dim, base, fraction):
        super().__init__()
        if head_dim % 2:
            raise ValueError("RoPE needs an even head dimension")
        self.register_buffer("theta", rotary_frequencies(head_dim, base, fraction).reshape(1, -1), persistent=False)

    def forward(self, x, positions):
        if not x.is_cuda:
            raise ValueError("nlogn_pisa_b200 runs on CUDA tensors only; there is no CPU path")
        frequency = self.theta.flatten().to(device=x.device, dtype=torch.float32).contiguous()
        return _Rotary.apply(x, frequency, positions)


class PyramidSparseAttention(nn.Module):
    """Drop-in PISA token mixer (same parameter names, forward signature and cache layout)."""

    METHODS = ("pisa1", "pisa2", "pisa")

    def __init__(self, config, layer_idx=0):
        super().__init__()
        if config.attention_method not in self.METHODS:
            raise ValueError(f"attention_method {config.attention_method!r} is not served by nlogn_pisa_b200")
        self.config = config
        self.layer_idx = layer_idx
        # pyramid branching: the reference's is 2; a config may ask for 4 (this library's extension)
        self.branching = getattr(config, "branching", 2)
        q_width = config.num_attention_heads * config.head_dim
        kv_width = config.num_key_value_heads * config.head_dim
        self.q_proj = nn.Linear(config.hidden_size, q_width, bias=config.bias)
        self.k_proj = nn.Linear(config.hidden_size, kv_width, bias=config.bias)
        self.v_proj = nn.Linear(config.hidden_size, kv_width, bias=config.bias)
        self.o_proj = nn.Linear(q_width, config.hidden_size, bias=config.bias)
        self.rope = RotaryEmbedding(config.head_dim, config.rope_theta, config.rope_fraction)

    def forward(self, x, cu_seqlens=None, cache=None, use_cache=False, backend=None, attention_mask=None,
                past_key_values=None, **kwargs):
        if attention_mask is not None and not bool(attention_mask.all()):
            raise ValueError("Remove evaluation padding before native attention")
        if past_key_values is not None:
            cache = past_key_values[self.layer_idx] if len(past_key_values) > self.layer_idx else None
        cfg = self.config
        batch, length, _ = x.shape
        q = self.q_proj(x).view(batch, length, cfg.num_attention_heads, cfg.head_dim)
        raw_k = self.k_proj(x).view(batch, length, cfg.num_key_value_heads, cfg.head_dim)
        v = self.v_proj(x).view(batch, length, cfg.num_key_value_heads, cfg.head_dim)
        offset = 0 if cache is None else cache["k"].shape[1]
        boundaries = cu_seqlens if cfg.rope_position_mode == "document" else None
        positions = token_positions(length, x.device, boundaries, offset)
        q = self.rope(q, positions)
        k = self.rope(raw_k, positions)
        pyramid = None
        next_cache = None
        if use_cache:
            next_cache = {} if cache is None else cache
            pyramid = (PyramidCache.from_keys(k.detach(), block_size=cfg.block_size, branching=self.branching)
                       if cache is None else cache["pyramid"].append(k.detach()))
            next_cache["pyramid"] = pyramid
            values = TensorCache.from_tensor(v.detach()) if cache is None else cache["value_storage"].append(v.detach())
            k, v = pyramid.keys, values.tensor
            next_cache.update(k=k, v=v, value_storage=values)
        elif cache is not None:
            k = torch.cat((cache["k"], k), dim=1)
            v = torch.cat((cache["v"], v), dim=1)
        schedule = "fused" if cache is not None and length == 1 else (cfg.prefill_routing or "auto")
        indices = select_blocks(q.detach(), k.detach(), method=cfg.attention_method, block_size=cfg.block_size,
                                topk=cfg.topk, cu_seqlens=cu_seqlens, query_offset=offset,
                                force_first=cfg.force_first, force_recent=cfg.force_recent, pyramid=pyramid,
                                leaf_tile=cfg.leaf_tile, routing_schedule=schedule, branching=self.branching)
        output = sparse_attention(q, k, v, indices, block_size=cfg.block_size, cu_seqlens=cu_seqlens,
                                  query_offset=offset)
        if past_key_values is not None and use_cache:
            while len(past_key_values) <= self.layer_idx:
                past_key_values.append(None)
            past_key_values[self.layer_idx] = next_cache
            next_cache = past_key_values
        return self.o_proj(output.reshape(batch, length, -1)), next_cache
