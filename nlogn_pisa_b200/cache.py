"""Incremental key / pyramid caches for decoding.

Mirrors TensorCache and PyramidCache of the reference's token-mixer package
(xmixers/xmixers/utils/attention_cache.py:8-140): geometric token storage and
one pyramid allocation [B, sum(capacities), H, D] whose level offsets change
only when the leaf capacity grows.  ``append`` recomputes only the changed
leaves and their ancestors, on the GPU (pisa_pyramid_update).  The object
exposes ``storage``, ``offsets``/``lengths`` (int32 device tensors, as the
reference), ``starts`` and ``level_sizes`` (host), so select_blocks can use it
as ``pyramid=``.
"""

from __future__ import annotations

import torch

from . import _lib
from .selection import _c_array


class TensorCache:
    """Append-only, detached [B,T,H,D] storage with power-of-two capacity."""

    def __init__(self):
        self.buffer = None
        self.length = 0

    @classmethod
    def from_tensor(cls, tensor):
        return cls().append(tensor)

    @property
    def tensor(self):
        if self.buffer is None:
            raise ValueError("the token cache is empty")
        return self.buffer[:, : self.length]

    @torch.no_grad()
    def append(self, tensor):
        if tensor.ndim != 4 or tensor.shape[1] == 0 or not tensor.is_floating_point():
            raise ValueError("new tokens must be a nonempty [B,T,H,D] floating tensor")
        if self.buffer is not None:
            old = self.buffer
            if (old.shape[0], *old.shape[2:], old.dtype, old.device) != (
                    tensor.shape[0], *tensor.shape[2:], tensor.dtype, tensor.device):
                raise ValueError("cache batch, heads, dimension, dtype and device cannot change")
        end = self.length + tensor.shape[1]
        if self.buffer is None or end > self.buffer.shape[1]:
            capacity = 1 << (end - 1).bit_length()
            grown = tensor.new_empty(tensor.shape[0], capacity, *tensor.shape[2:])
            if self.buffer is not None:
                grown[:, : self.length].copy_(self.tensor)
            self.buffer = grown
        self.buffer[:, self.length:end].copy_(tensor)
        self.length = end
        return self


class PyramidCache:
    """Key cache plus its mean pyramid, updated incrementally on the GPU."""

    def __init__(self, block_size=64, branching=2):
        if block_size < 1:
            raise ValueError("block_size must be positive")
        if branching < 2:
            raise ValueError("branching must be at least 2")
        self.block_size = block_size
        self.branching = branching
        self.tokens = TensorCache()
        self.storage = None
        self.capacities = ()
        self.starts = ()
        self.sizes = []
        self.offsets = None
        self.lengths = None

    @classmethod
    def from_keys(cls, keys, block_size=64, branching=2):
        return cls(block_size, branching).append(keys)

    @property
    def length(self):
        return self.tokens.length

    @property
    def key_buffer(self):
        return self.tokens.buffer

    @property
    def keys(self):
        return self.tokens.tensor

    @property
    def level_sizes(self):
        return tuple(self.sizes)

    @property
    def buffers(self):
        if self.storage is None:
            return []
        return [self.storage[:, s:s + c] for s, c in zip(self.starts, self.capacities)]

    @property
    def levels(self):
        return [buffer[:, :size] for buffer, size in zip(self.buffers, self.sizes)]

    def reserve(self, reference, leaves):
        if self.capacities and leaves <= self.capacities[0]:
            return
        capacity = 1 << (leaves - 1).bit_length()
        capacities, starts, total = [], [], 0
        while capacity:
            capacities.append(capacity)
            starts.append(total)
            total += capacity
            capacity = 0 if capacity == 1 else -(-capacity // self.branching)
        storage = reference.new_empty(reference.shape[0], total, *reference.shape[2:])
        for start, previous in zip(starts, self.levels):
            storage[:, start:start + previous.shape[1]].copy_(previous)
        self.storage = storage
        self.capacities, self.starts = tuple(capacities), tuple(starts)
        self.offsets = torch.tensor(starts, device=reference.device, dtype=torch.int32)
        self.lengths = torch.empty(len(starts), device=reference.device, dtype=torch.int32)

    @torch.no_grad()
    def append(self, keys):
        if not keys.is_cuda:
            raise ValueError("nlogn_pisa_b200 runs on CUDA tensors only; there is no CPU path")
        previous = self.length
        self.tokens.append(keys)
        leaves = -(-self.length // self.block_size)
        self.reserve(keys, leaves)
        sizes, n = [], leaves
        for _ in self.capacities:
            sizes.append(n)
            n = -(-n // self.branching)
        full = self.keys
        code = _lib.dtype_code(full)
        batch, length, heads, dim = full.shape
        with torch.cuda.device(full.device):
            _lib.check(_lib.lib().pisa_pyramid_update(
                _lib.ptr(full), code, batch, length, heads, dim, *full.stride()[:3], self.block_size,
                self.branching, len(self.capacities), _lib.ptr(self.storage), self.storage.stride(0),
                _c_array(self.starts), previous, _lib.stream_of(full.device)))
        self.sizes = sizes
        self.lengths.copy_(torch.tensor(sizes, dtype=torch.int32), non_blocking=True)
        return self
