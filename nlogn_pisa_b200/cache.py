"""Decode-time caches: growing token storage and a key pyramid kept current on the GPU.

The duck type is the one that ``select_blocks(pyramid=...)`` reads from the
reference's xmixers cache (xmixers/xmixers/utils/attention_cache.py:50-140):
``storage`` [B, sum of level capacities, H, D], ``starts`` (host) and
``offsets`` / ``lengths`` (int32 device tensors) per level, ``level_sizes``,
``levels`` and ``keys``.  The implementation is this library's own:

* keys live in a token buffer whose capacity grows in whole pages of leaf
  blocks by half of its size (amortised O(1) appends, no power-of-two
  rounding of long prompts);
* the pyramid storage is laid out by ``layout.storage_layout`` for the leaf
  capacity of that buffer, so the two grow together and a regrowth copies
  the finished levels once;
* ``append`` recomputes only the leaves touched by the new tokens and their
  ancestors in one library call (``pisa_pyramid_update``).
"""

from __future__ import annotations

import torch

from . import _lib
from .layout import level_sizes, storage_layout


def _grown_capacity(needed, current, page):
    """Next capacity for ``needed`` tokens: 1.5x growth, whole pages."""
    target = max(needed, current + current // 2)
    return -(-target // page) * page


class _TokenBuffer:
    """[B, capacity, H, D] storage with a valid prefix of ``length`` tokens."""

    def __init__(self, page):
        self.page = page
        self.data = None
        self.length = 0

    def view(self):
        if self.data is None:
            raise ValueError("the token cache is empty")
        return self.data[:, : self.length]

    def check_like(self, tensor):
        if tensor.ndim != 4 or tensor.shape[1] == 0 or not tensor.is_floating_point():
            raise ValueError("new tokens must be a nonempty [B,T,H,D] floating tensor")
        d = self.data
        if d is not None and (d.shape[0], d.shape[2], d.shape[3], d.dtype, d.device) != (
                tensor.shape[0], tensor.shape[2], tensor.shape[3], tensor.dtype, tensor.device):
            raise ValueError("cache batch, heads, dimension, dtype and device cannot change")

    def ensure(self, needed, like):
        """Grow to hold ``needed`` tokens; returns True when storage moved."""
        cap = 0 if self.data is None else self.data.shape[1]
        if needed <= cap:
            return False
        fresh = like.new_empty((like.shape[0], _grown_capacity(needed, cap, self.page), *like.shape[2:]))
        if self.length:
            fresh[:, : self.length] = self.data[:, : self.length]
        self.data = fresh
        return True

    def write(self, tensor):
        end = self.length + tensor.shape[1]
        self.data[:, self.length:end] = tensor
        self.length = end


class TensorCache:
    """Append-only detached token storage (the reference's value cache API)."""

    def __init__(self, page=256):
        self._buf = _TokenBuffer(page)

    @classmethod
    def from_tensor(cls, tensor):
        return cls().append(tensor)

    @property
    def buffer(self):
        return self._buf.data

    @property
    def length(self):
        return self._buf.length

    @property
    def tensor(self):
        return self._buf.view()

    @torch.no_grad()
    def append(self, tensor):
        self._buf.check_like(tensor)
        self._buf.ensure(self._buf.length + tensor.shape[1], tensor)
        self._buf.write(tensor)
        return self


class PyramidCache:
    """Key cache plus its mean pyramid (leaf blocks of ``block_size`` tokens,
    ``branching`` children per node), updated incrementally on the GPU."""

    def __init__(self, block_size=64, branching=2):
        if block_size < 1:
            raise ValueError("block_size must be positive")
        if branching < 2:
            raise ValueError("branching must be at least 2")
        self.block_size = block_size
        self.branching = branching
        # pages of 16 leaf blocks: a regrowth never splits a leaf
        self._keys = _TokenBuffer(16 * block_size)
        self.storage = None
        self.capacities = ()
        self.starts = ()
        self._sizes = ()
        self.offsets = None
        self.lengths = None

    @classmethod
    def from_keys(cls, keys, block_size=64, branching=2):
        return cls(block_size, branching).append(keys)

    # --- the duck type read by select_blocks(pyramid=...) ---
    @property
    def length(self):
        return self._keys.length

    @property
    def key_buffer(self):
        return self._keys.data

    @property
    def keys(self):
        return self._keys.view()

    @property
    def level_sizes(self):
        return self._sizes

    @property
    def buffers(self):
        if self.storage is None:
            return []
        return [self.storage[:, s:s + c] for s, c in zip(self.starts, self.capacities)]

    @property
    def levels(self):
        return [self.storage[:, s:s + n] for s, n in zip(self.starts, self._sizes)]

    def _relayout(self, like):
        """Pyramid storage for the key buffer's leaf capacity; finished levels move over."""
        leaf_cap = -(-self._keys.data.shape[1] // self.block_size)
        capacities, starts, total = storage_layout(leaf_cap, self.branching)
        fresh = like.new_empty((like.shape[0], total, *like.shape[2:]))
        if self.storage is not None:
            for old_start, new_start, n in zip(self.starts, starts, self._sizes):
                fresh[:, new_start:new_start + n] = self.storage[:, old_start:old_start + n]
        self.storage, self.capacities, self.starts = fresh, capacities, starts
        self.offsets = torch.tensor(starts, dtype=torch.int32, device=like.device)
        self.lengths = torch.zeros(len(starts), dtype=torch.int32, device=like.device)

    @torch.no_grad()
    def append(self, keys):
        if not keys.is_cuda:
            raise ValueError("nlogn_pisa_b200 runs on CUDA tensors only; there is no CPU path")
        self._keys.check_like(keys)
        first_new = self._keys.length
        moved = self._keys.ensure(first_new + keys.shape[1], keys)
        self._keys.write(keys)
        if moved or self.storage is None:
            self._relayout(keys)
        full = self.keys
        batch, length, heads, dim = full.shape
        with torch.cuda.device(full.device):
            _lib.check(_lib.lib().pisa_pyramid_update(
                _lib.ptr(full), _lib.dtype_code(full), batch, length, heads, dim, *full.stride()[:3],
                self.block_size, self.branching, len(self.starts), _lib.ptr(self.storage),
                self.storage.stride(0), _lib.int64_array(self.starts), first_new,
                _lib.stream_of(full.device)))
        sizes = level_sizes(-(-length // self.block_size), self.branching, len(self.starts))
        self._sizes = tuple(sizes)
        self.lengths.copy_(torch.tensor(sizes, dtype=torch.int32), non_blocking=True)
        return self
