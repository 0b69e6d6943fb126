"""Preallocated, API-compatible KV cache.

The reference passes ``past_kv = (past_k, past_v)`` to the attention and
builds ``k = cat(past_k, k)`` every step (REF modules/attention.py:89-93),
copying the whole history (1.07 GB per layer per step at 64 sequences x 8192
positions).  ``LayerKVCache`` holds one layer's K/V in buffers of a fixed
capacity, ``[B, Hkv, capacity, D]`` bf16; ``CudaFullAttention`` appends the new
rows in place (``q35_kv_append``) and attends over the buffers directly (the
attention kernels take the capacity as the per-head row stride).

Compatibility: a ``LayerKVCache`` unpacks and indexes like the ``(k, v)``
tuple of the reference API -- ``k, v = cache`` and ``cache[0]`` give views of
the valid rows ``[B, Hkv, length, D]`` -- and it is what the attention returns
as ``new_kv``.  ``KVCache`` is the per-model list (``past_key_values``).

The length advances on the host when the attention runs, so a cache is meant
for eager decode loops, one forward at a time.
"""
from __future__ import annotations

import torch


class LayerKVCache:
    def __init__(self, batch: int, num_kv_heads: int, capacity: int, head_dim: int,
                 device, dtype: torch.dtype = torch.bfloat16):
        if capacity < 1:
            raise ValueError("capacity must be positive")
        # zero-initialised: the last key tile of an attention call reads rows
        # past the valid length (masked), which must hold finite values
        self.k = torch.zeros(batch, num_kv_heads, capacity, head_dim, device=device, dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.length = 0

    @property
    def capacity(self) -> int:
        return self.k.shape[2]

    def views(self) -> tuple[torch.Tensor, torch.Tensor]:
        return self.k[:, :, :self.length], self.v[:, :, :self.length]

    def __iter__(self):
        return iter(self.views())

    def __getitem__(self, i):
        return self.views()[i]

    def __len__(self) -> int:
        return 2

    def reset(self) -> None:
        self.length = 0


class KVCache:
    """One ``LayerKVCache`` per attention layer; pass as ``past_key_values``."""

    def __init__(self, num_layers: int, batch: int, num_kv_heads: int, capacity: int,
                 head_dim: int, device, dtype: torch.dtype = torch.bfloat16):
        self.layers = [LayerKVCache(batch, num_kv_heads, capacity, head_dim, device, dtype)
                       for _ in range(num_layers)]

    def __getitem__(self, i) -> LayerKVCache:
        return self.layers[i]

    def __len__(self) -> int:
        return len(self.layers)

    def __iter__(self):
        return iter(self.layers)

    @property
    def length(self) -> int:
        return self.layers[0].length if self.layers else 0

    def reset(self) -> None:
        for layer in self.layers:
            layer.reset()
