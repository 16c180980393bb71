"""Preallocated BF16 KV cache with the interface of the reference's Cache
(agent-test/v2/engine.py:33-55), laid out for the B200 kernels.

All layers live in one device allocation [n_layers, 2, n_kv, cap, head_dim]:
per layer the K and V halves are each contiguous per KV head ([cap, 128] rows
of 256 bytes), which is what the split-KV decode kernel streams with 1-D bulk
copies and the prefill kernel tiles with TMA.  `cap` is the requested
capacity rounded up to a multiple of 256 (engine.py:37), e.g. 33024 for a
32768-token context plus new tokens.
"""
from __future__ import annotations

import torch

from . import kernels as _k


class Cache:
    """Preallocated per-layer KV buffer [2, n_kv, capacity, head_dim]."""

    def __init__(self, n_layers: int, n_kv: int, head_dim: int, capacity: int,
                 dtype=torch.bfloat16, device=None):
        if n_layers < 1 or n_kv < 1 or head_dim < 1 or capacity < 1:
            raise ValueError("n_layers, n_kv, head_dim and capacity must be positive")
        cap = (capacity + 255) // 256 * 256
        self.storage = torch.zeros((n_layers, 2, n_kv, cap, head_dim), dtype=dtype, device=device)
        self.kv = [self.storage[i] for i in range(n_layers)]
        self.offset = 0
        self.capacity = cap
        self.n_kv = n_kv
        self.head_dim = head_dim

    @classmethod
    def over(cls, storage: torch.Tensor) -> "Cache":
        """A cache over existing storage [n_layers, 2, n_kv, cap, head_dim]
        (e.g. rows of a KVPool arena); cap must be a multiple of 256."""
        if storage.dim() != 5 or storage.shape[1] != 2 or storage.shape[3] % 256 or not storage.is_contiguous():
            raise ValueError("storage must be contiguous [n_layers, 2, n_kv, cap % 256 == 0, head_dim]")
        c = cls.__new__(cls)
        c.storage = storage
        c.kv = [storage[i] for i in range(storage.shape[0])]
        c.offset = 0
        c.capacity = int(storage.shape[3])
        c.n_kv = int(storage.shape[2])
        c.head_dim = int(storage.shape[4])
        return c

    def update(self, i: int, kv: torch.Tensor) -> torch.Tensor:
        """Write kv [2, n_kv, n, d] at [offset, offset+n) (engine.py:42-48)."""
        a, b = self.offset, self.offset + kv.shape[2]
        if b > self.capacity:
            raise ValueError("KV capacity exceeded")
        self.kv[i][:, :, a:b, :] = kv
        return self.kv[i]

    def views(self, i: int, n: int):
        """K, V views [1, n_kv, n, d] of layer i (engine.py:50-52)."""
        buf = self.kv[i]
        return buf[0:1, :, :n, :], buf[1:2, :, :n, :]

    def state(self):
        return self.kv

    def append_qk_norm_rope(self, i: int, qkv, qw, kw, nq: int, base: float, Lp: int | None = None):
        """Fused path: norm + RoPE of qkv rows for positions offset.. and the
        K/V append into layer i, in one kernel.  Returns Q [nq, Lp, 128].
        Like update(), it does not advance `offset`; the engine does
        (engine.py:136, 159)."""
        return _k.qk_norm_rope_append(qkv, qw, kw, self.offset, nq, self.n_kv, base, self.kv[i], Lp)
