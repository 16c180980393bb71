"""KV-cache allocator: one device arena of cache rows from which every
sequence gets its own contiguous cache (the reference's per-sequence Cache,
agent-test/v2/engine.py:33-40, carved out of a shared pool instead of one
allocation per request).

A row here is one token position of every layer: n_layers * 2 * n_kv *
head_dim BF16 values (28 * 2 * 8 * 128 * 2 B = 114,688 B for Qwen3-0.6B).  A
cache of capacity c (a multiple of 256 rows, engine.py:37) is the arena range
[start * row, (start + c) * row) viewed as [n_layers, 2, n_kv, c, head_dim],
which is the layout of a stand-alone Cache, so every kernel takes either.

Blocks are whole pages of 256 rows.  Allocation is best fit over a free list
kept sorted by start page; freeing merges a block with free neighbours.  The
arena is zeroed once at creation; a freed block keeps the finite K/V values
its last sequence wrote, and no kernel reads a row at or past a sequence's
length, so reuse needs no clearing.
"""
from __future__ import annotations

import bisect

import torch

from .cache import Cache

PAGE_ROWS = 256


class PoolFull(MemoryError):
    """No free block of the requested size (the caller may retry after frees)."""


class KVPool:
    """Arena of `rows` cache rows (rounded up to whole pages) on `device`."""

    def __init__(self, n_layers: int, n_kv: int, rows: int, head_dim: int = 128,
                 dtype=torch.bfloat16, device=None):
        if n_layers < 1 or n_kv < 1 or head_dim < 1 or rows < 1:
            raise ValueError("n_layers, n_kv, head_dim and rows must be positive")
        self.n_layers, self.n_kv, self.head_dim = n_layers, n_kv, head_dim
        self.pages = (rows + PAGE_ROWS - 1) // PAGE_ROWS
        self.row_elems = n_layers * 2 * n_kv * head_dim
        self.arena = torch.zeros(self.pages * PAGE_ROWS * self.row_elems, dtype=dtype, device=device)
        self._free: list[tuple[int, int]] = [(0, self.pages)]     # (start page, pages), sorted by start
        self._used: dict[int, tuple[int, int]] = {}                # block token -> (start page, pages)
        self._next_token = 1

    @classmethod
    def for_engine(cls, engine, rows: int) -> "KVPool":
        return cls(engine.cfg.num_layers, engine.n_kv, rows, device=engine.device)

    @property
    def free_pages(self) -> int:
        return sum(n for _, n in self._free)

    @property
    def largest_free_rows(self) -> int:
        return max((n for _, n in self._free), default=0) * PAGE_ROWS

    def allocate(self, capacity: int) -> Cache:
        """A cache of at least `capacity` rows (offset 0).  Raises PoolFull
        when no free block is large enough."""
        if capacity < 1:
            raise ValueError("capacity must be positive")
        need = (capacity + PAGE_ROWS - 1) // PAGE_ROWS
        best = None
        for k, (start, n) in enumerate(self._free):
            if n >= need and (best is None or n < self._free[best][1]):
                best = k
        if best is None:
            raise PoolFull(f"no free block of {need} pages ({self.free_pages} free, "
                           f"largest {self.largest_free_rows // PAGE_ROWS})")
        start, n = self._free[best]
        if n == need:
            del self._free[best]
        else:
            self._free[best] = (start + need, n - need)
        rows = need * PAGE_ROWS
        a = start * PAGE_ROWS * self.row_elems
        view = self.arena[a:a + rows * self.row_elems].view(self.n_layers, 2, self.n_kv, rows, self.head_dim)
        cache = Cache.over(view)
        cache.pool_token = (id(self), self._next_token)
        self._used[self._next_token] = (start, need)
        self._next_token += 1
        return cache

    def free(self, cache: Cache) -> None:
        """Returns the cache's block to the pool; the cache must not be used
        afterwards."""
        token = getattr(cache, "pool_token", None)
        blk = self._used.pop(token[1], None) if token and token[0] == id(self) else None
        if blk is None:
            raise ValueError("cache was not allocated from this pool (or was freed already)")
        start, n = blk
        k = bisect.bisect_left(self._free, (start, 0))
        if k < len(self._free) and start + n == self._free[k][0]:      # merge with the next block
            n += self._free[k][1]
            del self._free[k]
        if k > 0 and self._free[k - 1][0] + self._free[k - 1][1] == start:   # and the previous one
            start, n = self._free[k - 1][0], self._free[k - 1][1] + n
            del self._free[k - 1]
            k -= 1
        self._free.insert(k, (start, n))
        cache.kv = []
        cache.capacity = 0
