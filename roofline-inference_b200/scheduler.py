"""Continuous batching of greedy generation requests on one GPU.

The reference serves one request at a time (Engine.generate,
agent-test/v2/engine.py:165-192: chunked prefill at a growing offset, then
one decode step per token).  Here many requests share the GPU:

  - every request gets its own contiguous cache of len(prompt) + max_tokens
    + 1 rows (engine.py:174) from a KVPool arena; a request that does not fit
    waits (first come, first served) until finished requests free space;
  - prompts are prefilled in chunks of at most `chunk` tokens at the cache's
    offset (engine.py:176-182), with at most `chunk` prompt tokens per
    scheduler step over all requests, so a long prompt never stalls the
    running sequences for more than one chunk;
  - the last chunk's logits give the first token (engine.py:183); the request
    then takes a free slot of a SlotDecoder, and every scheduler step runs
    one batched decode step (one CUDA-graph replay) for all slots;
  - a request finishes at an end-of-sequence id or after max_tokens tokens
    (engine.py:185-192); its slot and cache return at once.

Token order and the stopping rule per request are those of Engine.generate.
"""
from __future__ import annotations

import collections
from dataclasses import dataclass, field

import torch

from .batch import SlotDecoder
from .pool import KVPool, PoolFull


@dataclass
class Request:
    rid: int
    prompt: list[int]
    max_tokens: int
    eos_ids: frozenset
    out: list[int] = field(default_factory=list)
    cache: object = None
    prefilled: int = 0
    slot: int = -1
    pending: int = -1          # first token, waiting for a free slot
    done: bool = False
    reason: str = ""           # "eos" or "length"

    @property
    def capacity(self) -> int:
        return len(self.prompt) + self.max_tokens + 1


class Scheduler:
    """Serves submitted requests on `engine` (one GPU).

    pool_rows: cache rows of the KV arena shared by all requests.
    slots:     sequences decoded together per step.
    max_len:   largest capacity (prompt + max_tokens + 1) a request may ask
               for; it sizes the batched attention grid.
    chunk:     prefill chunk, and prompt tokens prefilled per step.
    """

    def __init__(self, engine, pool_rows: int, slots: int = 64, max_len: int = 8192, chunk: int = 4096,
                 use_graph: bool = True, pool=None, decoder=None, argmax_fn=None):
        if slots < 1 or max_len < 2 or chunk < 1:
            raise ValueError("need slots >= 1, max_len >= 2, chunk >= 1")
        self.e = engine
        self.pool = pool if pool is not None else KVPool.for_engine(engine, pool_rows)
        self.dec = decoder if decoder is not None else SlotDecoder(engine, slots, max_len)
        self.max_len, self.chunk, self.use_graph = max_len, chunk, use_graph
        if argmax_fn is None:
            from .kernels import argmax as argmax_fn
        self._argmax = argmax_fn
        self.waiting: collections.deque[Request] = collections.deque()
        self.prefilling: list[Request] = []
        self.ready: collections.deque[Request] = collections.deque()
        self.running: dict[int, Request] = {}
        self.finished: dict[int, Request] = {}
        self._next_id = 0
        self.steps = 0
        self.decode_steps = 0

    # ---------------------------------------------------------------- requests
    def submit(self, prompt: list[int], max_tokens: int = 65, eos_ids=()) -> int:
        """Queues a request; returns its id.  Argument checks of
        engine.py:166-169."""
        if not prompt or max_tokens < 0:
            raise ValueError("Nonempty prompt, nonnegative max_tokens required")
        if min(prompt) < 0 or max(prompt) >= self.e.cfg.vocab_size:
            raise ValueError("Token outside vocabulary")
        r = Request(self._next_id, [int(t) for t in prompt], int(max_tokens), frozenset(eos_ids))
        if r.capacity > self.max_len:  # rejected before it takes an id: ids stay consecutive
            raise ValueError(f"prompt + max_tokens + 1 = {r.capacity} exceeds max_len {self.max_len}")
        self._next_id += 1
        if max_tokens == 0:
            r.done, r.reason = True, "length"
            self.finished[r.rid] = r
        else:
            self.waiting.append(r)
        return r.rid

    @property
    def has_work(self) -> bool:
        return bool(self.waiting or self.prefilling or self.ready or self.running)

    def output(self, rid: int) -> list[int]:
        return self.finished[rid].out

    def _emit(self, r: Request, tok: int, events: list) -> None:
        r.out.append(tok)
        events.append((r.rid, tok))
        if tok in r.eos_ids:
            r.done, r.reason = True, "eos"
        elif len(r.out) >= r.max_tokens:
            r.done, r.reason = True, "length"

    def _retire(self, r: Request) -> None:
        if r.slot >= 0:
            self.dec.clear_slot(r.slot)
            self.running.pop(r.slot)
            r.slot = -1
        self.pool.free(r.cache)
        r.cache = None
        self.finished[r.rid] = r

    # ---------------------------------------------------------------- one step
    def step(self) -> list[tuple[int, int]]:
        """Admission, at most `chunk` prompt tokens of prefill, placement of
        prefilled requests into free slots, then one batched decode step.
        Returns the (request id, token) pairs produced, in order."""
        events: list[tuple[int, int]] = []
        self.steps += 1
        # 1. admission: first come, first served; the head of the queue waits
        #    for space rather than being overtaken.
        while self.waiting:
            r = self.waiting[0]
            try:
                r.cache = self.pool.allocate(r.capacity)
            except PoolFull:
                if not (self.prefilling or self.ready or self.running):
                    raise            # nothing will ever free space: the pool is too small for it
                break
            self.waiting.popleft()
            self.prefilling.append(r)
        # 2. chunked prefill at the cache offset, `chunk` tokens per step in all
        budget = self.chunk
        while self.prefilling and budget > 0:
            r = self.prefilling[0]
            a = r.prefilled
            b = min(len(r.prompt), a + min(budget, self.chunk))
            last = b == len(r.prompt)
            toks = torch.tensor(r.prompt[a:b], dtype=torch.int32).to(self.e.device, non_blocking=True)
            logits = self.e.prefill(toks, r.cache, last=last)
            r.prefilled = b
            budget -= b - a
            if not last:
                continue
            self.prefilling.pop(0)
            first = int(self._argmax(logits.reshape(-1)).reshape(-1)[0])
            self._emit(r, first, events)
            if r.done:
                self._retire(r)
            else:
                r.pending = first
                self.ready.append(r)
        # 3. prefilled requests take free slots
        free = self.dec.free_slots()
        while self.ready and free:
            r = self.ready.popleft()
            r.slot = free.pop(0)
            self.dec.set_slot(r.slot, r.cache, r.pending)
            self.running[r.slot] = r
        # 4. one decode step of every running sequence
        if self.running:
            if self.use_graph and getattr(self.dec, "graph", None) is None:
                self.dec.capture()
            nxt = self.dec.run_step().cpu().tolist()
            self.decode_steps += 1
            for slot in sorted(self.running):
                r = self.running[slot]
                self._emit(r, int(nxt[slot]), events)
                if r.done:
                    self._retire(r)
        return events

    def run(self) -> dict[int, list[int]]:
        """Steps until every submitted request has finished; returns the
        generated tokens per request id."""
        while self.has_work:
            self.step()
        return {rid: r.out for rid, r in sorted(self.finished.items())}
