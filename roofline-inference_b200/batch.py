"""Batched ragged decode of the Qwen3 forward: up to S independent sequences,
each in its own contiguous cache of its own capacity, decoding one token each
per step (engine.py:33-40 and :145-163 generalised to many sequences; the
reference engine is single-stream).

Per step and layer: norm + QKV GEMM over the S rows (cuBLAS up to 64 rows), the batched
qk-norm + RoPE + append (each sequence at its own position, into its own
cache), split-KV decode attention over the per-sequence caches (lengths on
the device), O GEMM + residual/RMSNorm (add_rms), gate/up GEMM + SwiGLU, down
GEMM; then the final norm, the LM head with FP32 logits and a per-row argmax.
With S rows the projections are GEMMs that read each weight once per step for
all S tokens, so the weight traffic of a step is shared by the batch.

SlotDecoder keeps S slots whose per-row state (cache pointers per layer,
capacity, position, key count, active flag, input token) lives in fixed
device tensors, so sequences join and leave between steps by rewriting one
slot, and a captured CUDA graph of the step stays valid.  An idle slot
points at a one-page scratch cache, stays at position 0 (positions advance
by the active flag) and its outputs are ignored.
"""
from __future__ import annotations

import torch

from . import _lib
from ._tensors import HEAD_DIM, stream_handle
from .cache import Cache
from .gemm import gemm
from .kernels import add_rms, embedding, rms_norm, swiglu


def _linear(x, W, epi: str = "bf16"):
    """x W^T for the S rows of a step.  Up to 64 rows cuBLAS (a plain library
    GEMM) is faster than both of this package's GEMMs: timed as CUDA graphs
    of 28 calls at M = 16-64 it takes 3.5-8.3 us per Qwen3 projection, the
    few-row tcgen05 GEMM (gemm.py) 7.7-8.1 us (two launches), the tiled one
    9-21 us.  Above 64 rows the tiled tcgen05 GEMM, SwiGLU fused."""
    if x.shape[0] > 64:
        return gemm(x, W, epi=epi)
    y = torch.matmul(x, W.t())
    return swiglu(y) if epi == "swiglu" else y


class SlotDecoder:
    """Decode steps over `slots` sequence slots.  `max_n` bounds every
    member's cache capacity (it sizes the attention grid)."""

    def __init__(self, engine, slots: int, max_n: int):
        if engine.world != 1:
            raise ValueError("batched decode runs on one GPU")
        if slots < 1 or max_n < 1:
            raise ValueError("need at least one slot and max_n >= 1")
        cfg, dev = engine.cfg, engine.device
        self.e, self.device, self.B = engine, dev, slots
        self.L = L = _lib.load()
        self.scratch = engine.new_cache(1)                                     # idle slots' target
        self.caches: list[Cache | None] = [None] * slots
        self.ptrs = torch.tensor([[self.scratch.kv[l].data_ptr()] * slots for l in range(cfg.num_layers)],
                                 dtype=torch.int64, device=dev)                  # [layers, S]
        self.caps = torch.full((slots,), self.scratch.capacity, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(slots, dtype=torch.int32, device=dev)
        self.lens = torch.ones(slots, dtype=torch.int32, device=dev)
        self.active = torch.zeros(slots, dtype=torch.int32, device=dev)
        self.tok = torch.zeros(slots, dtype=torch.int32, device=dev)             # next input tokens
        self.max_n = max(int(max_n), self.scratch.capacity)
        ws = int(L.rib_decode_workspace_bytes(slots, self.max_n, engine.n_kv))
        self.ws = torch.zeros(max(ws, 1 << 20), dtype=torch.uint8, device=dev)  # counters zero
        self.q = torch.empty((slots, engine.nq_local, HEAD_DIM), dtype=torch.bfloat16, device=dev)
        self.o = torch.empty((slots, engine.nq_local, HEAD_DIM), dtype=torch.bfloat16, device=dev)
        self.next = torch.empty(slots, dtype=torch.int32, device=dev)
        self.graph = None
        self.graph_logits = None
        # per layer: 4 projections (+ a SwiGLU launch up to 64 rows; above, the
        # tiled GEMM fuses it), append, attention, 2 add_rms
        per_layer = 4 + (1 if slots <= 64 else 0) + 4
        self.launches_per_step = per_layer * cfg.num_layers + 8

    # ---------------------------------------------------------------- membership
    def _slot_ptrs(self, cache: Cache) -> torch.Tensor:
        return torch.tensor([kv.data_ptr() for kv in cache.kv], dtype=torch.int64, device=self.device)

    def set_slot(self, i: int, cache: Cache, token) -> None:
        """Slot i decodes `cache` from its offset, next input `token` (int or
        int32 CUDA scalar)."""
        if self.caches[i] is not None:
            raise ValueError(f"slot {i} is busy")
        if cache.capacity > self.max_n:
            raise ValueError(f"cache capacity {cache.capacity} exceeds max_n {self.max_n}")
        if len(cache.kv) != len(self.e.layers) or cache.n_kv != self.e.n_kv:
            raise ValueError("cache does not match the engine's layers / KV heads")
        self.ptrs[:, i] = self._slot_ptrs(cache)
        self.caps[i] = cache.capacity
        self.pos[i] = cache.offset
        self.lens[i] = cache.offset + 1
        self.active[i] = 1
        if isinstance(token, torch.Tensor):
            self.tok[i:i + 1].copy_(token.reshape(-1)[:1])
        else:
            self.tok[i] = int(token)
        self.caches[i] = cache

    def clear_slot(self, i: int) -> Cache | None:
        """Slot i goes idle; returns the cache it held (offset up to date)."""
        c = self.caches[i]
        self.caches[i] = None
        self.ptrs[:, i] = self._slot_ptrs(self.scratch)
        self.caps[i] = self.scratch.capacity
        self.pos[i] = 0
        self.lens[i] = 1
        self.active[i] = 0
        return c

    def free_slots(self) -> list[int]:
        return [i for i, c in enumerate(self.caches) if c is None]

    def _check_capacity(self):
        if any(c is not None and c.offset + 1 > c.capacity for c in self.caches):
            raise ValueError("KV capacity exceeded")

    def _advance_host(self):
        for c in self.caches:
            if c is not None:
                c.offset += 1

    # ---------------------------------------------------------------- the step
    def _forward(self):
        """The device work of one step on the slots' input tokens; returns the
        FP32 logits [S, vocab].  Positions and key counts of active slots
        advance on the device."""
        e, B = self.e, self.B
        st = stream_handle(self.device)
        h = embedding(e.embed, self.tok)                                     # [S, hidden]
        x = rms_norm(h, e.layers[0]["in_norm"])
        nl = len(e.layers)
        for l, w in enumerate(e.layers):
            qkv = _linear(x, w["qkv"])
            _lib.check(self.L.rib_qk_norm_rope_append_batched(
                qkv.data_ptr(), w["q_norm"].data_ptr(), w["k_norm"].data_ptr(), self.pos.data_ptr(),
                self.ptrs[l].data_ptr(), self.caps.data_ptr(), B, e.nq_local, e.n_kv, float(e.base),
                self.q.data_ptr(), st), "qk_norm_rope_append_batched")
            _lib.check(self.L.rib_decode_attention_ragged(
                self.q.data_ptr(), self.ptrs[l].data_ptr(), self.caps.data_ptr(), self.lens.data_ptr(), B,
                self.max_n, e.nq_local, e.n_kv, float(e.scale), self.o.data_ptr(), self.ws.data_ptr(),
                self.ws.numel(), st), "decode_attention_ragged")
            h, x = add_rms(h, _linear(self.o.reshape(B, -1), w["o"]), w["post_norm"])
            r = _linear(_linear(x, w["gu"], "swiglu"), w["down"])
            if l == nl - 1:
                h = h + r
            else:
                h, x = add_rms(h, r, e.layers[l + 1]["in_norm"])
        hn = rms_norm(h, e.final_norm)
        out = torch.mm(hn, e.embed.t(), out_dtype=torch.float32)            # [S, vocab]
        self.pos.add_(self.active)
        self.lens.add_(self.active)
        return out

    def _argmax(self, lg):
        _lib.check(self.L.rib_argmax_rows_f32(lg.data_ptr(), self.B, lg.shape[1], self.next.data_ptr(),
                                              stream_handle(self.device)), "argmax_rows")

    def capture(self):
        """Records one whole step (forward, row argmax, next inputs: 9 launches
        per layer, 8 more per step; cuBLAS may add split-K reductions) in a CUDA graph;
        later steps replay it, so a step costs one host launch.  Every input
        of the step lives in a fixed device buffer, and the GEMM shapes
        depend only on the slot count, so one graph serves every position and
        every membership.  Replays on the stream current at capture time."""
        self._check_capacity()
        dev = self.device
        self.stream = torch.cuda.current_stream(dev)
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(self.stream)
        with torch.cuda.stream(side):
            # Warm-up outside the graph (first-call set-up of cuBLAS and every
            # launch).  It appends K/V at each active slot's next position,
            # which the next real step overwrites before any attention reads
            # it; the device positions are then wound back.
            self._argmax(self._forward())
            self.pos.sub_(self.active)
            self.lens.sub_(self.active)
        self.stream.wait_stream(side)
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(graph, stream=side):
            self.graph_logits = self._forward()                  # FP32 [S, vocab] of the last replay
            self._argmax(self.graph_logits)
            self.tok.copy_(self.next)
        self.stream.wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = graph
        return self

    def run_step(self) -> torch.Tensor:
        """One step of every active slot on the tokens in `tok`; the next
        greedy tokens land in `next` (int32 [S], device), which is returned,
        and become the next step's inputs in `tok`.  Idle slots' entries are
        meaningless."""
        self._check_capacity()
        if self.graph is None:
            self._argmax(self._forward())
            self.tok.copy_(self.next)
        else:
            self.graph.replay()
        self._advance_host()
        return self.next

    def run_logits(self) -> torch.Tensor:
        """One eager step; returns the FP32 logits [S, vocab]."""
        self._check_capacity()
        out = self._forward()
        self._advance_host()
        return out


class BatchDecoder(SlotDecoder):
    """Decode steps for the sequences held in `caches` (one Cache each, same
    layer count and KV heads, any capacities), one slot per cache.
    Positions start at each cache's offset and advance by one per step, on
    the device and in the caches' offsets."""

    def __init__(self, engine, caches: list[Cache]):
        if not caches:
            raise ValueError("no sequences")
        super().__init__(engine, len(caches), max(c.capacity for c in caches))
        for i, c in enumerate(caches):
            self.set_slot(i, c, 0)

    def logits(self, tokens):
        """One step for every sequence: appends its token's K/V at its position
        and returns the FP32 logits [B, vocab] of the next token."""
        self.tok.copy_(tokens.reshape(-1))
        return self.run_logits()

    def step(self, tokens):
        """One step; returns the next greedy token of every sequence, int32 [B]."""
        self.tok.copy_(tokens.reshape(-1))
        return self.run_step().clone()


def generate_batch(engine, prompts: list[list[int]], max_tokens: int, eos_ids=(),
                   use_graph: bool = True) -> list[list[int]]:
    """Greedy generation for several prompts at once: each prompt is
    prefilled into its own cache (sized to its prompt + max_tokens), then all
    sequences decode together, one batched step per token.  A sequence stops
    recording at an end-of-sequence id or after max_tokens tokens.  With
    use_graph the batched step is replayed from a CUDA graph."""
    if not prompts or max_tokens < 1:
        raise ValueError("need prompts and max_tokens >= 1")
    from .kernels import argmax
    eos_ids = set(eos_ids)
    dev = engine.device
    caches, first = [], []
    for p in prompts:
        if not p or min(p) < 0 or max(p) >= engine.cfg.vocab_size:
            raise ValueError("every prompt needs tokens inside the vocabulary")
        c = engine.new_cache(len(p) + max_tokens + 1)
        lg = engine.prefill(torch.tensor(p, dtype=torch.int32, device=dev), c, last=True)
        first.append(argmax(lg.reshape(-1)))
        caches.append(c)
    tok = torch.cat(first)
    dec = BatchDecoder(engine, caches)
    if use_graph and max_tokens > 1:
        dec.capture()
    out: list[list[int]] = [[] for _ in prompts]
    done = [False] * len(prompts)
    for t in range(max_tokens):
        host = tok.cpu().tolist()
        for i, v in enumerate(host):
            if not done[i]:
                out[i].append(v)
                done[i] = v in eos_ids or len(out[i]) >= max_tokens
        if all(done) or t + 1 == max_tokens:
            break
        tok = dec.step(tok)
    return out
