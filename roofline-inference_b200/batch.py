"""Batched ragged decode of the Qwen3 forward: B independent sequences, each in
its own contiguous cache of its own capacity, decoding one token each per
step (engine.py:33-40 and :145-163 generalised to many sequences; the
reference engine is single-stream).

Per step and layer: norm + QKV GEMM over the B rows (cuBLAS), the batched
qk-norm + RoPE + append (each sequence at its own position, into its own
cache), split-KV decode attention over the per-sequence caches (lengths on
the device), O GEMM + residual/RMSNorm (add_rms), gate/up GEMM + SwiGLU, down
GEMM; then the final norm, the LM head with FP32 logits and a per-row argmax.
With B rows the projections are GEMMs that read each weight once per step for
all B tokens, so the weight traffic of a step is shared by the batch.
"""
from __future__ import annotations

import torch

from . import _lib
from ._tensors import HEAD_DIM, stream_handle
from .cache import Cache
from .kernels import add_rms, embedding, rms_norm, swiglu


def _linear(x, W):
    return torch.matmul(x, W.t())


class BatchDecoder:
    """Decode steps for the sequences held in `caches` (one Cache each, same
    layer count and KV heads, any capacities).  Positions start at each
    cache's offset and advance by one per step, on the device and in the
    caches' offsets."""

    def __init__(self, engine, caches: list[Cache]):
        if engine.world != 1:
            raise ValueError("batched decode runs on one GPU")
        if not caches:
            raise ValueError("no sequences")
        cfg, dev = engine.cfg, engine.device
        self.e, self.caches, self.device = engine, caches, dev
        self.B = len(caches)
        L = _lib.load()
        self.L = L
        self.ptrs = torch.tensor([[c.kv[l].data_ptr() for c in caches] for l in range(cfg.num_layers)],
                                 dtype=torch.int64, device=dev)                  # [layers, B]
        self.caps = torch.tensor([c.capacity for c in caches], dtype=torch.int32, device=dev)
        self.pos = torch.tensor([c.offset for c in caches], dtype=torch.int32, device=dev)
        self.lens = self.pos + 1
        self.max_n = max(c.capacity for c in caches)
        ws = int(L.rib_decode_workspace_bytes(self.B, self.max_n, engine.n_kv))
        self.ws = torch.zeros(max(ws, 1 << 20), dtype=torch.uint8, device=dev)  # counters zero
        self.q = torch.empty((self.B, engine.nq_local, HEAD_DIM), dtype=torch.bfloat16, device=dev)
        self.o = torch.empty((self.B, engine.nq_local, HEAD_DIM), dtype=torch.bfloat16, device=dev)
        self.next = torch.empty(self.B, dtype=torch.int32, device=dev)

    def logits(self, tokens):
        """One step for every sequence: appends its token's K/V at its position
        and returns the FP32 logits [B, vocab] of the next token."""
        e, B = self.e, self.B
        if any(c.offset + 1 > c.capacity for c in self.caches):
            raise ValueError("KV capacity exceeded")
        st = stream_handle(self.device)
        h = embedding(e.embed, tokens.reshape(-1))                          # [B, hidden]
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
            r = _linear(swiglu(_linear(x, w["gu"])), w["down"])
            if l == nl - 1:
                h = h + r
            else:
                h, x = add_rms(h, r, e.layers[l + 1]["in_norm"])
        hn = rms_norm(h, e.final_norm)
        out = torch.mm(hn, e.embed.t(), out_dtype=torch.float32)            # [B, vocab]
        self.pos.add_(1)
        self.lens.add_(1)
        for c in self.caches:
            c.offset += 1
        return out

    def step(self, tokens):
        """One step; returns the next greedy token of every sequence, int32 [B]."""
        lg = self.logits(tokens)
        _lib.check(self.L.rib_argmax_rows_f32(lg.data_ptr(), self.B, lg.shape[1], self.next.data_ptr(),
                                              stream_handle(self.device)), "argmax_rows")
        return self.next.clone()


def generate_batch(engine, prompts: list[list[int]], max_tokens: int, eos_ids=()) -> list[list[int]]:
    """Greedy generation for several prompts at once: each prompt is
    prefilled into its own cache (sized to its prompt + max_tokens), then all
    sequences decode together, one batched step per token.  A sequence stops
    recording at an end-of-sequence id or after max_tokens tokens."""
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
