"""Qwen3 forward on B200 around the attention kernels: the reference's v2
engine (agent-test/v2/engine.py) restated for CUDA.

  Qwen3Config, random_weights(cfg, seed)   dense Qwen3 with tied embeddings
                                           (engine.py:58-88 preconditions)
  Engine(weights)
    .new_cache(capacity)                   Cache [L, 2, nkv, cap, 128]
    .prefill(tokens, cache, last=...)      engine.py:102-142
    .decode(token, cache)                  engine.py:145-163 (eager)
    .decode_graph(cache)                   the same step captured in a CUDA graph
    .generate(prompt, max_tokens, ...)     engine.py:165-192, one token of lookahead

Per decode step and layer the engine launches the reference's seven kernels
with two of them fused: norm + QKV GEMV, qk-norm + RoPE + KV append (one
kernel), split-KV decode attention, O GEMV + residual, norm + gate/up GEMV +
SwiGLU, down GEMV + residual; then the final norm + LM-head GEMV and argmax.
Prefill runs the projections on this library's tcgen05 GEMM (gemm.py) with
the QKV norm + RoPE + KV append and the SwiGLU fused into its epilogues, the
tcgen05 prefill kernel for attention and the add_rms kernel; as
in the reference, the last layer runs attention and MLP for the final row only
and the logits cover the final row only.
"""
from __future__ import annotations

import ctypes
import threading
from collections.abc import Iterator
from dataclasses import dataclass

import torch

from . import _lib
from .attention import attention, decode_attention
from .cache import Cache
from .kernels import (add_rms, argmax, embedding, gemv, qk_norm_rope_append, qk_norm_rope_append_at,
                      rms_norm, swiglu)
from ._tensors import HEAD_DIM, stream_handle
from .gemm import gemm, gemm_qkv_rope, rope_table


@dataclass(frozen=True)
class Qwen3Config:
    num_layers: int = 28
    hidden_size: int = 1024
    num_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 3072
    vocab_size: int = 151936
    rope_theta: float = 1e6
    rms_norm_eps: float = 1e-6

    def validate(self) -> None:
        """The kernels' preconditions (engine.py:69-70 plus the GEMV's K % 256)."""
        if self.head_dim != HEAD_DIM or self.num_heads != 2 * self.num_kv_heads:
            raise ValueError("Kernels assume head_dim 128 and GQA factor 2")
        if self.hidden_size % 256 or self.intermediate_size % 256 or (self.num_heads * 128) % 256:
            raise ValueError("hidden, intermediate and q widths must be multiples of 256")
        if abs(self.rms_norm_eps - 1e-6) > 1e-12:
            raise ValueError("the kernels' RMSNorm eps is 1e-6")

    @property
    def q_dim(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim


QWEN3_0_6B = Qwen3Config()


class Qwen3Weights:
    """BF16 weights in the engine's fused layout (engine.py:80-88): per layer
    qkv = [q_proj; k_proj; v_proj], gu = [gate_proj; up_proj], o, down and the
    four norm vectors; `embed` doubles as the LM head (tied)."""

    def __init__(self, config: Qwen3Config, embed, final_norm, layers: list[dict]):
        config.validate()
        self.config = config
        self.embed = embed
        self.final_norm = final_norm
        self.layers = layers

    def to(self, device) -> "Qwen3Weights":
        mv = lambda t: t.to(device)
        return Qwen3Weights(self.config, mv(self.embed), mv(self.final_norm),
                            [{k: mv(v) for k, v in l.items()} for l in self.layers])

    def nbytes(self) -> int:
        n = self.embed.numel() + self.final_norm.numel()
        n += sum(v.numel() for l in self.layers for v in l.values())
        return 2 * n


def random_weights(config: Qwen3Config = QWEN3_0_6B, seed: int = 0, device="cpu", std: float = 0.02,
                   norm_std: float = 0.1) -> Qwen3Weights:
    """Random-init weights: matrices N(0, std), norm weights 1 + N(0, norm_std),
    drawn from torch.Generator(device).manual_seed(seed) in a fixed order."""
    config.validate()
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    d, q, kv, f = config.hidden_size, config.q_dim, config.kv_dim, config.intermediate_size

    def mat(r, c):
        return (torch.randn((r, c), generator=g, device=dev) * std).to(torch.bfloat16)

    def norm(n):
        return (1.0 + norm_std * torch.randn((n,), generator=g, device=dev)).to(torch.bfloat16)

    embed = mat(config.vocab_size, d)
    layers = []
    for _ in range(config.num_layers):
        layers.append(dict(qkv=mat(q + 2 * kv, d), o=mat(d, q), gu=mat(2 * f, d), down=mat(d, f),
                           in_norm=norm(d), post_norm=norm(d), q_norm=norm(HEAD_DIM), k_norm=norm(HEAD_DIM)))
    return Qwen3Weights(config, embed, norm(d), layers)


def _linear(x, W, epi: str = "bf16"):
    """epi(x [m, k] @ W[n, k]^T) on this library's kernels (the reference's
    Engine.matmul, agent-test/v2/engine.py:95-99): the GEMV for one row, the
    tcgen05 GEMM (gemm.py) for more.  epi "bf16", "f32" or "swiglu"
    (W = [gate; up])."""
    if x.shape[0] == 1:
        return gemv(W, x.reshape(-1), swiglu=epi == "swiglu", out_float=epi == "f32").reshape(1, -1)
    return gemm(x, W, epi=epi)


def _shard_qkv_rows(W: torch.Tensor, h0: int, h1: int, nq: int, nkv: int) -> torch.Tensor:
    """Rows of a [(nq + 2 nkv) * 128, hidden] QKV weight for KV heads [h0, h1):
    their query heads, K heads and V heads, in the fused kernel's order."""
    x = W.reshape(nq + 2 * nkv, HEAD_DIM, W.shape[1])
    return torch.cat([x[2 * h0:2 * h1], x[nq + h0:nq + h1], x[nq + nkv + h0:nq + nkv + h1]]) \
        .reshape(-1, W.shape[1]).contiguous()


class Engine:
    """The Qwen3 forward on one GPU, or KV-head sharded over the ranks of a
    torch.distributed group (shard=True): rank r owns KV heads
    sharding.head_range(r, world) -- their rows of each QKV projection, their
    K/V cache and their attention -- and every rank receives every head's
    attention output (decode: the decode kernel's own NVLink stores; prefill:
    an NCCL all-gather), then runs the rest of the layer on the full hidden
    state, so all ranks hold the same activations and tokens.  Every rank
    makes the same calls in the same order.

    tp=True (implies shard) also splits the projections (tensor
    parallelism, tp.py): each rank keeps the O columns of its heads, a slice
    of the gate/up rows and down columns and a slice of the LM-head rows;
    attention outputs stay local, and the O / down partial sums and the argmax
    keys are exchanged over NVLink inside the GEMV and argmax kernels (prefill:
    the tcgen05 GEMM stores each row's FP32 partial to its owner rank, which
    reduces it and stores the BF16 row to every rank before the residual add
    and RMSNorm; tp.PrefillExchange)."""

    def __init__(self, weights: Qwen3Weights, *, shard: bool = False, tp: bool = False, group=None):
        cfg = weights.config
        cfg.validate()
        if not weights.embed.is_cuda:
            raise ValueError("weights must be on a CUDA device")
        _lib.load()  # fail loudly now if the CUDA library is missing
        self.cfg = cfg
        self.w = weights
        self.device = weights.embed.device
        self.n_heads = cfg.num_heads              # all query heads (the O projection's input)
        self.scale = HEAD_DIM ** -0.5
        self.base = cfg.rope_theta
        self.embed = weights.embed
        self.final_norm = weights.final_norm
        self.group = group
        self.world, self.rank = 1, 0
        self.gather = None
        self.tp = bool(tp)
        self.tpx = None
        self.tpp = None          # tensor-parallel prefill exchange, made by the first prefill
        if shard or tp:
            import torch.distributed as dist
            from .nvlink_gather import NVLinkGather
            from .sharding import head_range
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
            h0, h1 = head_range(self.rank, self.world, cfg.num_kv_heads)
        else:
            h0, h1 = 0, cfg.num_kv_heads
        self.n_kv = h1 - h0                       # KV heads of this rank
        self.nq_local = 2 * self.n_kv             # query heads of this rank
        self.lm_head, self.v0 = self.embed, 0
        if self.world > 1 and self.tp:
            from .tp import TPExchange, shard_layer, split_range
            f0, f1 = split_range(cfg.intermediate_size, self.rank, self.world)
            self.v0, v1 = split_range(cfg.vocab_size, self.rank, self.world)
            self.layers = [shard_layer(l, h0, h1, f0, f1, cfg.num_heads, cfg.num_kv_heads) for l in weights.layers]
            self.lm_head = self.embed[self.v0:v1]
            self.tpx = TPExchange(cfg.hidden_size, self.device, group)
        elif self.world > 1:
            self.layers = [dict(l, qkv=_shard_qkv_rows(l["qkv"], h0, h1, cfg.num_heads, cfg.num_kv_heads))
                           for l in weights.layers]
            self.gather = NVLinkGather(1, self.nq_local, self.device, group)
            self.epoch_dev = torch.zeros(1, dtype=torch.int64, device=self.device)
        else:
            self.tp = False
            self.layers = weights.layers
        self._sessions: dict = {}

    def new_cache(self, capacity: int) -> Cache:
        return Cache(self.cfg.num_layers, self.n_kv, HEAD_DIM, capacity, device=self.device)

    def close(self) -> None:
        """Collective when sharded: releases the NVLink gather buffers."""
        self._sessions.clear()
        if self.gather is not None:
            self.gather.close()
            self.gather = None
        if self.tpx is not None:
            self.tpx.close()
            self.tpx = None
        if self.tpp is not None:
            self.tpp.close()
            self.tpp = None

    def _attend_one(self, q, cache_layer, n: int, out=None):
        """Decode attention of one query row over n keys: [1, nq_local, 128] in,
        [1, n_heads, 128] out (all ranks' heads when KV-head sharded; this
        rank's heads under tensor parallelism)."""
        if self.world == 1 or self.tp:
            return decode_attention(q, cache_layer, n, self.scale).reshape(1, self.nq_local, HEAD_DIM)
        from .attention import decode_workspace
        L = _lib.load()
        ws = decode_workspace(self.device, int(L.rib_decode_workspace_bytes(1, n, self.n_kv)))
        ptrs = torch.tensor([cache_layer.data_ptr()], dtype=torch.int64, device=self.device)
        lens = torch.tensor([n], dtype=torch.int32, device=self.device)
        out = torch.empty((1, self.n_heads, HEAD_DIM), dtype=torch.bfloat16, device=self.device) \
            if out is None else out
        return self.gather.decode_into(q.reshape(1, self.nq_local, HEAD_DIM).contiguous(), ptrs, lens, n,
                                       cache_layer.shape[2], self.scale, ws, self.epoch_dev, out)

    def _prefill_exchange(self, rows: int):
        """The tensor-parallel prefill exchange, holding at least `rows` rows
        (collective: every rank prefills the same chunk lengths)."""
        if self.tpp is None or self.tpp.rows_cap < rows:
            from .tp import PrefillExchange
            if self.tpp is not None:
                self.tpp.close()
            self.tpp = PrefillExchange(self.cfg.hidden_size, max(rows, 4096), self.device, self.group)
        return self.tpp

    def _tp_add_rms(self, x, W, h, norm_w):
        """Under tensor parallelism: h <- bf16(h + bf16(sum over ranks of x W^T))
        in place over NVLink (tp.PrefillExchange); returns (h, RMSNorm(h) * norm_w),
        the second None when norm_w is None."""
        return self._prefill_exchange(x.shape[0]).project_add_rms(x.contiguous(), W, h, norm_w)

    def _gather_vocab(self, local):
        """[..., V/N] FP32 logit slices of every rank -> [..., V] (NCCL all-gather)."""
        import torch.distributed as dist
        parts = [torch.empty_like(local) for _ in range(self.world)]
        dist.all_gather(parts, local.contiguous(), group=self.group)
        return torch.cat(parts, dim=-1)

    def _gather_rows(self, o_local):
        """[n, nq_local * 128] per rank -> [n, n_heads * 128] (NCCL all-gather)."""
        if self.world == 1:
            return o_local
        import torch.distributed as dist
        n = o_local.shape[0]
        buf = torch.empty((self.world, n, o_local.shape[1]), dtype=o_local.dtype, device=o_local.device)
        dist.all_gather_into_tensor(buf, o_local.contiguous(), group=self.group)
        return buf.permute(1, 0, 2).reshape(n, -1)

    # ---------------- prefill (M >= 1) ----------------
    def prefill(self, tokens, cache: Cache, *, last: bool, all_logits: bool = False):
        """tokens: int32 CUDA [1, n] or [n].  Writes the K/V of every layer at
        [offset, offset+n) and advances cache.offset.  If `last`, returns the
        FP32 logits [1, 1, vocab] of the final row ([1, n, vocab] with
        all_logits), as engine.py:102-142."""
        tokens = tokens.reshape(-1)
        n = tokens.numel()
        off = cache.offset
        if off + n > cache.capacity:
            raise ValueError("KV capacity exceeded")
        Lp = (n + 31) // 32 * 32
        nl = len(self.layers)
        h = embedding(self.embed, tokens)                                   # [n, hidden]
        x = rms_norm(h, self.layers[0]["in_norm"])
        table = rope_table(off, n, self.base, self.device)                 # shared by every layer
        for i, w in enumerate(self.layers):
            # QKV projection + qk-norm + RoPE + KV append in one GEMM (engine.py:111-113)
            q = gemm_qkv_rope(x, w["qkv"], w["q_norm"], w["k_norm"], table, off, self.nq_local, self.n_kv,
                              cache.kv[i], Lp)                                # [nq_local, Lp, 128]
            final = i == nl - 1
            if final and not last:
                break        # a middle chunk only needs the final layer's cache rows, now written
            if final and not all_logits:
                # Only the final row feeds the logits: attention/MLP for one row (engine.py:118-121).
                qrow = q[:, n - 1, :].contiguous()
                o = self._attend_one(qrow, cache.kv[i], off + n).reshape(1, -1)
                h = h[n - 1:]
            else:
                kvl = cache.kv[i]
                o = attention(q, kvl[0], kvl[1], n, off + n, self.scale)       # [n, nq_local*128]
                o = o if self.tp else self._gather_rows(o)                     # [n, H*128]
            nxt = None if final else self.layers[i + 1]["in_norm"]
            if self.tp:  # row-parallel O and down: partial sums exchanged over NVLink
                h, x = self._tp_add_rms(o, w["o"], h.contiguous(), w["post_norm"])
                h, x = self._tp_add_rms(_linear(x, w["gu"], "swiglu"), w["down"], h, nxt)
                continue
            h, x = add_rms(h, _linear(o, w["o"]), w["post_norm"])
            r = _linear(_linear(x, w["gu"], "swiglu"), w["down"])
            if final:
                h = h + r
            else:
                h, x = add_rms(h, r, nxt)
        cache.offset += n
        if not last:
            return None
        if all_logits:
            hn = rms_norm(h, self.final_norm)
            lg = _linear(hn, self.lm_head, "f32")
            return (self._gather_vocab(lg) if self.tp else lg)[None]
        lg = gemv(self.lm_head, h.reshape(-1), nw=self.final_norm, out_float=True)
        return (self._gather_vocab(lg) if self.tp else lg)[None, None]

    # ---------------- decode (M = 1), eager ----------------
    def decode(self, token, cache: Cache, *, return_logits: bool = False):
        """token: int32 CUDA [1].  Returns the next greedy token, int32 CUDA [1]
        (or the FP32 logits [vocab]), as engine.py:145-163."""
        pos = cache.offset
        n = pos + 1
        if n > cache.capacity:
            raise ValueError("KV capacity exceeded")
        if self.tp:
            return self._decode_tp(token, cache, return_logits)
        h = embedding(self.embed, token.reshape(-1)).reshape(-1)
        for i, w in enumerate(self.layers):
            qkv = gemv(w["qkv"], h, nw=w["in_norm"])
            q = qk_norm_rope_append(qkv, w["q_norm"], w["k_norm"], pos, self.nq_local, self.n_kv,
                                    self.base, cache.kv[i])
            o = self._attend_one(q, cache.kv[i], n)
            h = gemv(w["o"], o.reshape(-1), res=h)
            a = gemv(w["gu"], h, nw=w["post_norm"], swiglu=True, wide=True)
            h = gemv(w["down"], a, res=h, wide=True)
        cache.offset += 1
        logits = gemv(self.embed, h, nw=self.final_norm, out_float=True)
        if return_logits:
            return logits
        return argmax(logits)

    def _tp_layer(self, i: int, w: dict, hA, hB, qkv, a, pos_dev, attend) -> None:
        """One tensor-parallel decode layer.  On entry hB holds the previous
        layer's post-attention residual and the exchange holds its down
        partials (layer 0: hA holds the embedding and nothing is pending); on
        exit hA holds this layer's input residual, hB its post-attention
        residual, and the exchange holds this layer's down partials."""
        from .tp import EPI_PEER_PARTIAL
        x = self.tpx
        if i == 0:
            x.gemv(w["qkv"], hA, nw=w["in_norm"], out=qkv)
        else:
            x.gemv(w["qkv"], hB, nw=w["in_norm"], out=qkv, in_sum=True, x_out=hA)
        q = attend(qkv, w, i, pos_dev)
        x.gemv(w["o"], q.reshape(-1), epi=EPI_PEER_PARTIAL)
        x.gemv(w["gu"], hA, nw=w["post_norm"], epi=2, out=a, in_sum=True, x_out=hB)
        x.gemv(w["down"], a, epi=EPI_PEER_PARTIAL)

    def _decode_tp(self, token, cache: Cache, return_logits: bool):
        """Engine.decode under tensor parallelism (eager)."""
        pos = cache.offset
        n = pos + 1
        cfg, dev = self.cfg, self.device
        bf = dict(dtype=torch.bfloat16, device=dev)
        hA, hB = torch.empty(cfg.hidden_size, **bf), torch.empty(cfg.hidden_size, **bf)
        qkv = torch.empty((self.nq_local + 2 * self.n_kv) * HEAD_DIM, **bf)
        a = torch.empty(cfg.intermediate_size // self.world, **bf)
        embedding(self.embed, token.reshape(-1), out=hA.view(1, -1))

        def attend(qkv_, w, i, _):
            q = qk_norm_rope_append(qkv_, w["q_norm"], w["k_norm"], pos, self.nq_local, self.n_kv, self.base,
                                    cache.kv[i])
            return decode_attention(q, cache.kv[i], n, self.scale)

        for i, w in enumerate(self.layers):
            self._tp_layer(i, w, hA, hB, qkv, a, None, attend)
        cache.offset += 1
        logits = torch.empty(self.lm_head.shape[0], dtype=torch.float32, device=dev)
        self.tpx.gemv(self.lm_head, hB, nw=self.final_norm, out=logits, out_float=True, in_sum=True, x_out=hA)
        if return_logits:
            return self._gather_vocab(logits)
        ws = torch.empty(int(_lib.load().rib_argmax_workspace_bytes()), dtype=torch.uint8, device=dev)
        out = torch.empty(1, dtype=torch.int32, device=dev)
        return self.tpx.argmax(logits, self.v0, out, ws)

    def decode_graph(self, cache: Cache) -> "DecodeGraph":
        return DecodeGraph(self, cache)

    def persistent_decode(self, cache: Cache) -> "PersistentDecode":
        return PersistentDecode(self, cache)

    def session(self, capacity: int, mode: str = "graph"):
        """A cache of at least `capacity` positions with its decode-step runner
        (mode "graph": the captured CUDA graph, "persistent": the one-launch
        step kernel), reused across requests (capacity rounded up to 1024):
        rows past the offset are never read, so a request only resets the
        offset.  One request at a time per session."""
        if mode not in ("persistent", "graph"):
            raise ValueError(f"unknown decode mode {mode!r}")
        bucket = (capacity + 1023) // 1024 * 1024
        key = (bucket, mode)
        sess = self._sessions.get(key)
        if sess is None:
            cache = self.new_cache(bucket)
            runner = PersistentDecode(self, cache) if mode == "persistent" else DecodeGraph(self, cache)
            sess = (cache, runner)
            self._sessions[key] = sess
        sess[0].offset = 0
        return sess

    # ---------------- generation ----------------
    def generate(self, prompt: list[int], *, max_tokens: int = 65, chunk: int = 4096, eos_ids=(),
                 use_graph: bool = True, mode: str = "graph") -> Iterator[int]:
        """Greedy generation (engine.py:165-192): chunked prefill, the first
        token, then decode steps with one step of lookahead (step t+1 is
        enqueued before token t is read on the host).  With use_graph the
        steps run on the session's runner: `mode` "graph" (a captured CUDA
        graph of the multi-kernel step, the faster on B200) or "persistent"
        (one cooperative launch per token); without it, eager multi-kernel
        steps."""
        if not prompt or max_tokens < 0 or chunk < 1:
            raise ValueError("Nonempty prompt, nonnegative max_tokens, positive chunk required")
        if min(prompt) < 0 or max(prompt) >= self.cfg.vocab_size:
            raise ValueError("Token outside vocabulary")
        if max_tokens == 0:
            return
        eos_ids = set(eos_ids)
        need = len(prompt) + max_tokens + 1
        if use_graph:
            cache, graph = self.session(need, mode)
        else:
            cache, graph = self.new_cache(need), None
        tokens = torch.tensor(prompt, dtype=torch.int32).pin_memory().to(self.device, non_blocking=True)
        logits = None
        for start in range(0, len(prompt), chunk):
            end = min(len(prompt), start + chunk)
            logits = self.prefill(tokens[start:end], cache, last=end == len(prompt))
        y = argmax(logits.reshape(-1))
        if graph is not None:
            yield from graph.run(y, max_tokens, eos_ids)
            return
        host = torch.empty(1, dtype=torch.int32).pin_memory()
        for _ in range(max_tokens):
            host.copy_(y, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            nxt = self.decode(y, cache) if cache.offset + 1 <= cache.capacity else None
            ev.synchronize()
            token = int(host[0])
            yield token
            if token in eos_ids or nxt is None:
                break
            y = nxt


class DecodeGraph:
    """One decode step captured in a CUDA graph.

    Static device state: the input token (overwritten in place by the step's
    argmax), the position and the key count (advanced by the step itself), the
    per-layer cache pointers and every intermediate buffer.  The decode
    attention geometry is fixed at capture time for max_n = cache.capacity and
    reads the live key count from the device, so one graph serves every
    position of this cache.  Replays on the stream that was current at
    construction."""

    _capture_lock = threading.Lock()

    def __init__(self, engine: Engine, cache: Cache):
        self.e, self.cache = engine, cache
        cfg, dev = engine.cfg, engine.device
        self.device = dev
        self.tok = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.nkeys = torch.ones(1, dtype=torch.int32, device=dev)
        self.ptrs = torch.tensor([cache.kv[i].data_ptr() for i in range(cfg.num_layers)],
                                 dtype=torch.int64, device=dev)
        d, qkvw = cfg.hidden_size, (engine.nq_local + 2 * engine.n_kv) * HEAD_DIM
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.h = [torch.empty(d, **bf), torch.empty(d, **bf), torch.empty(d, **bf)]
        self.x = torch.empty((1, d), **bf)
        self.qkv = torch.empty(qkvw, **bf)
        self.q = torch.empty((self.e.nq_local, 1, HEAD_DIM), **bf)
        heads = self.e.nq_local if engine.tp else self.e.n_heads        # attention outputs this rank holds
        self.o = torch.empty((1, heads, HEAD_DIM), **bf)
        self.a = torch.empty(cfg.intermediate_size // (engine.world if engine.tp else 1), **bf)
        self.logits = torch.empty(engine.lm_head.shape[0], dtype=torch.float32, device=dev)
        L = _lib.load()
        self.max_n = cache.capacity
        ws_bytes = int(L.rib_decode_workspace_bytes(1, self.max_n, engine.n_kv))
        self.ws = torch.zeros(max(ws_bytes, 1 << 20), dtype=torch.uint8, device=dev)  # counters zero
        self.argmax_ws = torch.empty(int(L.rib_argmax_workspace_bytes()), dtype=torch.uint8, device=dev)
        self.launches_per_step = 0
        self.stream = torch.cuda.current_stream(dev)
        self.graph = torch.cuda.CUDAGraph()
        with DecodeGraph._capture_lock:
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(self.stream)
            with torch.cuda.stream(side):
                # Warm-up run outside the graph (first-call set-up of every launch).
                # It appends at the last cache row, which no position below it
                # reads and a real step at that position overwrites first.
                if cache.offset < cache.capacity - 1:
                    self.pos.fill_(cache.capacity - 1)
                    self.nkeys.fill_(cache.capacity)
                    self._step(count=True)
            self.stream.wait_stream(side)
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(self.graph, stream=side):
                self._step(count=False)
            self.stream.wait_stream(side)
        torch.cuda.synchronize(dev)

    def _step(self, count: bool) -> None:
        if self.e.tp:
            return self._step_tp(count)
        e, cfg, L = self.e, self.e.cfg, _lib.load()
        st = stream_handle(self.device)
        launches = 0
        h = embedding(e.embed, self.tok, out=self.h[0].view(1, -1)).view(-1)
        launches += 1
        for i, w in enumerate(e.layers):
            gemv(w["qkv"], h, nw=w["in_norm"], out=self.qkv)
            if e.world > 1:   # this rank's heads, every rank's outputs into self.o over NVLink
                qk_norm_rope_append_at(self.qkv, w["q_norm"], w["k_norm"], self.pos, e.nq_local, e.n_kv, e.base,
                                       self.cache.kv[i], out=self.q)
                e.gather.decode_into(self.q.view(1, e.nq_local, HEAD_DIM), self.ptrs[i:i + 1], self.nkeys,
                                     self.max_n, self.cache.capacity, e.scale, self.ws, e.epoch_dev, self.o)
                launches += 1
            else:             # norm + RoPE + append inside the attention launch
                self._attend_fused(L, st, w, i)
            h1 = gemv(w["o"], self.o.view(-1), res=h, out=self.h[1])
            # (the wide GEMV form after another GEMV; the O GEMV, right after the
            # attention, keeps the narrow one)
            gemv(w["gu"], h1, nw=w["post_norm"], swiglu=True, out=self.a, wide=True)
            h = gemv(w["down"], self.a, res=h1, out=self.h[2 if h is not self.h[2] else 0], wide=True)
            launches += 5
        gemv(e.embed, h, nw=e.final_norm, out_float=True, out=self.logits)
        argmax(self.logits, out=self.tok, workspace=self.argmax_ws)
        launches += 2
        self.pos.add_(1)
        self.nkeys.add_(1)
        if count:
            self.launches_per_step = launches

    def _attend_fused(self, L, st, w, i: int) -> None:
        """Layer i's norm + RoPE + KV append of the new token and its decode
        attention in one launch (rib_decode_attention_qkv): q from self.qkv,
        the position is nkeys - 1, the output goes to self.o."""
        e = self.e
        rc = L.rib_decode_attention_qkv(self.qkv.data_ptr(), w["q_norm"].data_ptr(), w["k_norm"].data_ptr(),
                                        float(e.base), self.ptrs.data_ptr() + 8 * i, self.nkeys.data_ptr(), 1,
                                        self.max_n, self.cache.capacity, e.nq_local, e.n_kv, float(e.scale),
                                        self.o.data_ptr(), self.ws.data_ptr(), self.ws.numel(), st)
        _lib.check(rc, "decode_attention_qkv")

    def _step_tp(self, count: bool) -> None:
        """The step under tensor parallelism: per layer QKV GEMV (input: the
        residual plus the previous layer's down partials), RoPE + append and
        attention of this rank's heads, O GEMV to partials, gate/up GEMV +
        SwiGLU (input: residual plus the O partials), down GEMV to partials;
        then the LM-head slice and the cross-rank argmax."""
        e, L = self.e, _lib.load()
        st = stream_handle(self.device)
        hA, hB = self.h[0], self.h[1]
        embedding(e.embed, self.tok, out=hA.view(1, -1))
        ptrs = self.ptrs

        def attend(qkv, w, i, _):
            self._attend_fused(L, st, w, i)   # (qkv is self.qkv)
            return self.o

        for i, w in enumerate(e.layers):
            e._tp_layer(i, w, hA, hB, self.qkv, self.a, self.pos, attend)
        e.tpx.gemv(e.lm_head, hB, nw=e.final_norm, out=self.logits, out_float=True, in_sum=True, x_out=hA)
        e.tpx.argmax(self.logits, e.v0, self.tok, self.argmax_ws)
        self.pos.add_(1)
        self.nkeys.add_(1)
        if count:
            self.launches_per_step = 1 + 5 * len(e.layers) + 2

    def set_state(self, token, pos: int) -> None:
        """Next replay decodes `token` (int32 CUDA [1] or int) at position `pos`."""
        if isinstance(token, torch.Tensor):
            self.tok.copy_(token.reshape(-1)[:1])
        else:
            self.tok.fill_(int(token))
        self.pos.fill_(int(pos))
        self.nkeys.fill_(int(pos) + 1)

    def replay(self) -> None:
        """One decode step: reads tok/pos, appends K/V at pos, writes the next
        token into tok and advances pos.  Advances cache.offset on the host."""
        if self.cache.offset + 1 > self.cache.capacity:
            raise ValueError("KV capacity exceeded")
        self.graph.replay()
        self.cache.offset += 1

    def run(self, first_token, max_tokens: int, eos_ids=()) -> Iterator[int]:
        """Yields max_tokens tokens starting with first_token (int32 CUDA [1]),
        replaying the graph for each next one with one step of lookahead."""
        self.set_state(first_token, self.cache.offset)
        host = torch.empty(max_tokens, dtype=torch.int32).pin_memory()
        events = []
        for t in range(max_tokens):
            host[t:t + 1].copy_(self.tok, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            events.append(ev)
            more = t + 1 < max_tokens and self.cache.offset + 1 <= self.cache.capacity
            if more:
                self.replay()
            ev.synchronize()
            token = int(host[t])
            yield token
            if token in eos_ids or not more:
                break


class _Qwen3Layer(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in
                ("qkv", "o", "gu", "down", "in_norm", "post_norm", "q_norm", "k_norm")]


class _Qwen3Model(ctypes.Structure):
    """rib_qwen3_model (include/rib_attention.h)."""
    _fields_ = [("num_layers", ctypes.c_int), ("hidden", ctypes.c_int), ("num_heads", ctypes.c_int),
                ("num_kv_heads", ctypes.c_int), ("intermediate", ctypes.c_int), ("vocab", ctypes.c_int),
                ("rope_theta", ctypes.c_double), ("embed", ctypes.c_void_p), ("final_norm", ctypes.c_void_p),
                ("layers", _Qwen3Layer * 64)]


class PersistentDecode:
    """The decode step as one cooperative launch (rib_qwen3_decode_step): the
    same state and interface as DecodeGraph (token, position and key count on
    the device, advanced by the step itself), but the whole token runs in one
    persistent kernel with grid barriers between its phases."""

    def __init__(self, engine: Engine, cache: Cache):
        cfg, dev = engine.cfg, engine.device
        if cfg.num_layers > 64:
            raise ValueError("the persistent decode step takes at most 64 layers")
        if engine.world > 1:
            raise ValueError("the persistent decode step runs on one GPU (use mode='graph' when sharded)")
        self.e, self.cache, self.device = engine, cache, dev
        m = _Qwen3Model()
        m.num_layers, m.hidden, m.num_heads = cfg.num_layers, cfg.hidden_size, cfg.num_heads
        m.num_kv_heads, m.intermediate, m.vocab = cfg.num_kv_heads, cfg.intermediate_size, cfg.vocab_size
        m.rope_theta = float(cfg.rope_theta)
        m.embed, m.final_norm = engine.embed.data_ptr(), engine.final_norm.data_ptr()
        for i, w in enumerate(engine.layers):
            for k in ("qkv", "o", "gu", "down", "in_norm", "post_norm", "q_norm", "k_norm"):
                setattr(m.layers[i], k, w[k].data_ptr())
        self._model = m
        L = _lib.load()
        nbytes = int(L.rib_qwen3_step_workspace_bytes(ctypes.byref(m), cache.capacity))
        if nbytes == 0:
            raise ValueError("model shape not supported by the persistent decode step")
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)   # zero-filled: ready
        self.ptrs = torch.tensor([cache.kv[i].data_ptr() for i in range(cfg.num_layers)], dtype=torch.int64,
                                 device=dev)
        self.tok = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.nkeys = torch.ones(1, dtype=torch.int32, device=dev)
        self.logits = torch.empty(cfg.vocab_size, dtype=torch.float32, device=dev)
        self.launches_per_step = 1

    def set_state(self, token, pos: int) -> None:
        if isinstance(token, torch.Tensor):
            self.tok.copy_(token.reshape(-1)[:1])
        else:
            self.tok.fill_(int(token))
        self.pos.fill_(int(pos))
        self.nkeys.fill_(int(pos) + 1)

    def replay(self, logits: bool = False) -> None:
        """One decode step (see DecodeGraph.replay); with `logits` the FP32
        logits land in self.logits."""
        if self.cache.offset + 1 > self.cache.capacity:
            raise ValueError("KV capacity exceeded")
        st = _lib.load().rib_qwen3_decode_step(
            ctypes.byref(self._model), self.ptrs.data_ptr(), self.cache.capacity, self.tok.data_ptr(),
            self.pos.data_ptr(), self.nkeys.data_ptr(), self.logits.data_ptr() if logits else None,
            self.ws.data_ptr(), self.ws.numel(), stream_handle(self.device))
        _lib.check(st, "qwen3_decode_step")
        self.cache.offset += 1

    run = DecodeGraph.run
