"""numpy restatement of the Qwen3 forward around the attention path -- TEST
INFRASTRUCTURE ONLY.

Checker for the model kernels (csrc/model_kernels.cuh) and the engine
(model.py).  Only tests/ and __graft_entry__.smoke() use it.  BF16 data is
carried as uint16 bit patterns; dot products are FP64, so the CUDA path's
FP32 sums differ only by summation order.  The rounding points follow the
reference's Metal kernels and engine (aeilot/roofline-inference,
agent-test/v2):
  RMSNorm      inv = 1/sqrt(sum(x^2)/K + 1e-6), n = bf16(w * bf16(x * inv))
               (kernels.py:48-55; mx.fast.rms_norm at engine.py:109, 140)
  GEMV         bf16(W x), or FP32 for the logits       (kernels.py:58-81, 96)
  residual     bf16(res + bf16(W x))                   (kernels.py:84-85)
  SwiGLU       g = bf16(.), u = bf16(.), s = bf16(sigmoid(g)), a = bf16(g s),
               y = bf16(a u)                           (kernels.py:86-93; engine.py:28-30)
  add_rms      r = bf16(a + b), n = bf16(w * bf16(r * inv)) (kernels.py:227-268)
  forward      engine.py:102-163: the prefill's last layer runs attention and
               MLP for the final row only; greedy argmax of the final row.
Attention and qk-norm/RoPE come from reference_np (FP64 after the BF16
inputs); the attention output is rounded to BF16 where the kernels write it.
"""
from __future__ import annotations

import numpy as np

from .reference_np import (bf16_to_f32, decode_attention, f32_to_bf16, prefill_attention, qk_norm_rope,
                           round_bf16)

EPS = 1e-6


def _f(u16) -> np.ndarray:
    return bf16_to_f32(np.asarray(u16, dtype=np.uint16)).astype(np.float64)


def rms_norm(x, w) -> np.ndarray:
    """x u16 [..., K], w u16 [K] -> u16."""
    xf = bf16_to_f32(np.asarray(x, dtype=np.uint16))
    ss = np.sum(xf.astype(np.float64) ** 2, axis=-1, keepdims=True)
    inv = (1.0 / np.sqrt(ss / xf.shape[-1] + EPS)).astype(np.float32)
    return f32_to_bf16(bf16_to_f32(np.asarray(w, np.uint16)) * round_bf16(xf * inv))


def add_rms(a, b, w):
    r = f32_to_bf16(bf16_to_f32(np.asarray(a, np.uint16)) + bf16_to_f32(np.asarray(b, np.uint16)))
    return r, rms_norm(r, w)


def _silu_bf16(g: np.ndarray) -> np.ndarray:
    s = round_bf16((1.0 / (1.0 + np.exp(-g.astype(np.float64)))).astype(np.float32))
    return round_bf16(g * s)


def swiglu(gu) -> np.ndarray:
    """gu u16 [..., 2F] -> u16 [..., F]."""
    g = bf16_to_f32(np.asarray(gu, np.uint16))
    F = g.shape[-1] // 2
    return f32_to_bf16(_silu_bf16(g[..., :F]) * g[..., F:])


def gemv(W, x, nw=None, res=None, swiglu_epi=False, out_float=False):
    """W u16 [N, K], x u16 [K] -> u16 [N] ([N/2] for SwiGLU) or f32 [N]."""
    xin = rms_norm(x, nw) if nw is not None else np.asarray(x, np.uint16)
    acc = (_f(W) @ _f(xin)).astype(np.float32)
    if out_float:
        return acc
    if swiglu_epi:
        F = acc.shape[0] // 2
        g, u = round_bf16(acc[:F]), round_bf16(acc[F:])
        return f32_to_bf16(_silu_bf16(g) * u)
    if res is not None:
        return f32_to_bf16(bf16_to_f32(np.asarray(res, np.uint16)) + round_bf16(acc))
    return f32_to_bf16(acc)


def row_parallel_add_rms(parts, h, w=None):
    """A row-parallel projection over ranks followed by add_rms, as the
    tensor-parallel prefill computes it: parts = [(x_r u16 [m, K_r],
    W_r u16 [N, K_r])] in rank order; each rank's FP32 partial x_r W_r^T, the
    partials added in rank order in FP32, rounded once to BF16 (r), then
    residual = bf16(h + r) and, with the norm weight w, its RMSNorm -- the
    add_rms after each projection of Engine.prefill (engine.py:129-134,
    kernels.py:227-268).  Returns (residual, normalised or None) as u16."""
    acc = None
    for x, W in parts:
        p = (_f(x) @ _f(W).T).astype(np.float32)
        acc = p if acc is None else (acc + p).astype(np.float32)
    r = f32_to_bf16(acc)
    if w is None:
        return f32_to_bf16(bf16_to_f32(np.asarray(h, np.uint16)) + bf16_to_f32(r)), None
    return add_rms(h, r, w)


def matmul(x, W) -> np.ndarray:
    """x u16 [m, K] @ W u16 [N, K]^T -> u16 [m, N] (a BF16 GEMM, FP32 accumulate)."""
    return f32_to_bf16((_f(x) @ _f(W).T).astype(np.float32))


def argmax(logits) -> int:
    return int(np.argmax(np.asarray(logits)))


class Qwen3Oracle:
    """The forward on numpy copies of an engine's weights (u16 arrays).

    weights: dict with 'embed', 'final_norm' and 'layers' (list of dicts with
    qkv, o, gu, down, in_norm, post_norm, q_norm, k_norm); cfg: an object with
    num_heads, num_kv_heads, rope_theta."""

    def __init__(self, weights: dict, cfg, capacity: int):
        self.w = weights
        self.nq, self.nkv = cfg.num_heads, cfg.num_kv_heads
        self.base = cfg.rope_theta
        self.scale = 128 ** -0.5
        nl = len(weights["layers"])
        self.K = [np.zeros((self.nkv, capacity, 128), np.uint16) for _ in range(nl)]
        self.V = [np.zeros((self.nkv, capacity, 128), np.uint16) for _ in range(nl)]
        self.offset = 0

    def _append(self, i, qkv, off):
        Q, KV = qk_norm_rope(qkv, self.w["layers"][i]["q_norm"], self.w["layers"][i]["k_norm"], off,
                             self.nq, self.nkv, self.base)
        n = KV.shape[2]
        self.K[i][:, off:off + n] = KV[0]
        self.V[i][:, off:off + n] = KV[1]
        return Q  # [nq, n, 128]

    def prefill(self, tokens) -> np.ndarray:
        """Returns the FP32 logits of the final row; advances the offset."""
        tokens = np.asarray(tokens).reshape(-1)
        n, off = tokens.size, self.offset
        L = self.w["layers"]
        h = np.asarray(self.w["embed"])[tokens]
        x = rms_norm(h, L[0]["in_norm"])
        for i, w in enumerate(L):
            Q = self._append(i, matmul(x, w["qkv"]), off)
            if i == len(L) - 1:
                o = decode_attention(Q[:, n - 1], self.K[i][:, :off + n], self.V[i][:, :off + n], self.scale)
                o = f32_to_bf16(o.reshape(1, -1).astype(np.float32))
                h = h[n - 1:]
            else:
                o = f32_to_bf16(prefill_attention(Q, self.K[i], self.V[i], n, off + n, self.scale)
                                .astype(np.float32))
            h, x = add_rms(h, matmul(o, w["o"]), w["post_norm"])
            r = matmul(swiglu(matmul(x, w["gu"])), w["down"])
            if i == len(L) - 1:
                h = f32_to_bf16(bf16_to_f32(h) + bf16_to_f32(r))
            else:
                h, x = add_rms(h, r, L[i + 1]["in_norm"])
        self.offset += n
        return gemv(self.w["embed"], h.reshape(-1), nw=self.w["final_norm"], out_float=True)

    def decode(self, token: int) -> np.ndarray:
        """One token at the current offset; returns its FP32 logits."""
        pos = self.offset
        h = np.asarray(self.w["embed"])[int(token)]
        for i, w in enumerate(self.w["layers"]):
            qkv = gemv(w["qkv"], h, nw=w["in_norm"])
            Q = self._append(i, qkv.reshape(1, -1), pos)
            o = decode_attention(Q[:, 0], self.K[i][:, :pos + 1], self.V[i][:, :pos + 1], self.scale)
            h = gemv(w["o"], f32_to_bf16(o.reshape(-1).astype(np.float32)), res=h)
            a = gemv(w["gu"], h, nw=w["post_norm"], swiglu_epi=True)
            h = gemv(w["down"], a, res=h)
        self.offset += 1
        return gemv(self.w["embed"], h, nw=self.w["final_norm"], out_float=True)


def weights_to_numpy(weights) -> dict:
    """Qwen3Weights (torch BF16 tensors) -> the u16 dict Qwen3Oracle takes."""
    u = lambda t: t.detach().cpu().contiguous().view(__import__("torch").int16).numpy().view(np.uint16)
    return {"embed": u(weights.embed), "final_norm": u(weights.final_norm),
            "layers": [{k: u(v) for k, v in l.items()} for l in weights.layers]}
