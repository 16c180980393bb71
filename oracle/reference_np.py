"""Independent FP64 numpy restatement of the attention hot path -- TEST
INFRASTRUCTURE ONLY.

A second, vectorised implementation written separately from oracle.c, used to
pin the C oracle (and through it the CUDA path) on small cases.  It follows
the same reference semantics:
  - qk-norm + RoPE: agent-test/v2/kernels.py:116-146, 169-204; rounding points
    n = bf16(w * bf16(x * inv)) (kernels.py:131-133); non-traditional RoPE,
    pairs (d, d+64), theta = pos * base^(-d/64) (kernels.py:136-143), as pinned
    by agent-test/v2/test_engine.py:52-59.
  - decode: softmax(scale q K^T) V over n keys, GQA h -> h // 2
    (agent-test/v2/engine.py:154-155).
  - prefill: bottom-right aligned causal mask (agent-test/v2/attention.py:24).
Everything after the BF16 inputs is FP64 except the two FP32 BF16 rounding
points of RMSNorm, which the reference performs in FP32.
"""
from __future__ import annotations

import numpy as np


def bf16_to_f32(u16) -> np.ndarray:
    u = np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16
    return u.view(np.float32)


def f32_to_bf16(x) -> np.ndarray:
    """Round-to-nearest-even FP32 -> BF16 bit patterns (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def round_bf16(x) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(x))


def qk_norm_rope(qkv, qw, kw, offset, nq, nkv, base, Lp=None):
    """qkv u16 [L, (nq+2nkv)*128] -> (Q u16 [nq, Lp, 128], KV u16 [2, nkv, L, 128])."""
    items = nq + 2 * nkv
    x = bf16_to_f32(np.asarray(qkv).reshape(-1, items, 128))  # [L, items, 128]
    L = x.shape[0]
    Lp = L if Lp is None else Lp
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    inv = (1.0 / np.sqrt(ss / 128.0 + 1e-6)).astype(np.float32)
    w = np.concatenate([np.broadcast_to(bf16_to_f32(qw), (nq, 128)),
                        np.broadcast_to(bf16_to_f32(kw), (nkv, 128))])  # [nq+nkv, 128]
    nrm = round_bf16(w[None] * round_bf16(x[:, :nq + nkv] * inv[:, :nq + nkv])).astype(np.float64)
    pos = (offset + np.arange(L, dtype=np.float64))[:, None]
    inv_freq = base ** (-np.arange(64, dtype=np.float64) / 64.0)
    th = pos * inv_freq[None]  # [L, 64]
    c, s = np.cos(th)[:, None], np.sin(th)[:, None]
    x1, x2 = nrm[..., :64], nrm[..., 64:]
    rot = np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1).astype(np.float32)
    rot16 = f32_to_bf16(rot)  # [L, nq+nkv, 128]
    Q = np.zeros((nq, Lp, 128), np.uint16)
    Q[:, :L] = rot16[:, :nq].transpose(1, 0, 2)
    KV = np.zeros((2, nkv, L, 128), np.uint16)
    KV[0] = rot16[:, nq:].transpose(1, 0, 2)
    KV[1] = np.asarray(qkv).reshape(-1, items, 128)[:, nq + nkv:].transpose(1, 0, 2)
    return Q, KV


def decode_attention(q, K, V, scale):
    """q u16 [nq, 128]; K, V u16 [nkv, n, 128] -> float64 [nq, 128]."""
    qf = bf16_to_f32(q).astype(np.float64)
    Kf = bf16_to_f32(K).astype(np.float64)
    Vf = bf16_to_f32(V).astype(np.float64)
    nq, nkv = qf.shape[0], Kf.shape[0]
    g = nq // nkv
    out = np.zeros((nq, 128))
    for h in range(nq):
        s = Kf[h // g] @ qf[h] * scale
        p = np.exp(s - s.max())
        out[h] = (p @ Vf[h // g]) / p.sum()
    return out


def prefill_attention(Q, K, V, qL, kL, scale):
    """Q u16 [H, qLp, 128]; K, V u16 [nkv, >=kL, 128] -> float64 [qL, H*128]."""
    H = Q.shape[0]
    nkv = K.shape[0]
    g = H // nkv
    Qf = bf16_to_f32(Q[:, :qL]).astype(np.float64)
    Kf = bf16_to_f32(K[:, :kL]).astype(np.float64)
    Vf = bf16_to_f32(V[:, :kL]).astype(np.float64)
    off = kL - qL
    mask = np.arange(kL)[None, :] > (off + np.arange(qL))[:, None]
    out = np.zeros((qL, H * 128))
    for h in range(H):
        s = Qf[h] @ Kf[h // g].T * scale
        s[mask] = -np.inf
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        out[:, h * 128:(h + 1) * 128] = (p @ Vf[h // g]) / p.sum(axis=1, keepdims=True)
    return out
