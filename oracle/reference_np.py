"""Independent FP64 numpy restatement of the attention hot path -- TEST
INFRASTRUCTURE ONLY.

A second, vectorised implementation written separately from oracle.c, used to
pin the C oracle (and through it the CUDA path) on small cases.  It follows
the same reference semantics:
  - qk-norm + RoPE: agent-test/v2/kernels.py:116-146, 169-204; rounding points
    n = bf16(w * bf16(x * inv)) (kernels.py:131-133); non-traditional RoPE,
    pairs (d, d+64), theta = float(pos) * exp2(-(d/64) * float(log2(base)))
    formed in FP32 as the Metal code forms it (kernels.py:134-138, 152), as
    pinned by agent-test/v2/test_engine.py:52-59; cos/sin of that angle in
    FP64.  angle_f64=True forms the angle in FP64 instead.
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


def rope_inv_freq_f32(base) -> np.ndarray:
    """exp2(-(d/64) * log2(base)) as kernels.py:137-138 forms it: log2(base)
    rounded to FP32 (the f-string literal of kernels.py:152), the FP32 product
    with -(d/64), exp2 rounded once to FP32."""
    lb = np.float32(np.log2(np.float64(base)))
    x = (-(np.arange(64, dtype=np.float32) / np.float32(64.0))) * lb  # FP32 product
    return np.exp2(x.astype(np.float64)).astype(np.float32)


def rope_angles(pos, base, angle_f64=False) -> np.ndarray:
    """theta [len(pos), 64] in FP64: the FP32 product float(pos) * inv_freq
    (kernels.py:134-138), or the FP64 angle when angle_f64."""
    pos = np.asarray(pos)
    if angle_f64:
        inv = np.float64(base) ** (-np.arange(64, dtype=np.float64) / 64.0)
        return pos.astype(np.float64)[:, None] * inv[None]
    th = pos.astype(np.float32)[:, None] * rope_inv_freq_f32(base)[None]  # FP32 product
    return th.astype(np.float64)


def qk_norm_rope(qkv, qw, kw, offset, nq, nkv, base, Lp=None, angle_f64=False):
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
    th = rope_angles(offset + np.arange(L), base, angle_f64)  # [L, 64]
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


def prefill_attention_mlx_bf16(Q, K, V, qL, kL, scale, rows=None):
    """The error yardstick of the reference's prefill test: MLX's fused SDPA on
    BF16 inputs (agent-test/v2/test_engine.py:96, mask="causal").

    MLX (0.32.3, pinned in agent-test/v2/README.md:6; third-party, absent
    here) runs query lengths above 8 through its tiled "steel" attention
    kernel.  Its published algorithm, restated: the Q tile is scaled in place
    in the input type by T(scale * log2(e)) -- for BF16 both the factor and
    each product are rounded to BF16 -- then S = Q K^T, the exp2-domain online
    softmax and O = P V all run in FP32 (the reference kernel's own comment,
    attention.py:6, "P.V uses FP32 P ... like MLX's kernel"), and O / l is
    rounded once to BF16.  The causal mask is bottom-right aligned.  Returns
    u16 [qL, H*128], or the rows [r0, r1) only when rows=(r0, r1).  An FP32 softmax over the whole row stands in for the
    tiled online one (they differ by FP32 rounding only)."""
    H = Q.shape[0]
    nkv = K.shape[0]
    g = H // nkv
    r0, r1 = (0, qL) if rows is None else rows
    fac = round_bf16(np.float32(scale * 1.4426950408889634))
    Qs = round_bf16(bf16_to_f32(Q[:, r0:r1]) * fac).astype(np.float64)
    Kf = bf16_to_f32(K[:, :kL]).astype(np.float64)
    Vf = bf16_to_f32(V[:, :kL]).astype(np.float64)
    off = kL - qL
    mask = np.arange(kL)[None, :] > (off + np.arange(r0, r1))[:, None]
    out = np.zeros((r1 - r0, H * 128), np.float32)
    for h in range(H):
        s = (Qs[h] @ Kf[h // g].T).astype(np.float32).astype(np.float64)
        s[mask] = -np.inf
        p = np.exp2(s - s.max(axis=1, keepdims=True))
        out[:, h * 128:(h + 1) * 128] = (p @ Vf[h // g]) / p.sum(axis=1, keepdims=True)
    return f32_to_bf16(out)


def prefill_attention_bf16p(Q, K, V, qL, kL, scale, rows=None):
    """A plain BF16-P SDPA: FP32 scores and softmax against the exact row max,
    P rounded to BF16 before P V (FP32 accumulation), the row sum taken from
    the unrounded P, O / l rounded once to BF16.  The arithmetic of a
    tensor-core kernel that feeds P to a BF16 MMA, without its tiling.
    Returns u16 [qL, H*128], or the rows [r0, r1) only when rows=(r0, r1)."""
    H = Q.shape[0]
    nkv = K.shape[0]
    g = H // nkv
    r0, r1 = (0, qL) if rows is None else rows
    Qf = bf16_to_f32(Q[:, r0:r1]).astype(np.float64)
    Kf = bf16_to_f32(K[:, :kL]).astype(np.float64)
    Vf = bf16_to_f32(V[:, :kL]).astype(np.float64)
    off = kL - qL
    mask = np.arange(kL)[None, :] > (off + np.arange(r0, r1))[:, None]
    sl2 = np.float32(scale * 1.4426950408889634)
    out = np.zeros((r1 - r0, H * 128), np.float32)
    for h in range(H):
        s = ((Qf[h] @ Kf[h // g].T).astype(np.float32) * sl2).astype(np.float64)
        s[mask] = -np.inf
        p = np.exp2(s - s.max(axis=1, keepdims=True))
        out[:, h * 128:(h + 1) * 128] = (round_bf16(p.astype(np.float32)).astype(np.float64) @ Vf[h // g]) \
            / p.sum(axis=1, keepdims=True)
    return f32_to_bf16(out)
