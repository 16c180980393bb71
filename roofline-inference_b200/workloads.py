"""Seeded synthetic inputs with the shapes of the Qwen3-0.6B attention
workloads (16 query heads, 8 KV heads, head_dim 128, RoPE theta 1e6,
RMSNorm eps 1e-6), standing in for the reference's v3 scenarios
ctx512 / ctx4096 / ctx32768 / ttft* (agent-test/v3/run.py:33-35).

  decode_step    one layer: pre-norm qkv row of the new token, norm weights,
                 and a KV cache whose first `ctx` rows are filled (config:
                 single-layer decode, context 512 .. 32768)
  prefill_qkv    L rows of pre-norm qkv (config: causal prefill, L up to 32k)
  ragged_lengths context lengths of a batch of independent sequences

All values are BF16 drawn N(0, 1) from torch generators seeded per object;
norm weights are 1 + 0.1 N(0, 1) (agent-test/v2/test_engine.py:65-66).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

NQ, NKV, HEAD_DIM = 16, 8, 128
ROPE_THETA = 1e6
N_LAYERS = 28
SCALE = HEAD_DIM ** -0.5
QKV_WIDTH = (NQ + 2 * NKV) * HEAD_DIM  # 4096


def _gen(seed: int, device) -> torch.Generator:
    dev = torch.device(device)
    g = torch.Generator(device=dev if dev.type == "cuda" else "cpu")
    g.manual_seed(int(seed))
    return g


def randn_bf16(shape, seed: int, device="cpu", scale: float = 1.0) -> torch.Tensor:
    g = _gen(seed, device)
    x = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    if scale != 1.0:
        x = x * scale
    return x.to(torch.bfloat16)


def norm_weights(seed: int, device="cpu") -> torch.Tensor:
    g = _gen(seed, device)
    w = 1.0 + 0.1 * torch.randn((HEAD_DIM,), generator=g, device=device, dtype=torch.float32)
    return w.to(torch.bfloat16)


def round_cap(n: int) -> int:
    """Cache capacity rule of the reference (agent-test/v2/engine.py:37)."""
    return (n + 255) // 256 * 256


@dataclass
class DecodeStep:
    qkv: torch.Tensor    # [4096] pre-norm projection of the new token
    qw: torch.Tensor     # [128]
    kw: torch.Tensor     # [128]
    cache: torch.Tensor  # [2, nkv, cap, 128]; rows [0, ctx) filled
    pos: int             # position of the new token (== ctx)

    @property
    def n(self) -> int:  # keys attended after the append
        return self.pos + 1


def decode_step(ctx: int, seed: int, device="cpu", nkv: int = NKV, cap: int | None = None) -> DecodeStep:
    """One decode layer at context `ctx` (ctx cached tokens + the new one)."""
    cap = round_cap(ctx + 1) if cap is None else cap
    nq = 2 * nkv
    qkv = randn_bf16(((nq + 2 * nkv) * HEAD_DIM,), seed * 7919 + 1, device)
    qw = norm_weights(seed * 7919 + 2, device)
    kw = norm_weights(seed * 7919 + 3, device)
    cache = torch.zeros((2, nkv, cap, HEAD_DIM), dtype=torch.bfloat16, device=device)
    if ctx > 0:
        cache[:, :, :ctx] = randn_bf16((2, nkv, ctx, HEAD_DIM), seed * 7919 + 4, device)
    return DecodeStep(qkv, qw, kw, cache, ctx)


def prefill_qkv(L: int, seed: int, device="cpu", nkv: int = NKV):
    """Pre-norm qkv rows [L, (nq+2nkv)*128] and norm weights for a prefill."""
    nq = 2 * nkv
    qkv = randn_bf16((L, (nq + 2 * nkv) * HEAD_DIM), seed * 104729 + 1, device)
    return qkv, norm_weights(seed * 104729 + 2, device), norm_weights(seed * 104729 + 3, device)


def ragged_lengths(batch: int = 64, lo: int = 512, hi: int = 32768, seed: int = 0) -> list[int]:
    """Context lengths drawn uniformly from [lo, hi] (seeded)."""
    g = torch.Generator().manual_seed(int(seed))
    return [int(x) for x in torch.randint(lo, hi + 1, (batch,), generator=g)]


def decode_kv_bytes(n_keys: int, nkv: int = NKV) -> int:
    """Algorithmic HBM bytes of one decode-attention call: every cached K and V
    element read once (BF16), 4096 bytes per key at 8 KV heads."""
    return 2 * nkv * HEAD_DIM * 2 * n_keys


def prefill_flops(qL: int, kL: int | None = None, nq: int = NQ) -> int:
    """Algorithmic FLOPs of causal attention: QK^T and PV each 2*d per visible
    (query, key) pair; with qL == kL = L this is 4096 * L * (L + 1) at 16
    heads (matches src/roofline/workload.py:176-179)."""
    kL = qL if kL is None else kL
    off = kL - qL  # query i sees off + i + 1 keys
    pairs = qL * off + qL * (qL + 1) // 2
    return 4 * nq * HEAD_DIM * pairs


def scale_log2e() -> float:
    return SCALE * math.log2(math.e)
