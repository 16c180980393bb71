"""Fused QK-RMSNorm + RoPE entry points with the signatures of the reference's
agent-test/v2/kernels.py, backed by the sm_100a kernel in
csrc/qk_norm_rope.cuh through the C ABI (include/rib_attention.h).

  qk_norm_rope(qkv, qw, kw, pos, nq, nkv, base)                 kernels.py:157
  qk_norm_rope_prefill(qkv, qw, kw, offset, nq, nkv, base, Lp)  kernels.py:215
  qk_norm_rope_append(qkv, qw, kw, offset, nq, nkv, base, cache_layer, Lp=None)
      the two above fused with Cache.update (engine.py:42-48): K and V are
      written straight into one layer of the KV cache.

Tensors are torch BF16 CUDA tensors; outputs are allocated by torch on the
input's device and the kernels run on torch's current stream.
"""
from __future__ import annotations

import torch

from . import _lib
from ._tensors import HEAD_DIM, as_int, require_bf16_cuda, require_same_device, stream_handle


def _check_common(qkv, qw, kw, nq: int, nkv: int) -> int:
    require_bf16_cuda("qkv", qkv)
    require_bf16_cuda("qw", qw)
    require_bf16_cuda("kw", kw)
    require_same_device(qkv, qw, kw)
    if qw.numel() != HEAD_DIM or kw.numel() != HEAD_DIM:
        raise ValueError("qw and kw must hold head_dim (128) weights")
    width = (nq + 2 * nkv) * HEAD_DIM
    if qkv.numel() % width:
        raise ValueError(f"qkv size {qkv.numel()} is not a multiple of (nq + 2*nkv)*128 = {width}")
    return qkv.numel() // width


def qk_norm_rope(qkv, qw, kw, pos, nq: int, nkv: int, base: float):
    """Per-head RMSNorm on q/k, RoPE (non-traditional) at position `pos`; v copied.

    qkv: [(nq+2nkv)*128] (or [1, ...]) projection output of one token.
    Returns q [1, nq, 1, 128] and kv [2, nkv, 1, 128] (K and V stacked),
    as agent-test/v2/kernels.py:157-164."""
    L = _check_common(qkv, qw, kw, nq, nkv)
    if L != 1:
        raise ValueError("qk_norm_rope takes one token; use qk_norm_rope_prefill for L > 1")
    pos = as_int(pos, "pos")
    q = torch.empty((1, nq, 1, HEAD_DIM), dtype=torch.bfloat16, device=qkv.device)
    kv = torch.empty((2, nkv, 1, HEAD_DIM), dtype=torch.bfloat16, device=qkv.device)
    st = _lib.load().rib_qk_norm_rope(qkv.data_ptr(), qw.data_ptr(), kw.data_ptr(), pos, nq, nkv,
                                      float(base), q.data_ptr(), kv.data_ptr(),
                                      stream_handle(qkv.device))
    _lib.check(st, "qk_norm_rope")
    return q, kv


def qk_norm_rope_prefill(qkv, qw, kw, offset, nq: int, nkv: int, base: float, Lp: int):
    """qkv [L, (nq+2nkv)*128] -> Q [nq, Lp, 128] (pad rows zero), KV [2, nkv, L, 128].

    Tokens sit at positions offset .. offset+L-1 (agent-test/v2/kernels.py:215-224)."""
    L = _check_common(qkv, qw, kw, nq, nkv)
    offset = as_int(offset, "offset")
    if Lp < L:
        raise ValueError(f"Lp ({Lp}) must be >= L ({L})")
    q = torch.empty((nq, Lp, HEAD_DIM), dtype=torch.bfloat16, device=qkv.device)
    kv = torch.empty((2, nkv, L, HEAD_DIM), dtype=torch.bfloat16, device=qkv.device)
    st = _lib.load().rib_qk_norm_rope_prefill(qkv.data_ptr(), L, qw.data_ptr(), kw.data_ptr(),
                                              offset, nq, nkv, float(base), Lp, q.data_ptr(),
                                              kv.data_ptr(), stream_handle(qkv.device))
    _lib.check(st, "qk_norm_rope_prefill")
    return q, kv


def qk_norm_rope_append(qkv, qw, kw, offset, nq: int, nkv: int, base: float, cache_layer,
                        Lp: int | None = None):
    """Fused qk-norm + RoPE + KV-cache append for L tokens at `offset`.

    cache_layer: one layer of the cache, [2, nkv, cap, 128] (Cache.kv[i]).
    K (normed + roped) and V land in rows offset .. offset+L-1, replacing the
    reference's qk_norm_rope[_prefill] + Cache.update pair (engine.py:111-113,
    152-153).  Returns Q [nq, Lp, 128] (Lp defaults to L; pad rows zero).
    Raises ValueError("... KV capacity exceeded") if offset + L > cap
    (engine.py:45-46)."""
    L = _check_common(qkv, qw, kw, nq, nkv)
    require_bf16_cuda("cache_layer", cache_layer)
    require_same_device(qkv, cache_layer)
    if cache_layer.dim() != 4 or cache_layer.shape[0] != 2 or cache_layer.shape[1] != nkv \
            or cache_layer.shape[3] != HEAD_DIM:
        raise ValueError(f"cache_layer must be [2, {nkv}, cap, 128], got {tuple(cache_layer.shape)}")
    offset = as_int(offset, "offset")
    Lp = L if Lp is None else Lp
    if Lp < L:
        raise ValueError(f"Lp ({Lp}) must be >= L ({L})")
    cap = cache_layer.shape[2]
    q = torch.empty((nq, Lp, HEAD_DIM), dtype=torch.bfloat16, device=qkv.device)
    st = _lib.load().rib_qk_norm_rope_append(qkv.data_ptr(), L, qw.data_ptr(), kw.data_ptr(),
                                             offset, nq, nkv, float(base), Lp, q.data_ptr(),
                                             cache_layer.data_ptr(), cap,
                                             stream_handle(qkv.device))
    _lib.check(st, "qk_norm_rope_append")
    return q
