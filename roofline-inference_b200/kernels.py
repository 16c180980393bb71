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
from ._tensors import HEAD_DIM, as_int, device_position, require_bf16_cuda, require_same_device, stream_handle


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
    as agent-test/v2/kernels.py:157-164.  pos: an int, or a 1-element int32
    tensor as the engine passes it (engine.py:148); a CUDA tensor is read by
    the kernel on the device, so the call does not synchronise the host."""
    L = _check_common(qkv, qw, kw, nq, nkv)
    if L != 1:
        raise ValueError("qk_norm_rope takes one token; use qk_norm_rope_prefill for L > 1")
    q = torch.empty((1, nq, 1, HEAD_DIM), dtype=torch.bfloat16, device=qkv.device)
    kv = torch.empty((2, nkv, 1, HEAD_DIM), dtype=torch.bfloat16, device=qkv.device)
    pos_dev = device_position(pos, "pos", qkv.device)
    if pos_dev is not None:
        st = _lib.load().rib_qk_norm_rope_prefill_dev(qkv.data_ptr(), 1, qw.data_ptr(), kw.data_ptr(),
                                                      pos_dev.data_ptr(), nq, nkv, float(base), 1, q.data_ptr(),
                                                      kv.data_ptr(), stream_handle(qkv.device))
        _lib.check(st, "qk_norm_rope")
        return q, kv
    pos = as_int(pos, "pos")
    st = _lib.load().rib_qk_norm_rope(qkv.data_ptr(), qw.data_ptr(), kw.data_ptr(), pos, nq, nkv,
                                      float(base), q.data_ptr(), kv.data_ptr(),
                                      stream_handle(qkv.device))
    _lib.check(st, "qk_norm_rope")
    return q, kv


def qk_norm_rope_prefill(qkv, qw, kw, offset, nq: int, nkv: int, base: float, Lp: int):
    """qkv [L, (nq+2nkv)*128] -> Q [nq, Lp, 128] (pad rows zero), KV [2, nkv, L, 128].

    Tokens sit at positions offset .. offset+L-1 (agent-test/v2/kernels.py:215-224);
    a 1-element CUDA int32 offset is read on the device."""
    L = _check_common(qkv, qw, kw, nq, nkv)
    if Lp < L:
        raise ValueError(f"Lp ({Lp}) must be >= L ({L})")
    q = torch.empty((nq, Lp, HEAD_DIM), dtype=torch.bfloat16, device=qkv.device)
    kv = torch.empty((2, nkv, L, HEAD_DIM), dtype=torch.bfloat16, device=qkv.device)
    off_dev = device_position(offset, "offset", qkv.device)
    if off_dev is not None:
        st = _lib.load().rib_qk_norm_rope_prefill_dev(qkv.data_ptr(), L, qw.data_ptr(), kw.data_ptr(),
                                                      off_dev.data_ptr(), nq, nkv, float(base), Lp, q.data_ptr(),
                                                      kv.data_ptr(), stream_handle(qkv.device))
        _lib.check(st, "qk_norm_rope_prefill")
        return q, kv
    offset = as_int(offset, "offset")
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
    (engine.py:45-46).  A 1-element CUDA int32 offset goes to
    qk_norm_rope_append_at (read on the device, capacity checked there)."""
    L = _check_common(qkv, qw, kw, nq, nkv)
    require_bf16_cuda("cache_layer", cache_layer)
    require_same_device(qkv, cache_layer)
    if cache_layer.dim() != 4 or cache_layer.shape[0] != 2 or cache_layer.shape[1] != nkv \
            or cache_layer.shape[3] != HEAD_DIM:
        raise ValueError(f"cache_layer must be [2, {nkv}, cap, 128], got {tuple(cache_layer.shape)}")
    off_dev = device_position(offset, "offset", qkv.device)
    if off_dev is not None:
        return qk_norm_rope_append_at(qkv, qw, kw, off_dev, nq, nkv, base, cache_layer, Lp)
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


def qk_norm_rope_append_at(qkv, qw, kw, offset_dev, nq: int, nkv: int, base: float, cache_layer,
                           Lp: int | None = None, out=None):
    """qk_norm_rope_append with the offset read on the device.

    offset_dev: int32 CUDA tensor of one element (the reference's `pos` array,
    agent-test/v2/engine.py:148), read by the kernel, so a captured CUDA graph
    replays at whatever position the tensor holds.  offset + L > cap is caught
    on the device (no write; rib_take_device_status reports RIB_ECAPACITY)."""
    L = _check_common(qkv, qw, kw, nq, nkv)
    require_bf16_cuda("cache_layer", cache_layer)
    require_same_device(qkv, cache_layer)
    if cache_layer.dim() != 4 or cache_layer.shape[0] != 2 or cache_layer.shape[1] != nkv \
            or cache_layer.shape[3] != HEAD_DIM:
        raise ValueError(f"cache_layer must be [2, {nkv}, cap, 128], got {tuple(cache_layer.shape)}")
    _require_i32_scalar("offset_dev", offset_dev, qkv.device)
    Lp = L if Lp is None else Lp
    if Lp < L:
        raise ValueError(f"Lp ({Lp}) must be >= L ({L})")
    q = _out_or_new(out, (nq, Lp, HEAD_DIM), torch.bfloat16, qkv.device, "out")
    st = _lib.load().rib_qk_norm_rope_append_dev(qkv.data_ptr(), L, qw.data_ptr(), kw.data_ptr(),
                                                 offset_dev.data_ptr(), nq, nkv, float(base), Lp,
                                                 q.data_ptr(), cache_layer.data_ptr(),
                                                 cache_layer.shape[2], stream_handle(qkv.device))
    _lib.check(st, "qk_norm_rope_append_at")
    return q


def qk_norm_rope_append_batched(qkv, qw, kw, pos, cache_ptrs, caps, nq: int, nkv: int, base: float,
                                out=None):
    """qk_norm_rope_append of one new token for each of B caches in one launch.

    qkv [B, (nq + 2 nkv) * 128] BF16; pos int32 CUDA [B] (each token's
    position, the cache row written); cache_ptrs int64 CUDA [B] (device
    addresses of [2, nkv, caps[b], 128] BF16 caches: sequences of a batch, or
    the layers of one decode step); caps int32 CUDA [B].  Returns q [B, nq,
    128].  A position outside [0, caps[b]) writes nothing for that row and is
    reported by rib_take_device_status (RIB_ECAPACITY)."""
    require_bf16_cuda("qkv", qkv)
    require_bf16_cuda("qw", qw)
    require_bf16_cuda("kw", kw)
    if qkv.dim() != 2 or qkv.shape[1] != (nq + 2 * nkv) * HEAD_DIM or not qkv.is_contiguous():
        raise ValueError(f"qkv must be contiguous [B, {(nq + 2 * nkv) * HEAD_DIM}]")
    B = qkv.shape[0]
    for name, t, dt in (("pos", pos, torch.int32), ("cache_ptrs", cache_ptrs, torch.int64),
                        ("caps", caps, torch.int32)):
        if not isinstance(t, torch.Tensor) or t.dtype != dt or not t.is_cuda or t.numel() != B \
                or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous {dt} CUDA tensor of {B} elements")
        require_same_device(qkv, t)
    q = _out_or_new(out, (B, nq, HEAD_DIM), torch.bfloat16, qkv.device, "out")
    st = _lib.load().rib_qk_norm_rope_append_batched(
        qkv.data_ptr(), qw.data_ptr(), kw.data_ptr(), pos.data_ptr(), cache_ptrs.data_ptr(), caps.data_ptr(), B,
        nq, nkv, float(base), q.data_ptr(), stream_handle(qkv.device))
    _lib.check(st, "qk_norm_rope_append_batched")
    return q


# ----------------------------------------------------------------- model ops
# The remaining operations of the Qwen3 forward (agent-test/v2/engine.py:102-163):
# fused GEMVs for decode, residual + RMSNorm, RMSNorm, SwiGLU, embedding gather
# and greedy argmax, each one kernel of csrc/model_kernels.cuh.

EPI_NONE, EPI_RESIDUAL, EPI_SWIGLU = 0, 1, 2
GEMV_WIDE = 0x100  # RIB_GEMV_WIDE launch hint


def _require_i32_scalar(name, t, device):
    if not isinstance(t, torch.Tensor) or t.dtype != torch.int32 or not t.is_cuda or t.numel() != 1:
        raise ValueError(f"{name} must be a one-element int32 CUDA tensor")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")


def _out_or_new(out, shape, dtype, device, name):
    if out is None:
        return torch.empty(shape, dtype=dtype, device=device)
    if not isinstance(out, torch.Tensor) or out.dtype != dtype or out.device != device \
            or not out.is_contiguous() or out.numel() != int(torch.Size(shape).numel()):
        raise ValueError(f"{name} must be a contiguous {dtype} tensor of {tuple(shape)} on {device}")
    return out


def gemv(W, x, *, nw=None, res=None, swiglu=False, out_float=False, cfg=None, out=None, wide=False):
    """y = epi(W @ pre(x)) for one token (agent-test/v2/kernels.py:103-113).

    W [N, K] BF16 (K a multiple of 8); x [K]; nw: fuse the input RMSNorm
    (eps 1e-6) with this weight; res: y = bf16(res + bf16(W x)); swiglu: W is
    [gate; up] and y[N/2] = bf16(bf16(g * bf16(sigmoid(g))) * u); out_float:
    FP32 output (the logits).  wide: the RIB_GEMV_WIDE launch form (same
    results; faster after another GEMV, slower right after the decode
    attention).  `cfg` (Metal launch tuning) is accepted and ignored."""
    del cfg
    require_bf16_cuda("W", W)
    require_bf16_cuda("x", x)
    require_same_device(W, x)
    if W.dim() != 2:
        raise ValueError(f"W must be [N, K], got {tuple(W.shape)}")
    N, K = W.shape
    if x.numel() != K:
        raise ValueError(f"x holds {x.numel()} elements, W has K = {K}")
    if K % 8:
        raise ValueError(f"K ({K}) must be a multiple of 8")
    if nw is not None:
        require_bf16_cuda("nw", nw)
        require_same_device(W, nw)
        if nw.numel() != K:
            raise ValueError("nw must hold K elements")
    if swiglu and (res is not None or out_float):
        raise ValueError("swiglu takes neither res nor out_float")
    if res is not None and out_float:
        raise ValueError("res and out_float do not combine")
    epi = EPI_SWIGLU if swiglu else (EPI_RESIDUAL if res is not None else EPI_NONE)
    if wide:
        epi |= GEMV_WIDE
    n_out = N // 2 if swiglu else N
    if res is not None:
        require_bf16_cuda("res", res)
        require_same_device(W, res)
        if res.numel() != N:
            raise ValueError("res must hold N elements")
    y = _out_or_new(out, (n_out,), torch.float32 if out_float else torch.bfloat16, W.device, "out")
    st = _lib.load().rib_gemv(W.data_ptr(), N, K, x.data_ptr(),
                              nw.data_ptr() if nw is not None else None,
                              res.data_ptr() if res is not None else None, epi, int(bool(out_float)),
                              y.data_ptr(), stream_handle(W.device))
    _lib.check(st, "gemv")
    return y


def add_rms(a, b, weight, *, out=None):
    """(a + b, rms_norm(a + b) * weight) over rows of a, b [..., W]
    (agent-test/v2/kernels.py:262-268).  Returns (residual, normalized)."""
    for name, t in (("a", a), ("b", b), ("weight", weight)):
        require_bf16_cuda(name, t)
    require_same_device(a, b, weight)
    if a.shape != b.shape:
        raise ValueError(f"a {tuple(a.shape)} and b {tuple(b.shape)} differ")
    W = a.shape[-1]
    if weight.numel() != W:
        raise ValueError("weight must hold the row width")
    rows = a.numel() // W
    r, n = (None, None) if out is None else out
    r = _out_or_new(r, a.shape, torch.bfloat16, a.device, "out[0]")
    n = _out_or_new(n, a.shape, torch.bfloat16, a.device, "out[1]")
    st = _lib.load().rib_add_rms(a.data_ptr(), b.data_ptr(), weight.data_ptr(), rows, W, r.data_ptr(),
                                 n.data_ptr(), stream_handle(a.device))
    _lib.check(st, "add_rms")
    return r.view(a.shape), n.view(a.shape)


def rms_norm(x, weight, eps: float = 1e-6, *, out=None):
    """bf16(weight * bf16(x / sqrt(mean(x^2) + 1e-6))) per row (mx.fast.rms_norm as
    called at agent-test/v2/engine.py:109, 140; eps is fixed at 1e-6)."""
    if abs(float(eps) - 1e-6) > 1e-12:
        raise ValueError("the kernel's eps is 1e-6 (Qwen3 rms_norm_eps)")
    require_bf16_cuda("x", x)
    require_bf16_cuda("weight", weight)
    require_same_device(x, weight)
    W = x.shape[-1]
    if weight.numel() != W:
        raise ValueError("weight must hold the row width")
    y = _out_or_new(out, x.shape, torch.bfloat16, x.device, "out")
    st = _lib.load().rib_rms_norm(x.data_ptr(), weight.data_ptr(), x.numel() // W, W, y.data_ptr(),
                                  stream_handle(x.device))
    _lib.check(st, "rms_norm")
    return y.view(x.shape)


def swiglu(gu, *, out=None):
    """gu [rows, 2F] (gate columns, then up) -> [rows, F]: the prefill SwiGLU
    (agent-test/v2/engine.py:28-30 applied to mx.split(x @ W_gu^T, 2, -1))."""
    require_bf16_cuda("gu", gu)
    F2 = gu.shape[-1]
    if F2 % 16:
        raise ValueError("gate/up width must be a multiple of 16")
    rows = gu.numel() // F2
    y = _out_or_new(out, (*gu.shape[:-1], F2 // 2), torch.bfloat16, gu.device, "out")
    st = _lib.load().rib_swiglu(gu.data_ptr(), rows, F2 // 2, y.data_ptr(), stream_handle(gu.device))
    _lib.check(st, "swiglu")
    return y


def embedding(table, tokens, *, out=None):
    """table[tokens] for int32 CUDA token ids (agent-test/v2/engine.py:108, 147)."""
    require_bf16_cuda("table", table)
    if not isinstance(tokens, torch.Tensor) or tokens.dtype != torch.int32 or not tokens.is_cuda \
            or not tokens.is_contiguous():
        raise ValueError("tokens must be a contiguous int32 CUDA tensor")
    require_same_device(table, tokens)
    vocab, hidden = table.shape
    n = tokens.numel()
    if n < 1:
        raise ValueError("no tokens")
    y = _out_or_new(out, (n, hidden), torch.bfloat16, table.device, "out")
    st = _lib.load().rib_embed(table.data_ptr(), vocab, hidden, tokens.data_ptr(), n, y.data_ptr(),
                               stream_handle(table.device))
    _lib.check(st, "embedding")
    return y


_argmax_ws: dict = {}


def argmax(logits, *, out=None, workspace=None):
    """Index of the largest FP32 logit (the first on ties) as an int32 [1]
    CUDA tensor (mx.argmax at agent-test/v2/engine.py:163)."""
    if not isinstance(logits, torch.Tensor) or logits.dtype != torch.float32 or not logits.is_cuda \
            or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous float32 CUDA tensor")
    dev = logits.device
    y = _out_or_new(out, (1,), torch.int32, dev, "out")
    if workspace is None:
        key = (dev.index, stream_handle(dev))
        workspace = _argmax_ws.get(key)
        if workspace is None:
            workspace = torch.empty(int(_lib.load().rib_argmax_workspace_bytes()), dtype=torch.uint8,
                                    device=dev)
            _argmax_ws[key] = workspace
    st = _lib.load().rib_argmax_f32(logits.data_ptr(), logits.numel(), y.data_ptr(), workspace.data_ptr(),
                                    stream_handle(dev))
    _lib.check(st, "argmax")
    return y
