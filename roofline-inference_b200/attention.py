"""Attention entry points with the reference's call signatures, backed by the
sm_100a kernels through the C ABI (include/rib_attention.h).

  attention(Q, K, V, qL, kL, scale, nsg=4, bk=16, kt=False, vf32=False, skip=True)
      causal GQA prefill (agent-test/v2/attention.py:177); tcgen05/TMEM kernel
      in csrc/prefill_attention.cuh.  The Metal tuning kwargs are accepted and
      ignored.
  decode_attention(q, cache_layer, n, scale)
      replaces mx.fast.scaled_dot_product_attention(q, K, V, scale) with
      K, V = cache.views(i, n) (agent-test/v2/engine.py:154-155); split-KV
      kernel in csrc/decode_attention.cuh.
  decode_attention_batched(q, caches, lens, scale, max_n=None)
      B independent sequences, each with its own contiguous cache and length.
"""
from __future__ import annotations

import threading

import torch

from . import _lib
from ._tensors import HEAD_DIM, require_bf16_cuda, require_same_device, stream_handle

# --------------------------------------------------------------- workspace
# Split-KV decode needs an FP32 scratch of partial results plus per-(sequence,
# KV head) counters in a fixed region at its start.  The counters must be zero
# before first use (the scratch is allocated zero-filled) and every call leaves
# them zero, so calls of any shape can share one scratch without a memset per
# call.  One workspace per (device, stream): calls on one stream never overlap.
_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def decode_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           stream_handle(device))
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
        return ws


_prefill_workspaces: dict = {}


def prefill_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Scratch of the prefill kernel (its FP16 copy of V), one buffer per
    (device, stream), grown on demand; a separate buffer from the decode
    workspace, whose counter region must stay zero."""
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           stream_handle(device))
    with _ws_lock:
        ws = _prefill_workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _prefill_workspaces[key] = ws
        return ws


# --------------------------------------------------------------- decode
def decode_attention(q, cache_layer, n: int, scale: float):
    """One query token against the first `n` keys of one cache layer.

    q: [1, nq, 1, 128] (or [nq, 128]) post-RoPE query; cache_layer:
    [2, nkv, cap, 128]; n: number of valid keys (cache.offset + 1 after the
    append).  Returns [1, nq, 1, 128] BF16, the layout
    mx.fast.scaled_dot_product_attention returns at engine.py:155."""
    require_bf16_cuda("q", q)
    require_bf16_cuda("cache_layer", cache_layer)
    require_same_device(q, cache_layer)
    if cache_layer.dim() != 4 or cache_layer.shape[0] != 2 or cache_layer.shape[3] != HEAD_DIM:
        raise ValueError(f"cache_layer must be [2, nkv, cap, 128], got {tuple(cache_layer.shape)}")
    nkv, cap = cache_layer.shape[1], cache_layer.shape[2]
    if q.numel() % HEAD_DIM:
        raise ValueError("q must hold nq * 128 elements")
    nq = q.numel() // HEAD_DIM
    n = int(n)
    if n > cap:
        raise ValueError("KV capacity exceeded")
    L = _lib.load()
    out = torch.empty((1, nq, 1, HEAD_DIM), dtype=torch.bfloat16, device=q.device)
    with torch.cuda.device(q.device):
        nbytes = L.rib_decode_workspace_bytes(1, max(n, 1), nkv)
        ws = decode_workspace(q.device, nbytes)
        st = L.rib_decode_attention(q.data_ptr(), cache_layer.data_ptr(), cap, n, nq, nkv,
                                    float(scale), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                    stream_handle(q.device))
    _lib.check(st, "decode_attention")
    return out


def decode_attention_batched(q, caches, lens, scale: float, max_n: int | None = None):
    """B sequences, one new token each.

    q: [B, nq, 128]; caches: a [B, 2, nkv, cap, 128] tensor or a list of B
    [2, nkv, cap, 128] tensors (same cap); lens: int32 CUDA tensor [B] of key
    counts (or a Python list); max_n: host bound on lens (computed from lens,
    with a device sync, when omitted).  Returns [B, nq, 128] BF16."""
    require_bf16_cuda("q", q)
    if q.dim() != 3 or q.shape[2] != HEAD_DIM:
        raise ValueError(f"q must be [B, nq, 128], got {tuple(q.shape)}")
    B, nq = q.shape[0], q.shape[1]
    dev = q.device
    if isinstance(caches, torch.Tensor):
        require_bf16_cuda("caches", caches)
        if caches.dim() != 5 or caches.shape[0] != B or caches.shape[1] != 2:
            raise ValueError(f"caches must be [B, 2, nkv, cap, 128], got {tuple(caches.shape)}")
        nkv, cap = caches.shape[2], caches.shape[3]
        stride = caches[0].numel() * caches.element_size()
        base = caches.data_ptr()
        ptrs = torch.tensor([base + b * stride for b in range(B)], dtype=torch.int64)
    else:
        if len(caches) != B:
            raise ValueError("need one cache per sequence")
        for c in caches:
            require_bf16_cuda("cache", c)
            require_same_device(q, c)
        nkv, cap = caches[0].shape[1], caches[0].shape[2]
        if any(tuple(c.shape) != (2, nkv, cap, HEAD_DIM) for c in caches):
            raise ValueError("every cache must be [2, nkv, cap, 128] with the same nkv and cap")
        ptrs = torch.tensor([c.data_ptr() for c in caches], dtype=torch.int64)
    ptrs = ptrs.to(dev, non_blocking=True)
    if isinstance(lens, torch.Tensor):
        lens_d = lens.to(device=dev, dtype=torch.int32)
        if max_n is None:
            max_n = int(lens_d.max().item())
    else:
        if max_n is None:
            max_n = max(int(x) for x in lens)
        lens_d = torch.tensor([int(x) for x in lens], dtype=torch.int32).to(dev, non_blocking=True)
    if max_n > cap:
        raise ValueError("KV capacity exceeded")
    L = _lib.load()
    out = torch.empty((B, nq, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        nbytes = L.rib_decode_workspace_bytes(B, max(int(max_n), 1), nkv)
        ws = decode_workspace(dev, nbytes)
        st = L.rib_decode_attention_batched(q.data_ptr(), ptrs.data_ptr(), lens_d.data_ptr(), B,
                                            int(max_n), cap, nq, nkv, float(scale),
                                            out.data_ptr(), ws.data_ptr(), ws.numel(),
                                            stream_handle(dev))
    _lib.check(st, "decode_attention_batched")
    # ptrs / lens_d may be freed now: the caching allocator only hands their
    # memory to later work on the same stream, which runs after this kernel.
    return out


def decode_attention_qkv(qkv, qw, kw, base: float, caches, lens, scale: float, max_n: int | None = None):
    """One decode step of B sequences with the new token's norm + RoPE +
    append fused into the attention launch (engine.py:150-155 in one kernel).

    qkv: [B, (nq + 2 nkv) * 128] projections of the new tokens; qw, kw: the
    per-head norm weights; caches as decode_attention_batched (the token of
    sequence b is appended at row lens[b] - 1, then attends over lens[b]
    keys).  Returns [B, nq, 128] BF16; outputs and cache rows equal
    qk_norm_rope_append followed by decode_attention_batched, bit for bit."""
    require_bf16_cuda("qkv", qkv)
    require_bf16_cuda("qw", qw)
    require_bf16_cuda("kw", kw)
    if qkv.dim() != 2 or not qkv.is_contiguous():
        raise ValueError(f"qkv must be contiguous [B, (nq + 2 nkv) * 128], got {tuple(qkv.shape)}")
    B, dev = qkv.shape[0], qkv.device
    if isinstance(caches, torch.Tensor):
        require_bf16_cuda("caches", caches)
        if caches.dim() != 5 or caches.shape[0] != B or caches.shape[1] != 2:
            raise ValueError(f"caches must be [B, 2, nkv, cap, 128], got {tuple(caches.shape)}")
        nkv, cap = caches.shape[2], caches.shape[3]
        stride = caches[0].numel() * caches.element_size()
        ptrs = torch.tensor([caches.data_ptr() + b * stride for b in range(B)], dtype=torch.int64)
    else:
        if len(caches) != B:
            raise ValueError("need one cache per sequence")
        nkv, cap = caches[0].shape[1], caches[0].shape[2]
        for c in caches:
            require_bf16_cuda("cache", c)
            require_same_device(qkv, c)
            if tuple(c.shape) != (2, nkv, cap, HEAD_DIM):
                raise ValueError("every cache must be [2, nkv, cap, 128] with the same nkv and cap")
        ptrs = torch.tensor([c.data_ptr() for c in caches], dtype=torch.int64)
    nq = 2 * nkv
    if qkv.shape[1] != (nq + 2 * nkv) * HEAD_DIM:
        raise ValueError(f"qkv rows must hold {(nq + 2 * nkv) * HEAD_DIM} values for {nkv} KV heads")
    ptrs = ptrs.to(dev, non_blocking=True)
    if isinstance(lens, torch.Tensor):
        lens_d = lens.to(device=dev, dtype=torch.int32)
        if max_n is None:
            max_n = int(lens_d.max().item())
    else:
        if max_n is None:
            max_n = max(int(x) for x in lens)
        lens_d = torch.tensor([int(x) for x in lens], dtype=torch.int32).to(dev, non_blocking=True)
    if max_n > cap:
        raise ValueError("KV capacity exceeded")
    L = _lib.load()
    out = torch.empty((B, nq, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        ws = decode_workspace(dev, L.rib_decode_workspace_bytes(B, max(int(max_n), 1), nkv))
        st = L.rib_decode_attention_qkv(qkv.data_ptr(), qw.data_ptr(), kw.data_ptr(), float(base), ptrs.data_ptr(),
                                        lens_d.data_ptr(), B, int(max_n), cap, nq, nkv, float(scale),
                                        out.data_ptr(), ws.data_ptr(), ws.numel(), stream_handle(dev))
    _lib.check(st, "decode_attention_qkv")
    return out


# --------------------------------------------------------------- prefill
def attention(Q, K, V, qL: int, kL: int, scale: float, nsg=4, bk=16, kt=False, vf32=False,
              skip=True):
    """Causal GQA flash attention for prefill.

    Q: [H, qLp, 128] post-RoPE queries (rows >= qL ignored); K, V: the cache
    halves [1, nkv, cap, 128] (buf[0:1], buf[1:2] of one layer) or
    [nkv, cap, 128]; query i sees keys <= kL - qL + i.  Returns [qL, H*128],
    the o_proj input layout (agent-test/v2/attention.py:177-185)."""
    del nsg, bk, kt, vf32, skip  # Metal launch tuning; no meaning here
    require_bf16_cuda("Q", Q)
    for name, t in (("K", K), ("V", V)):
        if not isinstance(t, torch.Tensor) or t.dtype != torch.bfloat16 or not t.is_cuda:
            raise ValueError(f"{name} must be a bfloat16 CUDA tensor")
    require_same_device(Q, K, V)
    Kc = K[0] if K.dim() == 4 else K
    Vc = V[0] if V.dim() == 4 else V
    if not Kc.is_contiguous() or not Vc.is_contiguous():
        raise ValueError("K and V must be contiguous [nkv, cap, 128]")
    if Q.dim() != 3 or Q.shape[2] != HEAD_DIM:
        raise ValueError(f"Q must be [H, qLp, 128], got {tuple(Q.shape)}")
    H, qLp = Q.shape[0], Q.shape[1]
    nkv, cap = Kc.shape[0], Kc.shape[1]
    if tuple(Vc.shape) != tuple(Kc.shape) or Kc.shape[2] != HEAD_DIM:
        raise ValueError("K and V must both be [nkv, cap, 128]")
    if H != 2 * nkv:
        raise ValueError("attention assumes GQA factor 2 (H == 2 * nkv)")
    qL, kL = int(qL), int(kL)
    if not (1 <= qL <= qLp and qL <= kL <= cap):
        raise ValueError(f"need 1 <= qL <= qLp and qL <= kL <= cap (qL={qL}, qLp={qLp}, "
                         f"kL={kL}, cap={cap})")
    out = torch.empty((qL, H * HEAD_DIM), dtype=torch.bfloat16, device=Q.device)
    L = _lib.load()
    ws = prefill_workspace(Q.device, int(L.rib_prefill_workspace_bytes(kL, nkv)))
    st = L.rib_prefill_attention(Q.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), qL, kL, qLp, cap, H, nkv,
                                 float(scale), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                 stream_handle(Q.device))
    _lib.check(st, "attention")
    return out
