"""Prefill projections on the tcgen05 GEMM (csrc/gemm.cuh) through the C ABI.

The reference's engine multiplies a prompt's activations by each projection
with `matmul` (agent-test/v2/engine.py:95-99): mx.matmul for more than 32
rows, a library GEMM.  Here the same products run on this package's own
kernel, with the step that follows each projection fused into its epilogue:

  gemm(A, W)                    C = bf16(A W^T)                      (O, down)
  gemm(A, W, epi="f32")         C = A W^T in FP32       (tensor-parallel partials)
  gemm(A, W, epi="swiglu")      C = swiglu(A W^T), W = [gate; up]    (engine.py:133)
  gemm_qkv_rope(A, W, ...)      the QKV projection with the per-head RMSNorm,
                                RoPE and KV-cache append fused (engine.py:111-113)

All tensors are BF16 CUDA tensors (the RoPE table FP32); results are
allocated by torch and the kernels run on torch's current stream.
"""
from __future__ import annotations

import torch

from . import _lib
from ._tensors import HEAD_DIM, require_bf16_cuda, require_same_device, stream_handle

RIB_GEMM_BF16, RIB_GEMM_F32, RIB_GEMM_SWIGLU = 0, 1, 2
_EPI = {"bf16": RIB_GEMM_BF16, "f32": RIB_GEMM_F32, "swiglu": RIB_GEMM_SWIGLU}


def _bind(L) -> None:
    import ctypes
    vp, i, d, ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_double, ctypes.c_longlong
    L.rib_gemm.argtypes = [vp, i, i, vp, i, i, vp, ll, vp]
    L.rib_gemm.restype = i
    L.rib_rope_table.argtypes = [i, i, d, vp, vp]
    L.rib_rope_table.restype = i
    L.rib_gemm_qkv_rope.argtypes = [vp, i, i, vp, i, i, vp, vp, vp, i, vp, i, vp, i, vp]
    L.rib_gemm_qkv_rope.restype = i
    L.rib_gemm_small_workspace_bytes.argtypes = [i, i, i]
    L.rib_gemm_small_workspace_bytes.restype = ctypes.c_size_t
    L.rib_gemm_small.argtypes = [vp, i, i, vp, i, i, vp, ll, vp, ctypes.c_size_t, vp]
    L.rib_gemm_small.restype = i


_bound = None


def _L():
    global _bound
    L = _lib.load()
    if _bound is not L:
        _bind(L)
        _bound = L
    return L


def _check_operands(A, W):
    require_bf16_cuda("A", A)
    require_bf16_cuda("W", W)
    require_same_device(A, W)
    if A.dim() != 2 or W.dim() != 2 or A.shape[1] != W.shape[1]:
        raise ValueError(f"need A [M, K] and W [N, K], got {tuple(A.shape)} and {tuple(W.shape)}")
    if A.shape[1] % 64:
        raise ValueError(f"K ({A.shape[1]}) must be a multiple of 64")


SMALL_M = 64  # rows up to which gemm() takes the few-row kernel

_small_ws: dict[int, torch.Tensor] = {}


def _small_workspace(device, nbytes: int) -> torch.Tensor:
    """One partials buffer per device, grown on demand (a CUDA graph that
    captures gemm() must have run it once at its largest shape first)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _small_ws.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _small_ws[idx] = ws
    return ws


def small_ok(M: int, N: int, K: int, epi: str) -> bool:
    """Whether rib_gemm_small takes this shape."""
    cols = N // 2 if epi == "swiglu" else N
    return (1 <= M <= SMALL_M and epi in ("bf16", "swiglu") and N % 128 == 0 and K % 64 == 0
            and cols % 8 == 0)


def gemm(A: torch.Tensor, W: torch.Tensor, *, epi: str = "bf16", out: torch.Tensor | None = None,
         small: bool | None = None) -> torch.Tensor:
    """epi(A W^T) for A [M, K], W [N, K] (K a multiple of 64).

    epi "bf16": [M, N] BF16 (N a multiple of 8); "f32": [M, N] FP32;
    "swiglu": W = [gate; up] with N = 2F rows (F a multiple of 128), returns
    [M, F] = bf16(bf16(g bf16(sigmoid(g))) u), g and u the BF16 products.
    small: the few-row kernel (rib_gemm_small: weights as the 128-row
    operand, K split over the GPU); by default for M <= 64 where it applies."""
    _check_operands(A, W)
    if epi not in _EPI:
        raise ValueError(f"unknown epilogue {epi!r}")
    M, K = A.shape
    N = W.shape[0]
    cols = N // 2 if epi == "swiglu" else N
    dtype = torch.float32 if epi == "f32" else torch.bfloat16
    if out is None:
        out = torch.empty((M, cols), dtype=dtype, device=A.device)
    elif out.dtype != dtype or out.shape != (M, cols) or not out.is_contiguous() or out.device != A.device:
        raise ValueError(f"out must be a contiguous {dtype} tensor [{M}, {cols}] on {A.device}")
    if small is None:
        small = small_ok(M, N, K, epi)
    L = _L()
    if small:
        if not small_ok(M, N, K, epi):
            raise ValueError(f"the few-row GEMM does not take M={M}, N={N}, K={K}, epi={epi!r}")
        nbytes = int(L.rib_gemm_small_workspace_bytes(M, N, K))
        ws = _small_workspace(A.device, nbytes)
        st = L.rib_gemm_small(A.data_ptr(), M, K, W.data_ptr(), N, _EPI[epi], out.data_ptr(), cols,
                              ws.data_ptr(), ws.numel(), stream_handle(A.device))
        _lib.check(st, "gemm_small")
        return out
    st = L.rib_gemm(A.data_ptr(), M, K, W.data_ptr(), N, _EPI[epi], out.data_ptr(), cols,
                    stream_handle(A.device))
    _lib.check(st, "gemm")
    return out


def rope_table(pos0: int, count: int, base: float, device) -> torch.Tensor:
    """(cos, sin) of the 64 RoPE angles of positions pos0 .. pos0 + count - 1,
    FP32 [count, 64, 2], the angles as the reference forms them
    (agent-test/v2/kernels.py:134-138)."""
    t = torch.empty((max(int(count), 1), 64, 2), dtype=torch.float32, device=device)
    st = _L().rib_rope_table(int(pos0), int(count), float(base), t.data_ptr(), stream_handle(t.device))
    _lib.check(st, "rope_table")
    return t


def gemm_qkv_rope(A: torch.Tensor, W: torch.Tensor, qw: torch.Tensor, kw: torch.Tensor, table: torch.Tensor,
                  pos0: int, nq: int, nkv: int, cache_layer: torch.Tensor, Lp: int | None = None) -> torch.Tensor:
    """The QKV projection of M prompt tokens at positions pos0 .. pos0 + M - 1
    with the per-head RMSNorm + RoPE + KV append fused: returns Q
    [nq, Lp, 128] (rows past M zero) and writes the tokens' K and V into
    cache_layer [2, nkv, cap, 128] -- what matmul(x, qkv), qk_norm_rope_prefill
    and Cache.update do in Engine.prefill (engine.py:111-113).  table:
    rope_table(pos0, >= M, base)."""
    _check_operands(A, W)
    for name, t in (("qw", qw), ("kw", kw), ("cache_layer", cache_layer)):
        require_bf16_cuda(name, t)
    require_same_device(A, W, qw, kw, cache_layer, table)
    M, K = A.shape
    if W.shape[0] != (nq + 2 * nkv) * HEAD_DIM:
        raise ValueError(f"W must have (nq + 2 nkv) * 128 = {(nq + 2 * nkv) * HEAD_DIM} rows")
    if cache_layer.dim() != 4 or cache_layer.shape[0] != 2 or cache_layer.shape[1] != nkv \
            or cache_layer.shape[3] != HEAD_DIM:
        raise ValueError(f"cache_layer must be [2, {nkv}, cap, 128], got {tuple(cache_layer.shape)}")
    if table.dtype != torch.float32 or not table.is_contiguous() or table.numel() < M * 128:
        raise ValueError("table must be a contiguous FP32 rope_table of at least M positions")
    Lp = M if Lp is None else int(Lp)
    if Lp < M:
        raise ValueError(f"Lp ({Lp}) must be >= M ({M})")
    q = torch.empty((nq, Lp, HEAD_DIM), dtype=torch.bfloat16, device=A.device)
    st = _L().rib_gemm_qkv_rope(A.data_ptr(), M, K, W.data_ptr(), nq, nkv, qw.data_ptr(), kw.data_ptr(),
                                table.data_ptr(), int(pos0), q.data_ptr(), Lp, cache_layer.data_ptr(),
                                cache_layer.shape[2], stream_handle(A.device))
    _lib.check(st, "gemm_qkv_rope")
    return q
