"""ctypes wrapper of the C oracle (oracle.c) -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, as the checker of (or the timed CPU stand-in for) the CUDA path.  The
product path never imports it.

All tensors are numpy arrays; BF16 data is carried as uint16 bit patterns.
Semantics and reference citations are in oracle.c.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

from . import build as _build

_LIB = None

_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = _build.build()
        L = ctypes.CDLL(str(path))
        L.oracle_qk_norm_rope.argtypes = [_u16p, ctypes.c_int, _u16p, _u16p, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_int, ctypes.c_double,
                                          ctypes.c_int, _u16p, _u16p, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int]
        L.oracle_qk_norm_rope.restype = None
        L.oracle_decode_attention_batched.argtypes = [
            _u16p, ctypes.POINTER(ctypes.c_void_p), _i32p, ctypes.c_int, ctypes.c_int,
            ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
        L.oracle_decode_attention_batched.restype = None
        L.oracle_prefill_attention.argtypes = [_u16p, _u16p, _u16p, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                               ctypes.c_int, _f32p]
        L.oracle_prefill_attention.restype = None
        _LIB = L
    return _LIB


def set_threads(n: int | None) -> int:
    """Sets the OpenMP thread count used by later calls; returns it."""
    n = n or os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(n)
    try:
        gomp = ctypes.CDLL("libgomp.so.1")
        gomp.omp_set_num_threads(ctypes.c_int(n))
    except OSError:
        pass
    return n


def _u16(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint16)


def qk_norm_rope(qkv, qw, kw, offset: int, nq: int, nkv: int, base: float, Lp: int | None = None,
                 angle_f64: bool = False):
    """qkv [L, (nq+2nkv)*128] u16 -> (Q [nq, Lp, 128] u16 with zero pad rows,
    KV [2, nkv, L, 128] u16).  agent-test/v2/kernels.py:169-224.

    The RoPE angle is the reference's FP32 one (kernels.py:134-138); with
    angle_f64 it is formed in FP64 instead (the idealised rope)."""
    qkv = _u16(qkv).reshape(-1, (nq + 2 * nkv) * 128)
    L = qkv.shape[0]
    Lp = L if Lp is None else Lp
    q = np.zeros((nq, Lp, 128), np.uint16)
    kv = np.zeros((2, nkv, L, 128), np.uint16)
    lib().oracle_qk_norm_rope(qkv, L, _u16(qw), _u16(kw), int(offset), nq, nkv, float(base), Lp,
                              q, kv, L, 0, int(bool(angle_f64)))
    return q, kv


def decode_attention_batched(q, caches, lens, scale: float):
    """q [B, nq, 128] u16; caches: B arrays [2, nkv, cap, 128] u16 (same cap);
    lens [B].  Returns (out_f32 [B, nq, 128], out_bf16 [B, nq, 128] u16).
    Restates mx.fast.scaled_dot_product_attention at agent-test/v2/engine.py:155."""
    q = _u16(q)
    B, nq, _ = q.shape
    caches = [_u16(c) for c in caches]
    nkv, cap = caches[0].shape[1], caches[0].shape[2]
    ptrs = (ctypes.c_void_p * B)(*[c.ctypes.data for c in caches])
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    of = np.zeros((B, nq, 128), np.float32)
    ob = np.zeros((B, nq, 128), np.uint16)
    lib().oracle_decode_attention_batched(q, ptrs, lens, B, cap, nq, nkv, float(scale),
                                          of.ctypes.data, ob.ctypes.data)
    return of, ob


def decode_attention(q, cache, n: int, scale: float):
    """q [nq, 128] u16, cache [2, nkv, cap, 128] u16 -> (out_f32 [nq,128], out_bf16)."""
    q = _u16(q)
    of, ob = decode_attention_batched(q[None], [cache], [n], scale)
    return of[0], ob[0]


def prefill_attention(Q, K, V, qL: int, kL: int, scale: float, rows=None):
    """Q [H, qLp, 128], K/V [nkv, cap, 128] u16 -> O [qL, H*128] float32.
    rows: optional (begin, end) subset of query rows; other rows are NaN.
    Restates agent-test/v2/attention.py:177 (bottom-right causal mask)."""
    Q, K, V = _u16(Q), _u16(K), _u16(V)
    H, qLp, _ = Q.shape
    nkv, cap, _ = K.shape
    r0, r1 = (0, qL) if rows is None else rows
    out = np.full((qL, H * 128), np.nan, np.float32)
    lib().oracle_prefill_attention(Q, K, V, qL, kL, qLp, cap, H, nkv, float(scale), r0, r1, out)
    return out
