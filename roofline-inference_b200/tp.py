"""Tensor parallelism of the Qwen3 projections over the GPUs of one node.

The single-GPU reference runs every GEMV of a decode step on one device
(Engine.decode, agent-test/v2/engine.py:150-162).  Split over N ranks:

  - rank r keeps KV heads head_range(r, N): their rows of the QKV projection,
    their cache and their attention (as the KV-head sharded engine);
  - the O projection keeps the columns of r's query heads, the gate and up
    projections a slice of the intermediate rows, the down projection the
    matching columns, the LM head a slice of the vocabulary rows;
  - the O and down GEMVs then produce FP32 partial sums of the hidden vector.
    Each rank's GEMV stores its partials straight into every rank's exchange
    buffer over NVLink (RIB_EPI_PEER_PARTIAL), each value in an 8-byte word
    tagged with the exchange's epoch; the next GEMV of every rank polls the
    words until they carry the epoch and forms its input as
    bf16(residual + bf16(sum of partials in rank order)).  No fence, flag or
    separate collective runs, and every rank computes the same activations;
  - the LM-head slices give per-rank argmax keys, exchanged the same way, so
    every rank gets the same token.

Per layer each rank reads 1/N of the projection weights, at the price of two
cross-GPU exchanges (a few KB each).

A prefill's O and down projections are GEMMs over M prompt rows; their
exchange (PrefillExchange) splits the rows over the ranks: the tcgen05 GEMM's
epilogue stores each row's FP32 partial into its owner rank's receive slot
over NVLink, and one kernel then sums each owned row in rank order, stores the
BF16 row into every rank's gather buffer and applies the residual add and
RMSNorm to all rows -- a reduce-scatter and an all-gather fused into the
GEMM and the add_rms, with no NCCL call.  Setup and close() are collective.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .peer_memory import PeerBuffers

MAX_RANKS = 8
EPI_PEER_PARTIAL = 3


class _TpExchangeStruct(ctypes.Structure):
    """rib_tp_exchange (include/rib_attention.h)."""
    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int),
                ("buf", ctypes.c_uint64 * MAX_RANKS), ("epoch", ctypes.c_uint64),
                ("done", ctypes.c_uint64), ("slot", ctypes.c_int)]


class _PrefillExchangeStruct(ctypes.Structure):
    """rib_tp_prefill_exchange (include/rib_attention.h)."""
    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int),
                ("buf", ctypes.c_uint64 * MAX_RANKS), ("rows_cap", ctypes.c_int), ("hidden", ctypes.c_int)]


def _bind(L: ctypes.CDLL) -> None:
    vp, i, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    L.rib_tp_buffer_bytes.argtypes = [i, i]
    L.rib_tp_buffer_bytes.restype = sz
    L.rib_gemv_tp.argtypes = [vp, i, i, vp, vp, i, i, vp, ctypes.POINTER(_TpExchangeStruct), i, vp, vp]
    L.rib_gemv_tp.restype = i
    L.rib_argmax_f32_tp.argtypes = [vp, i, i, vp, vp, ctypes.POINTER(_TpExchangeStruct), vp]
    L.rib_argmax_f32_tp.restype = i
    L.rib_tp_prefill_buffer_bytes.argtypes = [i, i, i]
    L.rib_tp_prefill_buffer_bytes.restype = sz
    L.rib_gemm_tp_partial.argtypes = [vp, i, i, vp, ctypes.POINTER(_PrefillExchangeStruct), vp]
    L.rib_gemm_tp_partial.restype = i
    L.rib_tp_reduce_add_rms.argtypes = [ctypes.POINTER(_PrefillExchangeStruct), i, ctypes.c_ulonglong, vp, vp, vp,
                                        vp]
    L.rib_tp_reduce_add_rms.restype = i


def split_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [a, b) of an n-row dimension owned by `rank` (n % world == 0)."""
    if world < 1 or not 0 <= rank < world or n % world:
        raise ValueError(f"{n} does not split evenly over {world} ranks")
    k = n // world
    return rank * k, (rank + 1) * k


def shard_layer(layer: dict, h0: int, h1: int, f0: int, f1: int, nq: int, nkv: int) -> dict:
    """One layer's weights for the rank owning KV heads [h0, h1) and
    intermediate rows [f0, f1): QKV rows of those heads, O columns of their
    query heads, gate rows and up rows [f0, f1) (gate block first, as the
    SwiGLU epilogue reads them), down columns [f0, f1)."""
    from .model import HEAD_DIM, _shard_qkv_rows
    F = layer["gu"].shape[0] // 2
    out = dict(layer)
    out["qkv"] = _shard_qkv_rows(layer["qkv"], h0, h1, nq, nkv)
    out["o"] = layer["o"][:, 2 * h0 * HEAD_DIM:2 * h1 * HEAD_DIM].contiguous()
    out["gu"] = torch.cat([layer["gu"][f0:f1], layer["gu"][F + f0:F + f1]]).contiguous()
    out["down"] = layer["down"][:, f0:f1].contiguous()
    return out


class TPExchange:
    """This rank's exchange buffer, its peers' mappings and the device
    counters; `struct` is the rib_tp_exchange to pass to the kernels.
    slot: the longest vector exchanged (words; rounded up to a multiple of 4)."""

    def __init__(self, slot: int, device, group=None):
        self.L = L = _lib.load()
        _bind(L)
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if self.world > MAX_RANKS:
            raise ValueError(f"at most {MAX_RANKS} ranks")
        self.device = torch.device(device)
        self.dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.slot = (int(slot) + 3) // 4 * 4
        self.nbytes = int(L.rib_tp_buffer_bytes(self.world, self.slot))
        if self.nbytes == 0:
            raise ValueError("bad exchange geometry")
        self.peers = PeerBuffers(self.nbytes, self.device, group)
        self.base = self.peers.base
        self.epoch = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        s = _TpExchangeStruct()
        s.world, s.rank, s.slot = self.world, self.rank, self.slot
        for r in range(self.world):
            s.buf[r] = self.base[r]
        s.epoch, s.done = self.epoch.data_ptr(), self.done.data_ptr()
        self.struct = s
        self.closed = False
        dist.barrier(group=group)

    def gemv(self, W, x, *, nw=None, epi: int = 0, out=None, out_float: bool = False, in_sum: bool = False,
             x_out=None, stream=None):
        """rib_gemv_tp on torch's current stream; returns `out`."""
        from ._tensors import stream_handle
        if self.closed:
            raise RuntimeError("TPExchange is closed")
        st = stream_handle(self.device) if stream is None else stream
        N, K = W.shape
        _lib.check(self.L.rib_gemv_tp(
            W.data_ptr(), N, K, x.data_ptr(), None if nw is None else nw.data_ptr(), epi, int(out_float),
            None if out is None else out.data_ptr(), ctypes.byref(self.struct), int(in_sum),
            None if x_out is None else x_out.data_ptr(), st), "gemv_tp")
        return out

    def argmax(self, logits, offset: int, out, workspace):
        """Global greedy token over every rank's logit slice into out (int32 [1])."""
        from ._tensors import stream_handle
        _lib.check(self.L.rib_argmax_f32_tp(logits.data_ptr(), logits.numel(), int(offset), out.data_ptr(),
                                            workspace.data_ptr(), ctypes.byref(self.struct),
                                            stream_handle(self.device)), "argmax_f32_tp")
        return out

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's."""
        if self.closed:
            return
        self.peers.close()
        self.closed = True


class PrefillExchange:
    """The exchange after the row-parallel O and down projections of a
    tensor-parallel prefill (the add_rms after each projection of
    Engine.prefill, agent-test/v2/engine.py:111-116), fused over NVLink in
    place of an NCCL all-reduce.  rib_gemm_tp_partial stores each row's FP32
    partial into the owner rank's receive slot (rows split over the ranks in
    contiguous runs); rib_tp_reduce_add_rms sums each owned row in rank
    order, rounds it to BF16, stores it into every rank's gather buffer and
    then applies residual add + RMSNorm to all rows on every rank.

    rows_cap: the most rows one call may carry.  Setup and close() are
    collective, and every rank makes the same calls in the same order.
    local=True makes a one-rank exchange over a plain device buffer, with no
    process group: every row is this rank's own and every signal its own
    (the two kernels alone, for tests and profiling)."""

    def __init__(self, hidden: int, rows_cap: int, device, group=None, *, local: bool = False):
        self.L = L = _lib.load()
        _bind(L)
        if local:
            self.world, self.rank = 1, 0
        else:
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if self.world > MAX_RANKS:
            raise ValueError(f"at most {MAX_RANKS} ranks")
        self.device = torch.device(device)
        self.hidden, self.rows_cap = int(hidden), int(rows_cap)
        nbytes = int(L.rib_tp_prefill_buffer_bytes(self.world, self.rows_cap, self.hidden))
        if nbytes == 0:
            raise ValueError(f"unsupported prefill exchange geometry (hidden {hidden}, rows {rows_cap})")
        self.peers, self._local = None, None
        if local:
            self._local = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            base = [self._local.data_ptr()]
        else:
            self.peers = PeerBuffers(nbytes, self.device, group)
            base = self.peers.base
        s = _PrefillExchangeStruct()
        s.world, s.rank, s.rows_cap, s.hidden = self.world, self.rank, self.rows_cap, self.hidden
        for r in range(self.world):
            s.buf[r] = base[r]
        self.struct = s
        self.epoch = 0
        self.closed = False

    def project_add_rms(self, x, W, residual, norm_w=None, out=None):
        """residual <- bf16(residual + bf16(sum over ranks of x W^T)), in place;
        with norm_w, out <- its RMSNorm (allocated when None).  x [M, K] BF16
        (this rank's columns of the projection's input), W [hidden, K] BF16,
        residual [M, hidden] BF16.  Returns (residual, out)."""
        from ._tensors import stream_handle
        if self.closed:
            raise RuntimeError("PrefillExchange is closed")
        M, K = x.shape
        if W.shape != (self.hidden, K) or residual.shape != (M, self.hidden) or M > self.rows_cap:
            raise ValueError(f"shapes x {tuple(x.shape)}, W {tuple(W.shape)}, residual "
                             f"{tuple(residual.shape)} do not fit the exchange (hidden {self.hidden}, "
                             f"rows {self.rows_cap})")
        for t in (x, W, residual):
            if not (t.is_contiguous() and t.dtype == torch.bfloat16 and t.device == self.device):
                raise ValueError("x, W and residual must be contiguous BF16 tensors on the exchange's device")
        if norm_w is not None and out is None:
            out = torch.empty_like(residual)
        st = stream_handle(self.device)
        self.epoch += 1
        _lib.check(self.L.rib_gemm_tp_partial(x.data_ptr(), M, K, W.data_ptr(), ctypes.byref(self.struct), st),
                   "gemm_tp_partial")
        _lib.check(self.L.rib_tp_reduce_add_rms(
            ctypes.byref(self.struct), M, self.epoch, residual.data_ptr(),
            None if norm_w is None else norm_w.data_ptr(), None if out is None else out.data_ptr(), st),
            "tp_reduce_add_rms")
        return residual, out

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's."""
        if self.closed:
            return
        if self.peers is not None:
            self.peers.close()
        self._local = None
        self.closed = True
