"""Decode attention fused with the NVLink all-gather of head outputs.

With the KV heads sharded over the GPUs of one node (sharding.head_range),
each rank's decode kernel stores every finished head output straight into
every rank's gathered buffer through CUDA IPC peer mappings and exchanges an
epoch flag with its peers, so no separate collective runs.  The reference is
single-GPU; this replaces the decode SDPA (agent-test/v2/engine.py:155) plus
the all-gather a head-sharded engine needs.

Setup is collective: every rank constructs NVLinkGather with the same
arguments inside an initialised torch.distributed process group (used only
to exchange the 64-byte IPC handles); every rank then makes the same
sequence of decode() calls; close() is collective too.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .peer_memory import PeerBuffers
from ._tensors import require_bf16_cuda, stream_handle

MAX_PEERS = 8


class _PeerGatherStruct(ctypes.Structure):
    """rib_peer_gather (include/rib_attention.h)."""
    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int),
                ("out", ctypes.c_uint64 * MAX_PEERS), ("sig", ctypes.c_uint64 * MAX_PEERS),
                ("region_bytes", ctypes.c_size_t)]


class _DeviceView:
    """Exposes raw device memory to torch (__cuda_array_interface__ v3)."""

    def __init__(self, ptr: int, shape: tuple[int, ...]):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": "<i2", "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


def _bind(L: ctypes.CDLL) -> None:
    vp, i, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    L.rib_peer_buffer_bytes.argtypes = [i, i]
    L.rib_peer_buffer_bytes.restype = sz
    L.rib_decode_attention_gather.argtypes = [vp, vp, vp, i, i, i, i, i, ctypes.c_float,
                                              ctypes.POINTER(_PeerGatherStruct),
                                              ctypes.c_ulonglong, vp, sz, vp]
    L.rib_decode_attention_gather.restype = i
    L.rib_decode_attention_gather_dev.argtypes = [vp, vp, vp, i, i, i, i, i, ctypes.c_float,
                                                  ctypes.POINTER(_PeerGatherStruct), vp, vp, vp, sz, vp]
    L.rib_decode_attention_gather_dev.restype = i


class NVLinkGather:
    """Per-rank state: this rank's gathered buffer and its peers' mappings.

    batch: sequences (or independent layers) per call; nq_local: query heads
    owned by this rank (2 x its KV heads)."""

    def __init__(self, batch: int, nq_local: int, device, group=None):
        self.L = _lib.load()
        _bind(self.L)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > MAX_PEERS:
            raise ValueError(f"at most {MAX_PEERS} ranks per NVLink gather")
        self.device = torch.device(device)
        self.dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.batch, self.nq_local = batch, nq_local
        self.nq_total = nq_local * self.world
        self.nbytes = self.L.rib_peer_buffer_bytes(batch, self.nq_total)
        self.region_bytes = (self.nbytes - 256) // 2
        self.peers = PeerBuffers(self.nbytes, self.device, group)
        self.base = self.peers.base
        self.g = _PeerGatherStruct()
        self.g.world, self.g.rank, self.g.region_bytes = self.world, self.rank, self.region_bytes
        for r in range(self.world):
            self.g.out[r] = self.base[r]
            self.g.sig[r] = self.base[r] + 2 * self.region_bytes
        self.epoch = 0
        self._views = [torch.as_tensor(
            _DeviceView(self.base[self.rank] + k * self.region_bytes,
                        (batch, self.nq_total, 128)), device=self.device).view(torch.bfloat16)
            for k in range(2)]
        self.closed = False
        dist.barrier(group=group)

    def output(self) -> torch.Tensor:
        """Gathered outputs of the last call, [batch, world*nq_local, 128]."""
        return self._views[self.epoch & 1]

    def decode(self, q, cache_ptrs, lens, max_n: int, cap: int, scale: float,
               workspace: torch.Tensor) -> torch.Tensor:
        """One fused decode + all-gather on torch's current stream.

        q [batch, nq_local, 128]; cache_ptrs int64 CUDA tensor of `batch`
        cache addresses ([2, nkv_local, cap, 128] each); lens int32 CUDA
        tensor; workspace uint8 CUDA tensor of rib_decode_workspace_bytes
        (zeroed once).  Returns the gathered view of this call."""
        require_bf16_cuda("q", q)
        if self.closed:
            raise RuntimeError("NVLinkGather is closed")
        self.epoch += 1
        nkv = self.nq_local // 2
        st = self.L.rib_decode_attention_gather(
            q.data_ptr(), cache_ptrs.data_ptr(), lens.data_ptr(), self.batch, int(max_n), int(cap),
            self.nq_local, nkv, float(scale), ctypes.byref(self.g), self.epoch,
            workspace.data_ptr(), workspace.numel(), stream_handle(self.device))
        _lib.check(st, "decode_attention_gather")
        return self.output()

    def decode_into(self, q, cache_ptrs, lens, max_n: int, cap: int, scale: float, workspace: torch.Tensor,
                    epoch_dev: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """decode() with the epoch in `epoch_dev` (int64 CUDA tensor of one
        element, zero on every rank before the first call) and the gathered
        outputs copied into `out` [batch, world*nq_local, 128]: every argument
        is a fixed device address, so the call can be captured in a CUDA graph
        and replayed."""
        require_bf16_cuda("q", q)
        require_bf16_cuda("out", out)
        if self.closed:
            raise RuntimeError("NVLinkGather is closed")
        if out.numel() != self.batch * self.nq_total * 128:
            raise ValueError("out must hold [batch, world * nq_local, 128]")
        if epoch_dev.dtype != torch.int64 or epoch_dev.numel() != 1 or not epoch_dev.is_cuda:
            raise ValueError("epoch_dev must be a one-element int64 CUDA tensor")
        nkv = self.nq_local // 2
        st = self.L.rib_decode_attention_gather_dev(
            q.data_ptr(), cache_ptrs.data_ptr(), lens.data_ptr(), self.batch, int(max_n), int(cap),
            self.nq_local, nkv, float(scale), ctypes.byref(self.g), epoch_dev.data_ptr(), out.data_ptr(),
            workspace.data_ptr(), workspace.numel(), stream_handle(self.device))
        _lib.check(st, "decode_attention_gather_dev")
        return out

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's."""
        if self.closed:
            return
        self.peers.close()
        self._views = []
        self.closed = True
