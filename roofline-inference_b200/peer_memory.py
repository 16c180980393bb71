"""Device buffers shared between the ranks of one node over NVLink.

Each rank cudaMallocs a zeroed buffer and exports a CUDA IPC handle
(rib_peer_buffer_alloc); the 64-byte handles are exchanged with
torch.distributed.all_gather_object, and every rank maps every peer's buffer
(rib_peer_buffer_open), so a kernel can store into any rank's buffer with
plain stores over NVLink.  Used by the fused decode all-gather
(nvlink_gather.py) and the tensor-parallel exchange (tp.py).  Both calls are
collective."""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib


def bind(L: ctypes.CDLL) -> None:
    vp, i, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    L.rib_peer_buffer_alloc.argtypes = [i, sz, ctypes.POINTER(ctypes.c_void_p), vp]
    L.rib_peer_buffer_alloc.restype = i
    L.rib_peer_buffer_open.argtypes = [i, vp, ctypes.POINTER(ctypes.c_void_p)]
    L.rib_peer_buffer_open.restype = i
    L.rib_peer_buffer_close.argtypes = [i, vp]
    L.rib_peer_buffer_close.restype = i
    L.rib_peer_buffer_free.argtypes = [i, vp]
    L.rib_peer_buffer_free.restype = i


class PeerBuffers:
    """This rank's buffer of `nbytes` and its mappings of every peer's:
    base[r] is rank r's buffer as seen from this process."""

    def __init__(self, nbytes: int, device, group=None):
        self.L = _lib.load()
        bind(self.L)
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        dev = torch.device(device)
        self.dev = dev.index if dev.index is not None else torch.cuda.current_device()
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        _lib.check(self.L.rib_peer_buffer_alloc(self.dev, nbytes, ctypes.byref(own), handle),
                   "rib_peer_buffer_alloc")
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.base = [0] * self.world
        self._opened: list[int] = []
        for r in range(self.world):
            if r == self.rank:
                self.base[r] = own.value
                continue
            ptr = ctypes.c_void_p()
            buf = ctypes.create_string_buffer(handles[r], 64)
            _lib.check(self.L.rib_peer_buffer_open(self.dev, buf, ctypes.byref(ptr)), "rib_peer_buffer_open")
            self.base[r] = ptr.value
            self._opened.append(ptr.value)
        self.closed = False

    def close(self) -> None:
        """Collective: every rank unmaps its peers' buffers, then frees its own."""
        if self.closed:
            return
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        for ptr in self._opened:
            self.L.rib_peer_buffer_close(self.dev, ctypes.c_void_p(ptr))
        dist.barrier(group=self.group)
        self.L.rib_peer_buffer_free(self.dev, ctypes.c_void_p(self.base[self.rank]))
        self.closed = True
