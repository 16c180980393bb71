"""Argument checks shared by the host-side wrappers (raise before any launch)."""
from __future__ import annotations

import torch

HEAD_DIM = 128


def require_bf16_cuda(name: str, t) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"{name} must be a torch.Tensor")
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bfloat16, got {t.dtype}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def require_same_device(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts[1:]:
        if t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


def stream_handle(device: torch.device) -> int:
    """cudaStream_t of torch's current stream on `device`."""
    return torch.cuda.current_stream(device).cuda_stream


def as_int(x, name: str) -> int:
    """Position/offset given as int or a 1-element host tensor.  (A CUDA
    tensor goes to the device-position kernels instead: device_position.)"""
    if isinstance(x, torch.Tensor):
        if x.numel() != 1:
            raise ValueError(f"{name} must hold one element")
        if x.is_cuda:
            raise ValueError(f"{name}: a CUDA tensor is read on the device, not here")
        return int(x.reshape(-1)[0].item())
    return int(x)


def device_position(x, name: str, device) -> torch.Tensor | None:
    """The reference passes positions as mx.array([pos], int32)
    (agent-test/v2/engine.py:148).  For a 1-element CUDA tensor on `device`,
    returns it as a contiguous int32 tensor for the kernels to read there (no
    host synchronisation); None for an int or a host tensor."""
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        return None
    if x.numel() != 1:
        raise ValueError(f"{name} must hold one element")
    if x.device != torch.device(device):
        raise ValueError(f"{name} is on {x.device}, the data on {device}")
    return x.reshape(1).to(torch.int32).contiguous()
