"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on CPU."""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def rib():
    return importlib.import_module("roofline-inference_b200")


@pytest.fixture(scope="session")
def wl():
    return importlib.import_module("roofline-inference_b200.workloads")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    return o


@pytest.fixture(scope="session")
def ref_np():
    from oracle import reference_np as r
    return r


def load_golden(name: str):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def u16(t: torch.Tensor) -> np.ndarray:
    """BF16 torch tensor -> uint16 bit patterns (numpy, on the host)."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_u16(a: np.ndarray, device="cpu") -> torch.Tensor:
    """uint16 bit patterns -> BF16 torch tensor."""
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)


def bf16f(a) -> np.ndarray:
    """uint16 bit patterns or BF16 tensor -> float32 numpy."""
    if isinstance(a, torch.Tensor):
        return a.detach().float().cpu().numpy()
    return (np.asarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def parity_errors(out, exact) -> dict:
    """max/mean absolute error of `out` against FP32/FP64 `exact`, plus the
    error of simply rounding `exact` to BF16 (the floor any BF16 output has)."""
    from oracle.reference_np import round_bf16
    o = bf16f(out).astype(np.float64)
    e = np.asarray(exact, dtype=np.float64)
    floor = np.abs(round_bf16(e.astype(np.float32)).astype(np.float64) - e)
    d = np.abs(o - e)
    return {"max": float(d.max()), "mean": float(d.mean()), "floor_max": float(floor.max())}
