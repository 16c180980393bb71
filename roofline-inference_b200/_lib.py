"""Loader of the C-ABI library librib_attention.so (CUDA kernels for sm_100a).

The library is built in-tree from csrc/ with nvcc.  `load()` rebuilds it when
the sources changed (content hash, not mtimes, so a copied tree is recognised
correctly) and then binds the entry points declared in
include/rib_attention.h with ctypes.  There is no fallback: if the library
cannot be built or loaded, every call raises.
"""
from __future__ import annotations

import ctypes
import fcntl
import hashlib
import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
HEADER = REPO_DIR / "include" / "rib_attention.h"
LIB_PATH = PKG_DIR / "librib_attention.so"
STAMP = PKG_DIR / "librib_attention.so.srchash"
MAIN_SOURCE = CSRC / "rib_attention.cu"

EXPORTS = CSRC / "exports.map"
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xlinker", f"--version-script={EXPORTS}",
]

# status codes (include/rib_attention.h)
RIB_OK, RIB_EINVAL, RIB_ECAPACITY, RIB_EALIGN, RIB_ECUDA, RIB_ETIMEOUT = range(6)

_lib: ctypes.CDLL | None = None


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [HEADER, EXPORTS]


def source_hash() -> str:
    h = hashlib.sha256()
    for p in _sources():
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(f for f in NVCC_FLAGS if not f.startswith("--version-script")).encode())
    return h.hexdigest()


def is_current() -> bool:
    return LIB_PATH.exists() and STAMP.exists() and STAMP.read_text().strip() == source_hash()


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: cannot build librib_attention.so")


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles csrc/rib_attention.cu for sm_100a into librib_attention.so.

    Serialised with a file lock so that several ranks importing the package at
    once build it only once."""
    if not force and is_current():
        return LIB_PATH
    lock_path = PKG_DIR / ".librib_attention.lock"
    with open(lock_path, "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            if not force and is_current():
                return LIB_PATH
            tmp = LIB_PATH.with_name(f"{LIB_PATH.name}.{os.getpid()}.tmp")
            cmd = [_nvcc(), *NVCC_FLAGS, "-o", str(tmp), str(MAIN_SOURCE)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
            if verbose:
                print(res.stdout + res.stderr)
            tmp.replace(LIB_PATH)
            STAMP.write_text(source_hash() + "\n")
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)
    return LIB_PATH


def _bind(L: ctypes.CDLL) -> None:
    vp, i, d, f, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_double, ctypes.c_float, ctypes.c_size_t
    sig = {
        "rib_version": ([], i),
        "rib_status_string": ([i], ctypes.c_char_p),
        "rib_last_error_string": ([], ctypes.c_char_p),
        "rib_take_device_status": ([ctypes.POINTER(ctypes.c_int)], i),
        "rib_set_wait_limit_ns": ([ctypes.c_ulonglong], i),
        "rib_get_wait_limit_ns": ([ctypes.POINTER(ctypes.c_ulonglong)], i),
        "rib_qk_norm_rope": ([vp, vp, vp, i, i, i, d, vp, vp, vp], i),
        "rib_qk_norm_rope_prefill": ([vp, i, vp, vp, i, i, i, d, i, vp, vp, vp], i),
        "rib_qk_norm_rope_append": ([vp, i, vp, vp, i, i, i, d, i, vp, vp, i, vp], i),
        "rib_decode_workspace_bytes": ([i, i, i], sz),
        "rib_decode_kernel_choice": ([i, i, i], i),
        "rib_decode_workspace_init": ([vp, sz, vp], i),
        "rib_decode_attention": ([vp, vp, i, i, i, i, f, vp, vp, sz, vp], i),
        "rib_decode_attention_noalloc": ([vp, vp, i, i, i, i, f, vp, vp], i),
        "rib_decode_attention_batched": ([vp, vp, vp, i, i, i, i, i, f, vp, vp, sz, vp], i),
        "rib_prefill_workspace_bytes": ([i, i], sz),
        "rib_prefill_attention": ([vp, vp, vp, i, i, i, i, i, i, f, vp, vp, sz, vp], i),
        "rib_qk_norm_rope_append_dev": ([vp, i, vp, vp, vp, i, i, d, i, vp, vp, i, vp], i),
        "rib_qk_norm_rope_prefill_dev": ([vp, i, vp, vp, vp, i, i, d, i, vp, vp, vp], i),
        "rib_gemv": ([vp, i, i, vp, vp, vp, i, i, vp, vp], i),
        "rib_add_rms": ([vp, vp, vp, i, i, vp, vp, vp], i),
        "rib_rms_norm": ([vp, vp, i, i, vp, vp], i),
        "rib_swiglu": ([vp, i, i, vp, vp], i),
        "rib_embed": ([vp, i, i, vp, i, vp, vp], i),
        "rib_argmax_workspace_bytes": ([], sz),
        "rib_argmax_f32": ([vp, i, vp, vp, vp], i),
        "rib_qwen3_step_workspace_bytes": ([vp, i], sz),
        "rib_qwen3_step_workspace_init": ([vp, sz, vp], i),
        "rib_qwen3_decode_step": ([vp, vp, i, vp, vp, vp, vp, vp, sz, vp], i),
        "rib_decode_attention_ragged": ([vp, vp, vp, vp, i, i, i, i, f, vp, vp, sz, vp], i),
        "rib_qk_norm_rope_append_batched": ([vp, vp, vp, vp, vp, vp, i, i, i, d, vp, vp], i),
        "rib_argmax_rows_f32": ([vp, i, i, vp, vp], i),
        "rib_decode_attention_qkv": ([vp, vp, vp, d, vp, vp, i, i, i, i, i, f, vp, vp, sz, vp], i),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res


def load() -> ctypes.CDLL:
    """Builds if needed, loads and binds the library (once per process)."""
    global _lib
    if _lib is None:
        path = build()
        L = ctypes.CDLL(str(path))
        _bind(L)
        _lib = L
    return _lib


def check(status: int, what: str) -> None:
    """Raises like the reference: ValueError for shape/capacity/alignment
    problems (agent-test/v2/engine.py:45-46, 69-70), RuntimeError otherwise."""
    if status == RIB_OK:
        return
    msg = load().rib_status_string(status).decode()
    if status in (RIB_EINVAL, RIB_ECAPACITY, RIB_EALIGN):
        raise ValueError(f"{what}: {msg}")
    detail = load().rib_last_error_string().decode()
    raise RuntimeError(f"{what}: {msg} (status {status}): {detail}")


def take_device_status() -> int:
    """Reads and clears the device status word (synchronises the device)."""
    v = ctypes.c_int(0)
    check(load().rib_take_device_status(ctypes.byref(v)), "rib_take_device_status")
    return v.value


DEFAULT_WAIT_LIMIT_NS = 2_000_000_000


def set_wait_limit_ns(ns: int) -> None:
    """Sets the wall-clock limit of every device-side wait on the current
    device (1 ms .. 60 s; the default is 2 s).  Takes effect for kernels
    launched afterwards; call it while none of this library's kernels runs."""
    check(load().rib_set_wait_limit_ns(int(ns)), "rib_set_wait_limit_ns")


def wait_limit_ns() -> int:
    v = ctypes.c_ulonglong(0)
    check(load().rib_get_wait_limit_ns(ctypes.byref(v)), "rib_get_wait_limit_ns")
    return v.value
