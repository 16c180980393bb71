"""Runs the reference's own Metal kernels on the CPU -- TEST INFRASTRUCTURE ONLY.

The reference keeps its hot-path kernels as MSL source strings that its Python
host code (agent-test/v2/kernels.py, agent-test/v2/attention.py) hands to
mx.fast.metal_kernel together with the launch grid.  MLX is not installed
here, so this module puts a small stand-in `mlx.core` into sys.modules, imports
the reference's kernels.py / attention.py from the reference checkout and
calls their public functions (qk_norm_rope, qk_norm_rope_prefill, attention,
gemv, add_rms, skinny_matmul) unchanged.  The stand-in records the exact
source, template constants, buffers and grid each call produces, compiles the
source as C++ against oracle/msl/shim.h (Metal built-ins emulated on the CPU,
see its header) into oracle/_ref/, and runs it.

So these outputs come from the reference's kernel code and launch geometry,
with three stand-ins: the C library's float math functions for Metal's fast
ones, and the summation orders of simd_sum and of the SIMD-group matrix
product (shim.h).  They pin the oracle (tests/golden/make_golden.py writes
them into the committed fixtures); nothing in the product path imports this.

Needs the reference checkout (REFERENCE_ROOT, default the checkout this build
reads) and g++; the GPU tests use only the committed fixtures.
"""
from __future__ import annotations

import ctypes
import hashlib
import importlib
import os
import re
import subprocess
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE.parent / "_ref"
SHIM = HERE / "shim.h"


def reference_root() -> Path:
    return Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))


def available() -> bool:
    return (reference_root() / "agent-test" / "v2" / "kernels.py").exists()


# ------------------------------------------------------------------ stand-in arrays
class Dtype:
    def __init__(self, name: str, np_dtype, ctype: str):
        self.name, self.np, self.ctype = name, np.dtype(np_dtype), ctype

    def __repr__(self):
        return f"mlx.{self.name}"


BF16 = Dtype("bfloat16", np.uint16, "bfloat16_t")
F32 = Dtype("float32", np.float32, "float")
I32 = Dtype("int32", np.int32, "int")


class Array:
    """What the reference's host code sees of an mlx array: shape, dtype, size
    (BF16 data carried as uint16 bit patterns)."""

    def __init__(self, data, dtype: Dtype):
        self.data = np.ascontiguousarray(data, dtype=dtype.np)
        self.dtype = dtype

    @property
    def shape(self):
        return tuple(self.data.shape)

    @property
    def size(self):
        return int(self.data.size)

    @property
    def ndim(self):
        return self.data.ndim

    def reshape(self, *shape):
        return Array(self.data.reshape(*shape), self.dtype)

    def __getitem__(self, idx):
        return Array(self.data[idx], self.dtype)


def bf16(u16) -> Array:
    return Array(u16, BF16)


def _array(values, dtype=None):
    dtype = dtype or I32
    return Array(np.asarray(values), dtype)


def _pad(x: Array, widths):
    return Array(np.pad(x.data, widths), x.dtype)


# ------------------------------------------------------------------ kernels
_INPUT_CTYPE = {"bfloat16": "bfloat16_t", "float32": "float", "int32": "int"}


class MetalKernel:
    """Stand-in for mx.fast.metal_kernel: compiles the MSL body against the
    shim on first use of each (template, dtype) combination and runs it."""

    def __init__(self, name, input_names, output_names, source, header="", **_):
        self.name, self.inputs, self.outputs = name, list(input_names), list(output_names)
        self.source, self.header = source, header
        self.calls = []  # (grid, threadgroup) of every launch, for the tests

    def _translate(self, src: str) -> str:
        src = src.replace("(threadgroup ", "(")          # casts to threadgroup pointers
        return re.sub(r"\bthreadgroup\s", "TG_STATIC ", src)  # threadgroup arrays

    def _tu(self, in_types, out_types, template) -> str:
        lines = ['#include "shim.h"', "namespace {", "struct Args {", "  void *buf[32];",
                 "  const int *shape[32];", "  uint3 tg, tpt, grid;", "};"]
        lines.append("void body(void *argp, int tid) {")
        lines.append("  Args &A = *static_cast<Args *>(argp);")
        for i, (n, t) in enumerate(zip(self.inputs, in_types)):
            lines.append(f"  const device {t} *{n} = static_cast<const {t} *>(A.buf[{i}]); (void){n};")
            if f"{n}_shape" in self.source:
                lines.append(f"  const constant int *{n}_shape = A.shape[{i}]; (void){n}_shape;")
        for j, (n, t) in enumerate(zip(self.outputs, out_types)):
            k = len(self.inputs) + j
            lines.append(f"  device {t} *{n} = static_cast<{t} *>(A.buf[{k}]); (void){n};")
        for k, v in template:
            lines.append(f"  constexpr int {k} = {int(v)}; (void){k};")
        lines += [
            "  const uint3 threadgroup_position_in_grid = A.tg;",
            "  const uint3 threads_per_threadgroup = A.tpt;",
            "  const uint3 thread_position_in_threadgroup = {uint(tid) % A.tpt.x, (uint(tid) / A.tpt.x) % A.tpt.y,"
            " uint(tid) / (A.tpt.x * A.tpt.y)};",
            "  const uint3 thread_position_in_grid = {A.tg.x * A.tpt.x + thread_position_in_threadgroup.x,"
            " A.tg.y * A.tpt.y + thread_position_in_threadgroup.y,"
            " A.tg.z * A.tpt.z + thread_position_in_threadgroup.z};",
            "  const uint simdgroup_index_in_threadgroup = uint(tid) / 32;",
            "  const uint thread_index_in_simdgroup = uint(tid) % 32;",
            "  (void)threadgroup_position_in_grid; (void)threads_per_threadgroup;",
            "  (void)thread_position_in_threadgroup; (void)thread_position_in_grid;",
            "  (void)simdgroup_index_in_threadgroup; (void)thread_index_in_simdgroup;",
            "  {",
            self._translate(self.header + "\n" + self.source),
            "  }",
            "}",
            "}  // namespace",
            'extern "C" void msl_run(void **bufs, const int **shapes, int gx, int gy, int gz, int tx, int ty,'
            " int tz) {",
            "  const int total = gx * gy * gz;",
            "#pragma omp parallel for schedule(dynamic)",
            "  for (int i = 0; i < total; ++i) {",
            "    Args a;",
            "    for (int b = 0; b < 32; ++b) { a.buf[b] = bufs[b]; a.shape[b] = shapes[b]; }",
            "    a.tg = {uint(i % gx), uint((i / gx) % gy), uint(i / (gx * gy))};",
            "    a.tpt = {uint(tx), uint(ty), uint(tz)};",
            "    a.grid = {uint(gx), uint(gy), uint(gz)};",
            "    msl::run_group(tx * ty * tz, body, &a);",
            "  }",
            "}",
        ]
        return "\n".join(lines) + "\n"

    def _compile(self, tu: str) -> ctypes.CDLL:
        OUT.mkdir(parents=True, exist_ok=True)
        h = hashlib.sha256((tu + SHIM.read_text()).encode()).hexdigest()[:16]
        so = OUT / f"msl_{self.name}_{h}.so"
        if not so.exists():
            cpp = OUT / f"msl_{self.name}_{h}.cpp"
            cpp.write_text(tu)
            tmp = so.with_suffix(f".{os.getpid()}.tmp")
            subprocess.run(["g++", "-O2", "-std=c++17", "-fopenmp", "-fPIC", "-shared", "-w",
                            "-I", str(HERE), "-o", str(tmp), str(cpp)], check=True)
            tmp.replace(so)
        lib = ctypes.CDLL(str(so))
        lib.msl_run.restype = None
        return lib

    def __call__(self, inputs, output_shapes, output_dtypes, grid, threadgroup, template=None,
                 init_value=None, verbose=False, **_):
        template = list(template or [])
        in_types = [_INPUT_CTYPE[a.dtype.name] for a in inputs]
        out_types = [_INPUT_CTYPE[d.name] for d in output_dtypes]
        lib = self._compile(self._tu(in_types, out_types, template))
        outs = [Array(np.full(s, 0 if init_value is None else init_value, dtype=d.np), d)
                for s, d in zip(output_shapes, output_dtypes)]
        bufs = (ctypes.c_void_p * 32)()
        shapes = (ctypes.c_void_p * 32)()
        keep = []
        for i, a in enumerate(list(inputs) + outs):
            bufs[i] = a.data.ctypes.data
            shp = np.ascontiguousarray(a.shape, dtype=np.int32)
            keep.append(shp)
            shapes[i] = shp.ctypes.data
        for g, t in zip(grid, threadgroup):
            if g % t:
                raise ValueError(f"{self.name}: grid {grid} is not a multiple of threadgroup {threadgroup}")
        gx, gy, gz = (g // t for g, t in zip(grid, threadgroup))
        self.calls.append((tuple(grid), tuple(threadgroup)))
        lib.msl_run(bufs, shapes, gx, gy, gz, *(int(t) for t in threadgroup))
        return outs


# ------------------------------------------------------------------ the reference modules
_MODULES: dict[str, types.ModuleType] = {}


def _stand_in_mlx() -> types.ModuleType:
    core = types.ModuleType("mlx.core")
    core.bfloat16, core.float32, core.int32 = BF16, F32, I32
    core.array = _array
    core.pad = _pad
    core.fast = types.SimpleNamespace(metal_kernel=MetalKernel)
    pkg = types.ModuleType("mlx")
    pkg.core = core
    return pkg


def reference(name: str) -> types.ModuleType:
    """The reference's agent-test/v2/<name>.py, imported with the stand-in
    mlx.core (module-level code only builds kernels and reads its tuning
    table)."""
    if name in _MODULES:
        return _MODULES[name]
    v2 = reference_root() / "agent-test" / "v2"
    if not available():
        raise FileNotFoundError(f"reference checkout not found under {v2}")
    saved = {k: sys.modules.get(k) for k in ("mlx", "mlx.core", name)}
    pkg = _stand_in_mlx()
    sys.modules["mlx"], sys.modules["mlx.core"] = pkg, pkg.core
    sys.path.insert(0, str(v2))
    try:
        sys.modules.pop(name, None)
        mod = importlib.import_module(name)
    finally:
        sys.path.remove(str(v2))
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    _MODULES[name] = mod
    return mod


# ------------------------------------------------------------------ convenience wrappers
def qk_norm_rope(qkv_u16, qw_u16, kw_u16, pos: int, nq=16, nkv=8, base=1e6):
    """kernels.py:157 qk_norm_rope -> (q [1,nq,1,128], kv [2,nkv,1,128]) u16."""
    k = reference("kernels")
    q, kv = k.qk_norm_rope(bf16(qkv_u16), bf16(qw_u16), bf16(kw_u16), _array([pos], I32), nq, nkv, base)
    return q.data, kv.data


def qk_norm_rope_prefill(qkv_u16, qw_u16, kw_u16, offset: int, nq=16, nkv=8, base=1e6, Lp=None):
    """kernels.py:215 qk_norm_rope_prefill -> (Q [nq,Lp,128], KV [2,nkv,L,128]) u16."""
    k = reference("kernels")
    L = np.asarray(qkv_u16).shape[0]
    Lp = Lp or (L + 31) // 32 * 32
    q, kv = k.qk_norm_rope_prefill(bf16(qkv_u16), bf16(qw_u16), bf16(kw_u16), offset, nq, nkv, base, Lp)
    return q.data, kv.data


def attention(Q_u16, K_u16, V_u16, qL: int, kL: int, scale: float, **kw):
    """attention.py:177 attention(Q [H,qLp,128], K/V [1,nkv,cap,128]) -> O [qL, H*128] u16."""
    a = reference("attention")
    return a.attention(bf16(Q_u16), bf16(K_u16), bf16(V_u16), qL, kL, scale, **kw).data


def gemv(W_u16, x_u16, nw_u16=None, res_u16=None, swiglu=False, out_float=False):
    """kernels.py:103 gemv -> y (u16, or float32 with out_float)."""
    k = reference("kernels")
    y = k.gemv(bf16(W_u16), bf16(x_u16), nw=None if nw_u16 is None else bf16(nw_u16),
               res=None if res_u16 is None else bf16(res_u16), swiglu=swiglu, out_float=out_float)
    return y.data


def add_rms(a_u16, b_u16, w_u16):
    """kernels.py:262 add_rms -> (residual, normalized) u16."""
    k = reference("kernels")
    r, n = k.add_rms(bf16(a_u16), bf16(b_u16), bf16(w_u16))
    return r.data, n.data


def skinny_matmul(x_u16, W_u16):
    """kernels.py:323 skinny_matmul (8 < M <= 32) -> Y [M, N] u16."""
    k = reference("kernels")
    return k.skinny_matmul(bf16(x_u16), bf16(W_u16)).data
