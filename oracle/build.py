"""Build recipe for the CPU oracle (test infrastructure only).

Compiles oracle.c into oracle/liboracle.so with the system gcc (OpenMP,
AVX2/FMA).  The compiler is taken from PATH as `gcc`, not from $CC, because
some images point $CC at a toolchain without libgomp.
"""
from __future__ import annotations

import hashlib
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "oracle.c"
LIB = HERE / "liboracle.so"
STAMP = HERE / "liboracle.so.srchash"
FLAGS = ["-O3", "-mavx2", "-mfma", "-fopenmp", "-fPIC", "-std=c11", "-Wall", "-Wextra",
         "-Wno-unused-parameter", "-shared"]


def source_hash() -> str:
    h = hashlib.sha256(SRC.read_bytes())
    h.update(" ".join(FLAGS).encode())
    return h.hexdigest()


def is_current() -> bool:
    return LIB.exists() and STAMP.exists() and STAMP.read_text().strip() == source_hash()


def build(force: bool = False) -> Path:
    if not force and is_current():
        return LIB
    cc = shutil.which("gcc") or "gcc"
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([cc, *FLAGS, "-o", str(tmp), str(SRC), "-lm"], check=True)
    tmp.replace(LIB)
    STAMP.write_text(source_hash() + "\n")
    return LIB


if __name__ == "__main__":
    print(build(force=True))
