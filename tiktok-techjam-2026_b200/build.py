"""Build libtjb200.so (the sm_100a kernels and their C ABI) in-tree.

The library is one nvcc translation unit (``csrc/tjb200.cu``) compiled for
``sm_100a`` only and written next to the Python package
(``tjkernels/libtjb200.so``), where ``tjkernels._lib`` loads it.  The CUDA
runtime is linked statically; the driver's tensor-map encoder is resolved at
run time, so the library needs no libcuda at link time.

    python tiktok-techjam-2026_b200/build.py
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
TARGET = HERE / "tjkernels" / "libtjb200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3", "-shared",
    "-cudart", "static",
]


def find_nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libtjb200")


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [HERE.parent / "include" / "tjb200.h"]


def up_to_date() -> bool:
    if not TARGET.exists():
        return False
    t = TARGET.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return TARGET
    cmd = [find_nvcc(), *NVCC_FLAGS]
    if verbose:
        cmd.append("-Xptxas=-v")
    tmp = TARGET.with_suffix(".so.tmp")
    cmd += ["-o", str(tmp), str(CSRC / "tjb200.cu")]
    proc = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stderr[-4000:]}")
    if verbose:
        print(proc.stderr)
    os.replace(tmp, TARGET)
    return TARGET


if __name__ == "__main__":
    out = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(out)
