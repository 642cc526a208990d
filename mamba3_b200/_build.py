"""Build the in-tree CUDA library ``mamba3_b200/_lib/libmamba3_b200.so`` for sm_100a.

The library is a plain C-ABI shared object (no torch symbols); it is loaded with ctypes by
``mamba3_b200._ext``. nvcc cross-compiles it without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libmamba3_b200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]
UNITS = ["capi.cu", "step.cu", "scan_simt.cu", "scan_umma.cu", "noalloc.cu", "norm.cu", "ssd_train.cu", "gemv.cu"]


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h")))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    return any(src.stat().st_mtime > built for src in sources())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and not needs_build():
        return LIB
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    LIB_DIR.mkdir(exist_ok=True)
    objs = []
    procs = []
    for unit in UNITS:
        obj = LIB_DIR / (Path(unit).stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, *(extra or []), "-I", str(ROOT / "include"), "-I", str(CSRC), "-c",
               str(CSRC / unit), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((unit, subprocess.Popen(cmd)))
        objs.append(obj)
    failed = [unit for unit, proc in procs if proc.wait() != 0]
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static",
            *map(str, objs), "-o", str(tmp)]
    subprocess.run(link, check=True)
    os.replace(tmp, LIB)
    for obj in objs:
        obj.unlink()
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, extra=["-Xptxas", "-v"] if "--ptxas" in sys.argv else None)
