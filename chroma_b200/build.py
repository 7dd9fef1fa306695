"""Build step: compile the sm_100a kernels and the C ABI into ``chroma_b200/libchroma_b200.so`` (in-tree).

nvcc cross-compiles without a GPU. The library links the CUDA runtime statically so it loads wherever the driver
is present.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
SOURCES = [PACKAGE / "csrc" / "runtime.cu", PACKAGE / "csrc" / "graph.cu"]
DEPENDS = sorted((PACKAGE / "csrc").glob("*.cu*")) + [ROOT / "include" / "chroma_b200.h"]
TARGET = PACKAGE / "libchroma_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    found = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists() and shutil.which(found) is None:
        raise RuntimeError("nvcc not found; set NVCC or add the CUDA toolkit to PATH")
    return found


def command(target: Path = TARGET) -> list[str]:
    return [nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC", "-shared", "--cudart=static",
            "-I", str(ROOT / "include"), *map(str, SOURCES), "-o", str(target)]


def stale() -> bool:
    if not TARGET.exists():
        return True
    built = TARGET.stat().st_mtime
    return any(p.stat().st_mtime > built for p in DEPENDS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if force or stale():
        tmp = TARGET.with_suffix(".so.tmp")
        res = subprocess.run(command(tmp), capture_output=True, text=True)
        if res.returncode:
            raise RuntimeError(f"nvcc failed:\n{res.stderr}")
        if verbose and res.stderr:
            print(res.stderr, file=sys.stderr)
        os.replace(tmp, TARGET)
    return TARGET


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
