"""Build liborigami_b200.so (the C-ABI library with the sm_100a kernels) in-tree.

nvcc cross-compiles for sm_100a without a GPU, so this runs on any machine with the
CUDA 12.9 toolkit. The library lands next to this file and travels with the tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "liborigami_b200.so"
SOURCES = ["abi.cu", "quant.cu", "attention.cu", "host_codec.cpp"]
# every kernel header and source, plus the public header
DEPS = sorted(p.name for p in CSRC.iterdir() if p.suffix in (".cu", ".cuh", ".h", ".cpp")) + ["../../include/origami_b200.h"]

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-shared",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the origami_b200 CUDA library cannot be built")
    return cand


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any((CSRC / d).stat().st_mtime > t for d in DEPS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(tmp), *[str(CSRC / s) for s in SOURCES], "-lz"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
