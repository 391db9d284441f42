"""Build liborigami_b200.so (the C-ABI library with the sm_100a kernels) in-tree.

nvcc cross-compiles for sm_100a without a GPU, so this runs on any machine with the
CUDA 12.9 toolkit. Every source is compiled to its own object under `_build/` (in
parallel, and only when it or a header changed), then the objects are linked. The library
lands next to this file and travels with the tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OBJ = HERE / "_build"
LIB = HERE / "liborigami_b200.so"
SOURCES = ["abi.cu", "quant.cu", "attention.cu", "host_codec.cpp"]
HEADERS = [CSRC / p for p in sorted(os.listdir(CSRC)) if p.endswith((".cuh", ".h"))] + [
    HERE.parent / "include" / "origami_b200.h"]

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the origami_b200 CUDA library cannot be built")
    return cand


def _obj(src: str) -> Path:
    return OBJ / (src + ".o")


def _deps(src: str) -> list[Path]:
    """The source and the headers it includes (from the compiler's dependency file)."""
    d = OBJ / (src + ".d")
    if not d.exists():
        return [CSRC / src, *HEADERS]
    text = d.read_text().replace("\\\n", " ")
    names = text.split(":", 1)[1].split() if ":" in text else []
    return [CSRC / src] + [CSRC / n for n in names if not n.startswith("/usr")]


def _obj_stale(src: str) -> bool:
    o = _obj(src)
    if not o.exists():
        return True
    t = o.stat().st_mtime
    return any(not p.exists() or p.stat().st_mtime > t for p in _deps(src))


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [*(CSRC / s for s in SOURCES), *HEADERS])


def _compile(src: str, verbose: bool) -> None:
    cmd = [nvcc(), *NVCC_FLAGS, "-MD", "-MF", str(OBJ / (src + ".d")), "-c", str(CSRC / src), "-o", str(_obj(src))]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True, cwd=CSRC)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    OBJ.mkdir(exist_ok=True)
    todo = [s for s in SOURCES if force or _obj_stale(s)]
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        list(ex.map(lambda s: _compile(s, verbose), todo))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(tmp),
                    *[str(_obj(s)) for s in SOURCES], "-lz"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
