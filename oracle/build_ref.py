"""TEST INFRASTRUCTURE ONLY: compile the reference's CUDA bitpack extension.

The reference ships its layout unpack only as a CUDA/ATen extension
(csrc/origami/bitpack_layout_cuda.{cpp,cu}, built by lossless/native_gpu.py:35-49 with
torch.utils.cpp_extension). This script builds those two files, where they lie in the
reference checkout, for sm_100a into oracle/_ref/ so the GPU tests can run the
reference kernel itself as a parity pin. Nothing is copied into this repository; the
built module stays out of git (oracle/_ref/ is ignored) and travels to the GPU box.

Usage: python oracle/build_ref.py [reference_root]
The checkout is the argument, else $ORIGAMI_REFERENCE_ROOT; without either nothing is built.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
MODULE = "origami_ref_bitpack"


def reference_root() -> str | None:
    """The reference checkout named by $ORIGAMI_REFERENCE_ROOT, or None."""
    return os.environ.get("ORIGAMI_REFERENCE_ROOT") or None


def build(reference_root: str | None = None) -> Path | None:
    reference_root = reference_root or globals()["reference_root"]()
    if not reference_root:
        return None
    src = Path(reference_root) / "csrc" / "origami"
    sources = [src / "bitpack_layout_cuda.cpp", src / "bitpack_layout_cuda.cu"]
    if not all(p.exists() for p in sources):
        return None
    OUT.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load

    load(
        name=MODULE,
        sources=[str(p) for p in sources],
        extra_cflags=["-O3"],
        extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"],
        build_directory=str(OUT),
        verbose=False,
    )
    built = OUT / f"{MODULE}.so"
    return built if built.exists() else None


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else reference_root()
    path = build(root)
    print(path if path else "reference sources not found; oracle/_ref not built")
