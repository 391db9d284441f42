"""Drop-in for the reference's ``lossless/native_cpu.py`` layout entry points.

Keeps the reference names, signatures and error messages
(lossless/native_cpu.py:30-196). Where the reference's packers are stubs that raise
("paper path only", native_cpu.py:137-161), these run the canonical pack / unpack on
the GPU through liborigami_b200 and return tensors on the caller's device: CPU symbols
in, CPU chunks out, as the worker's host codec expects (worker.py:2010-2016).
"""
from __future__ import annotations

from typing import Iterable, Sequence

import torch

_REQUIRED_AXES = ("token", "head", "head_dim")
_AXIS_ALIASES = {
    "token": "token",
    "tokens": "token",
    "seq": "token",
    "sequence": "token",
    "head": "head",
    "heads": "head",
    "kv_head": "head",
    "kv_heads": "head",
    "head_dim": "head_dim",
    "channel": "head_dim",
    "channels": "head_dim",
    "dim": "head_dim",
    "layer": "layer",
    "layers": "layer",
}
STORAGE_LAYOUT = ["layer", "head", "head_dim", "token"]


def normalize_symbol_layout(layout: Sequence[str]) -> list[str]:
    """Canonical axis names of a symbol layout (native_cpu.py:81-100)."""
    names: list[str] = []
    for axis in layout:
        key = str(axis).lower()
        if key not in _AXIS_ALIASES:
            raise ValueError(f"Unsupported Origami symbol layout axis {axis!r}")
        names.append(_AXIS_ALIASES[key])
    if len(set(names)) != len(names):
        raise ValueError(f"Origami symbol layout axes must be unique: {layout!r}")
    if any(req not in names for req in _REQUIRED_AXES):
        raise ValueError("Origami symbol layout must include token, head, and head_dim axes")
    extra = set(names) - set(_REQUIRED_AXES) - {"layer"}
    if extra:
        raise ValueError(f"Unsupported Origami symbol layout axes: {sorted(extra)}")
    if len(names) not in {3, 4}:
        raise ValueError("Origami symbol layout supports rank 3 or rank 4")
    return names


def canonical_axis_sizes(
    source_shape: Sequence[int],
    source_layout: Sequence[str],
) -> tuple[int, int, int, list[int], list[str]]:
    """(token_count, num_heads, head_dim, shape, layout) (native_cpu.py:103-120)."""
    shape = [int(dim) for dim in source_shape]
    layout = normalize_symbol_layout(source_layout)
    if len(shape) != len(layout):
        raise ValueError("origami_symbol_shape rank must match origami_symbol_layout")
    if len(shape) not in {3, 4}:
        raise ValueError("origami_symbol_shape supports rank 3 or rank 4")
    if any(dim <= 0 for dim in shape):
        raise ValueError("origami_symbol_shape dimensions must be positive")
    if "layer" in layout and shape[layout.index("layer")] != 1:
        raise ValueError("per-layer Origami worker requires layer axis size 1")
    return (shape[layout.index("token")], shape[layout.index("head")],
            shape[layout.index("head_dim")], shape, layout)


def axis_positions(source_layout: Sequence[str]) -> list[int]:
    """[token, head, head_dim, layer or -1] (native_cpu.py:123-130)."""
    layout = normalize_symbol_layout(source_layout)
    return [
        layout.index("token"),
        layout.index("head"),
        layout.index("head_dim"),
        layout.index("layer") if "layer" in layout else -1,
    ]


def pack_canonical_storage_chunks(
    symbols: torch.Tensor,
    bits: int,
    source_shape: Sequence[int],
    source_layout: Sequence[str],
    chunk_specs: torch.Tensor | Iterable[Iterable[int]],
) -> list[torch.Tensor]:
    """Pack uint8 symbols into canonical chunks (one tensor per spec row)."""
    from origami_b200.lossless import native_gpu

    return native_gpu.pack_canonical_storage_chunks(symbols, bits, source_shape, source_layout, chunk_specs)


def unpack_canonical_storage_chunks(
    chunks: Iterable[torch.Tensor],
    bits: int,
    source_shape: Sequence[int],
    source_layout: Sequence[str],
    chunk_specs: torch.Tensor | Iterable[Iterable[int]],
) -> torch.Tensor:
    """Inverse of pack_canonical_storage_chunks; returns a flat uint8 tensor in source
    layout on the chunks' device."""
    from origami_b200.lossless import native_gpu

    chunks = list(chunks)
    home = chunks[0].device if chunks else torch.device("cpu")
    out = native_gpu.unpack_canonical_storage_chunks(
        chunks, bits, source_shape, source_layout, chunk_specs,
        device=home if home.type == "cuda" else None,
    )
    return out if home.type == "cuda" else out.cpu()


def pack_head_channel_chunks(
    symbols: torch.Tensor,
    bits: int,
    token_count: int,
    num_heads: int,
    head_dim: int,
    chunk_specs: torch.Tensor | Iterable[Iterable[int]],
) -> list[torch.Tensor]:
    return pack_canonical_storage_chunks(
        symbols, bits, [int(token_count), int(num_heads), int(head_dim)],
        ["token", "head", "head_dim"], chunk_specs)


def unpack_head_channel_chunks(
    chunks: Iterable[torch.Tensor],
    bits: int,
    token_count: int,
    num_heads: int,
    head_dim: int,
    chunk_specs: torch.Tensor | Iterable[Iterable[int]],
) -> torch.Tensor:
    return unpack_canonical_storage_chunks(
        chunks, bits, [int(token_count), int(num_heads), int(head_dim)],
        ["token", "head", "head_dim"], chunk_specs)


def cpu_isa() -> str:
    return "cuda"
