"""Plane split of 16-bit KV elements and the per-layer chunk table of the plane format.

A bf16/fp16 element x is split into planes, plane p holding (x >> shift[p]) &
((1 << bits[p]) - 1). Every plane of K and of V is a [token, head, head_dim] symbol
tensor stored with Origami's canonical head > channel > token chunk layout and dense
LSB-first bitpacking (the format of csrc/origami/bitpack_layout_cuda.cu:70-128), chunked
by the head/channel planner with the connector's chunk sizes (worker.py:1992-2001). The
chunks of one layer are ordered K plane 0, K plane 1, ..., V plane 0, ...; each
component uses the same spec list.

Presets:
  byte      : high byte (sign + exponent bits) and low byte, 8 bits each
  bf16_bits : exponent (8), sign (1), mantissa (7)
  fp16_bits : sign + exponent (6), mantissa high (2), mantissa low (8)
  raw       : no split; the reference's raw-bytes layout (gathered blocks, 1 MiB chunks)

The split is arithmetic of this library (the reference has none); its invariant is
merge(split(x)) == x for every 16-bit pattern.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import numpy as np
import torch

from origami_b200.lossless.chunking import plan_head_channel_chunks
from origami_b200.metadata import ChunkLayout

FORMAT_NAME = "origami_planes_v1"


@dataclass(frozen=True)
class PlaneSpec:
    name: str
    shifts: tuple[int, ...]
    bits: tuple[int, ...]

    def __post_init__(self) -> None:
        seen = 0
        if not 1 <= len(self.shifts) <= 8 or len(self.shifts) != len(self.bits):
            raise ValueError("a plane spec needs 1..8 planes with one shift and one width each")
        for s, b in zip(self.shifts, self.bits):
            if not 1 <= b <= 8 or s < 0 or s + b > 16:
                raise ValueError(f"plane (shift={s}, bits={b}) does not fit a 16-bit element")
            m = ((1 << b) - 1) << s
            if seen & m:
                raise ValueError("planes overlap")
            seen |= m
        if seen != 0xFFFF:
            raise ValueError("planes must cover all 16 bits")

    @property
    def num_planes(self) -> int:
        return len(self.bits)

    def split(self, x: np.ndarray) -> list[np.ndarray]:
        """Host-side reference of the split (used to describe the format in tests)."""
        x = np.asarray(x, dtype=np.uint16)
        return [((x >> s) & ((1 << b) - 1)).astype(np.uint8) for s, b in zip(self.shifts, self.bits)]


BYTE_PLANES = PlaneSpec("byte", (8, 0), (8, 8))
BF16_BIT_PLANES = PlaneSpec("bf16_bits", (7, 15, 0), (8, 1, 7))
FP16_BIT_PLANES = PlaneSpec("fp16_bits", (10, 8, 0), (6, 2, 8))


def plane_spec(policy: str, dtype: torch.dtype | None = None) -> PlaneSpec:
    """Plane preset for a layout policy: 'byte', 'bit' (dtype-dependent) or a preset name."""
    name = str(policy).lower()
    if name in {"byte", "byte_planes", "head_first"}:
        return BYTE_PLANES
    if name in {"bit", "bit_planes"}:
        if dtype == torch.float16:
            return FP16_BIT_PLANES
        return BF16_BIT_PLANES
    if name == "bf16_bits":
        return BF16_BIT_PLANES
    if name == "fp16_bits":
        return FP16_BIT_PLANES
    raise ValueError(f"unknown plane policy {policy!r}")


@dataclass
class LayerFormat:
    """Chunk table of one layer: T tokens x H heads x D channels, K and V, P planes."""

    num_tokens: int
    num_heads: int
    head_dim: int
    planes: PlaneSpec = BYTE_PLANES
    chunk_min_bytes: int = 1 << 20
    chunk_target_bytes: int = 1 << 20
    chunk_max_bytes: int = 1 << 20
    layer_index: int = 0
    specs: np.ndarray = field(init=False)
    offsets: np.ndarray = field(init=False)
    _device_tables: dict = field(init=False, default_factory=dict, repr=False)

    def __post_init__(self) -> None:
        if self.num_tokens <= 0 or self.num_heads <= 0 or self.head_dim <= 0:
            raise ValueError("layer format dimensions must be positive")
        plan = plan_head_channel_chunks(
            layer_index=self.layer_index, num_heads=self.num_heads, head_dim=self.head_dim,
            token_count=self.num_tokens, bytes_per_symbol=1, min_bytes=self.chunk_min_bytes,
            target_bytes=self.chunk_target_bytes, max_bytes=self.chunk_max_bytes)
        self.specs = np.asarray([c.layout.spec() for c in plan], dtype=np.int64).reshape(-1, 6)
        n = (self.specs[:, 1] - self.specs[:, 0]) * (self.specs[:, 3] - self.specs[:, 2]) * (
            self.specs[:, 5] - self.specs[:, 4])
        sizes = []
        for _kv in range(2):
            for b in self.planes.bits:
                sizes.append((n * b + 7) // 8)
        sizes = np.concatenate(sizes).astype(np.int64)
        self.offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)

    @property
    def num_specs(self) -> int:
        return int(self.specs.shape[0])

    @property
    def num_chunks(self) -> int:
        return 2 * self.planes.num_planes * self.num_specs

    @property
    def packed_bytes(self) -> int:
        return int(self.offsets[-1])

    @property
    def kv_bytes(self) -> int:
        """Bytes of the K and V elements this format covers (2 bytes per element)."""
        return 2 * self.num_tokens * self.num_heads * self.head_dim * 2

    def chunk_bits(self) -> list[int]:
        out = []
        for _kv in range(2):
            for b in self.planes.bits:
                out.extend([int(b)] * self.num_specs)
        return out

    def device_tables(self, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
        """(specs, offsets) on `device`, uploaded once and cached."""
        key = str(device)
        if key not in self._device_tables:
            from origami_b200.lossless.native_gpu import upload_i64

            self._device_tables[key] = (upload_i64(self.specs, device), upload_i64(self.offsets, device))
        return self._device_tables[key]

    def chunk_views(self, packed: torch.Tensor) -> list[torch.Tensor]:
        return [packed[int(a):int(b)] for a, b in zip(self.offsets[:-1], self.offsets[1:])]

    def chunk_layouts(self) -> list[ChunkLayout]:
        """ChunkLayout of every chunk k = q * S + s (metadata.py:22-31): spec s of the
        planner, unpacked_bytes = the chunk's packed byte count (what the codec decodes)."""
        out = []
        for k in range(self.num_chunks):
            h0, h1, c0, c1, t0, t1 = (int(v) for v in self.specs[k % self.num_specs])
            out.append(ChunkLayout(self.layer_index, h0, h1, c0, c1, t0, t1,
                                   int(self.offsets[k + 1] - self.offsets[k])))
        return out

    def alloc_packed(self, device: torch.device | str, *, pin: bool = False) -> torch.Tensor:
        """A packed buffer whose allocation extends to a multiple of 16 bytes."""
        n = (self.packed_bytes + 15) // 16 * 16
        if pin:
            return torch.empty((n,), dtype=torch.uint8, pin_memory=True)[: self.packed_bytes]
        return torch.empty((n,), dtype=torch.uint8, device=device)[: self.packed_bytes]

    def metadata(self, dtype: torch.dtype | None = None) -> dict[str, Any]:
        """Native-layout metadata of an artifact layer (worker.py:2026-2039 style)."""
        comps = []
        for kv, kv_name in enumerate(("key", "value")):
            for p, (s, b) in enumerate(zip(self.planes.shifts, self.planes.bits)):
                q = kv * self.planes.num_planes + p
                comps.append({
                    "name": f"{kv_name}_plane{p}",
                    "kind": "quant",
                    "shift": int(s),
                    "bits": int(b),
                    "source_shape": [self.num_tokens, self.num_heads, self.head_dim],
                    "source_layout": ["token", "head", "head_dim"],
                    "chunk_start": q * self.num_specs,
                    "chunk_count": self.num_specs,
                })
        return {
            "version": 3,
            "format": FORMAT_NAME,
            "dtype": str(dtype).replace("torch.", "") if dtype is not None else None,
            "planes": self.planes.name,
            "storage_layout": ["layer", "head", "head_dim", "token"],
            "token_count": self.num_tokens,
            "num_heads": self.num_heads,
            "head_dim": self.head_dim,
            "chunk_specs": self.specs.tolist(),
            "components": comps,
        }
