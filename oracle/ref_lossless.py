"""TEST INFRASTRUCTURE ONLY: the reference connector's CPU lossless restore of one layer
in its raw-bytes layout, restated step for step with the same library calls, so that
bench.py can time it on the GPU box's host cores (where the reference checkout is not
available) as a CPU baseline. Nothing in the product imports this module.

Reference steps (paths inside vllm/distributed/kv_transfer/kv_connector/v1/origami/):

save     RawBytesTensorAdapter.quantize (quantization/raw_tensor.py:100-122): the layer's
         gathered blocks on the host, viewed as bytes (symbols [1, 1, N], 8 bits);
         the planner's 1 MiB slices of them (lossless/chunking.py:22-123 with
         bytes_per_symbol = 1, worker.py:1992-2001); each slice through
         CpuLosslessCodec("zlib") (lossless/cpu_qat.py:64-73: zlib level 1, raw deflate,
         window bits -15, default strategy).
restore  each chunk through zlib.decompress(wbits=-15) with the length check
         (cpu_qat.py:75-84); torch.cat of the chunks; RawBytesTensorAdapter.dequantize
         (raw_tensor.py:125-157: byte count check, view as the cache dtype, reshape);
         _assign_blocks (benchmark_utils.py:434-444): index_copy_ of the blocks into the
         cache along its block dimension.

Pinned by tests/test_ref_lossless.py against the reference's own zlib streams
(tests/golden/zlib_case.npz), raw-bytes symbols and chunk plan
(tests/golden/raw_bytes_case.npz) and block selection (tests/golden/select_blocks.npz).
"""
from __future__ import annotations

import zlib
from dataclasses import dataclass

import numpy as np
import torch

CHUNK_BYTES = 1 << 20


def raw_quantize(gathered: torch.Tensor) -> tuple[torch.Tensor, dict]:
    """raw_tensor.py:100-122."""
    tensor = gathered.detach().cpu().contiguous()
    symbols = tensor.view(torch.uint8).reshape(-1).clone()
    meta = {
        "format": "raw_bytes",
        "dtype": str(tensor.dtype).replace("torch.", ""),
        "shape": [int(d) for d in tensor.shape],
        "byte_count": int(symbols.numel()),
        "origami_bits": 8,
        "origami_symbol_shape": [1, 1, int(symbols.numel())],
        "origami_symbol_layout": ["token", "head", "head_dim"],
    }
    return symbols, meta


def slice_bounds(n: int, chunk_bytes: int = CHUNK_BYTES) -> list[int]:
    """The planner's plan for [1, 1, n] byte symbols at min = target = max = chunk_bytes:
    consecutive chunk_bytes-wide channel ranges of the single head (chunking.py:95-121)."""
    return list(range(0, n, chunk_bytes)) + [n]


def zlib_compress(chunk: np.ndarray) -> bytes:
    """cpu_qat.py:64-73."""
    c = zlib.compressobj(level=1, wbits=-15, strategy=zlib.Z_DEFAULT_STRATEGY)
    return c.compress(chunk.tobytes()) + c.flush()


def zlib_decompress(data: bytes, output_bytes: int) -> torch.Tensor:
    """cpu_qat.py:75-84."""
    decoded = zlib.decompress(data, wbits=-15)
    if len(decoded) != int(output_bytes):
        raise RuntimeError(f"Origami CPU lossless decoded {len(decoded)} bytes, expected {int(output_bytes)}")
    return torch.frombuffer(bytearray(decoded), dtype=torch.uint8).clone()


def raw_dequantize(symbols: torch.Tensor, meta: dict) -> torch.Tensor:
    """raw_tensor.py:125-157 (without a destination cache)."""
    raw = symbols.detach().cpu().to(torch.uint8).reshape(-1).contiguous()
    dtype = getattr(torch, meta["dtype"])
    shape = [int(d) for d in meta["shape"]]
    expected = int(np.prod(shape)) * torch.empty((), dtype=dtype).element_size()
    if int(raw.numel()) != expected:
        raise RuntimeError(f"Origami raw-bytes payload size mismatch: got {int(raw.numel())}, expected {expected}")
    return raw.view(dtype).reshape(shape).contiguous()


def assign_blocks(cache: torch.Tensor, block_ids: list[int], value: torch.Tensor) -> None:
    """benchmark_utils.py:434-444 for an already block-shaped value."""
    ids = torch.tensor(list(block_ids), dtype=torch.long, device=cache.device)
    value = value.to(device=cache.device, dtype=cache.dtype)
    if cache.dim() >= 2 and cache.shape[0] == 2 and value.shape[0] == 2:
        cache.index_copy_(1, ids, value)
    else:
        cache.index_copy_(0, ids, value)


@dataclass
class SavedLayer:
    chunks: list[bytes]
    sizes: list[int]
    meta: dict


def save_layer(cache: torch.Tensor, block_ids: list[int], chunk_bytes: int = CHUNK_BYTES) -> SavedLayer:
    """Gather (worker.py:1881-1897), raw-bytes symbols, 1 MiB slices, zlib."""
    ids = torch.tensor(list(block_ids), dtype=torch.long)
    dim = 1 if cache.shape[0] == 2 else 0
    return save_gathered(torch.index_select(cache, dim, ids), chunk_bytes)


def save_gathered(gathered: torch.Tensor, chunk_bytes: int = CHUNK_BYTES) -> SavedLayer:
    """Raw-bytes symbols of already gathered blocks, 1 MiB slices, zlib."""
    symbols, meta = raw_quantize(gathered)
    data = symbols.numpy()
    bounds = slice_bounds(data.size, chunk_bytes)
    chunks = [zlib_compress(data[a:b]) for a, b in zip(bounds[:-1], bounds[1:])]
    return SavedLayer(chunks, [b - a for a, b in zip(bounds[:-1], bounds[1:])], meta)


def restore_layer(saved: SavedLayer, cache: torch.Tensor, block_ids: list[int]) -> None:
    """Decompress, concatenate, dequantize, index_copy_ into the cache."""
    parts = [zlib_decompress(c, n) for c, n in zip(saved.chunks, saved.sizes)]
    value = raw_dequantize(torch.cat(parts), saved.meta)
    assign_blocks(cache, block_ids, value)
