"""Per-layer save / restore on a vLLM paged KV cache (torch front end of the C ABI).

pack_layer    : gather a request's blocks, split into planes, pack into the layer's
                chunks (replaces _select_blocks + quantize + _pack_quantized_symbols,
                worker.py:1881-2040).
restore_layer : unpack, merge planes and scatter into the paged cache by block table
                (replaces the bit-unpack + materialize + copy_kv_to_hbm restore,
                worker.py:1087-1248, benchmark_utils.py:434-532).
gather_blocks / scatter_blocks : the reference's raw-bytes layout (index_select /
                index_copy_ along the block dimension).

Every op enqueues on the given (or current) stream and never synchronises. The cache
layouts are vLLM's [2, num_blocks, block_size, H, D] and [num_blocks, 2, block_size, H,
D]; the block dimension follows the reference rule (worker.py:1881-1885).
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import numpy as np
import torch

from origami_b200 import _lib
from origami_b200.planes import LayerFormat


def cache_layout(kv_layer: torch.Tensor) -> int:
    if kv_layer.dim() != 5:
        raise ValueError(f"paged KV cache layer must be 5-D, got shape {tuple(kv_layer.shape)}")
    if int(kv_layer.shape[0]) in (1, 2):
        if int(kv_layer.shape[0]) != 2:
            raise ValueError("KV-first cache must have 2 planes (K, V) on dim 0")
        return _lib.ORIGAMI_KV_FIRST
    if int(kv_layer.shape[1]) == 2:
        return _lib.ORIGAMI_BLOCKS_FIRST
    raise ValueError(f"unsupported paged KV cache shape {tuple(kv_layer.shape)}")


def paged_desc(kv_layer: torch.Tensor) -> _lib.PagedKV:
    if not kv_layer.is_cuda or not kv_layer.is_contiguous():
        raise ValueError("paged KV cache must be a contiguous CUDA tensor")
    if kv_layer.element_size() != 2:
        raise ValueError("paged KV cache elements must be 16-bit (bf16 / fp16)")
    layout = cache_layout(kv_layer)
    if layout == _lib.ORIGAMI_KV_FIRST:
        _, nb, bs, h, d = kv_layer.shape
    else:
        nb, _, bs, h, d = kv_layer.shape
    return _lib.PagedKV(kv_layer.data_ptr(), layout, 2, int(nb), int(bs), int(h), int(d))


def planes_desc(fmt: LayerFormat) -> _lib.Planes:
    pl = _lib.Planes()
    pl.num_planes = fmt.planes.num_planes
    for i, (s, b) in enumerate(zip(fmt.planes.shifts, fmt.planes.bits)):
        pl.shift[i] = s
        pl.bits[i] = b
    return pl


def block_ids_tensor(block_ids, device: torch.device) -> torch.Tensor:
    if isinstance(block_ids, torch.Tensor):
        t = block_ids
        if t.device != device or t.dtype != torch.int64:
            t = t.to(device=device, dtype=torch.int64, non_blocking=True)
        return t.contiguous()
    host = torch.tensor([int(b) for b in block_ids], dtype=torch.int64).pin_memory()
    return host.to(device, non_blocking=True)


def _stream_handle(stream: torch.cuda.Stream | None, device: torch.device) -> int:
    return (stream or torch.cuda.current_stream(device)).cuda_stream


def _table(fmt: LayerFormat, device: torch.device) -> _lib.ChunkTable:
    d_specs, d_offsets = fmt.device_tables(device)
    return _lib.ChunkTable(d_specs.data_ptr(), d_offsets.data_ptr(), fmt.specs.ctypes.data,
                           fmt.offsets.ctypes.data, fmt.num_specs)


def pack_layer(kv_layer: torch.Tensor, block_ids, fmt: LayerFormat, *, out: torch.Tensor | None = None,
               stream: torch.cuda.Stream | None = None, error_count: torch.Tensor | None = None) -> torch.Tensor:
    """Pack the first fmt.num_tokens tokens of a request into fmt's chunk layout.

    Returns the packed uint8 buffer (device); fmt.chunk_views(result) are the chunks.
    """
    device = kv_layer.device
    desc = paged_desc(kv_layer)
    if desc.num_heads != fmt.num_heads or desc.head_dim != fmt.head_dim:
        raise ValueError("layer format heads / head_dim do not match the cache")
    ids = block_ids_tensor(block_ids, device)
    if out is None:
        out = fmt.alloc_packed(device)
    if out.numel() < fmt.packed_bytes or out.dtype != torch.uint8 or not out.is_cuda:
        raise ValueError("packed output must be a uint8 CUDA tensor of fmt.packed_bytes bytes")
    pl = planes_desc(fmt)
    tab = _table(fmt, device)
    with torch.cuda.device(device):
        rc = _lib.lib().origami_pack_layer_from_paged(
            ctypes.byref(desc), ids.data_ptr(), ids.numel(), fmt.num_tokens, ctypes.byref(pl), ctypes.byref(tab),
            out.data_ptr(), out.numel(), error_count.data_ptr() if error_count is not None else None,
            _stream_handle(stream, device))
    _lib.check(rc, "origami_pack_layer_from_paged")
    return out


def restore_layer(packed: torch.Tensor, fmt: LayerFormat, kv_layer: torch.Tensor, block_ids, *,
                  stream: torch.cuda.Stream | None = None, error_count: torch.Tensor | None = None,
                  num_tokens: int | None = None) -> None:
    """Restore tokens [0, fmt.num_tokens) of a request into the paged cache, or only the
    first `num_tokens` of them (a prefix restore: later token rows are left as they are)."""
    device = kv_layer.device
    desc = paged_desc(kv_layer)
    if desc.num_heads != fmt.num_heads or desc.head_dim != fmt.head_dim:
        raise ValueError("layer format heads / head_dim do not match the cache")
    if not packed.is_cuda or packed.device != device or packed.dtype != torch.uint8:
        raise ValueError("packed input must be a uint8 tensor on the cache's device")
    ids = block_ids_tensor(block_ids, device)
    pl = planes_desc(fmt)
    tab = _table(fmt, device)
    err = error_count.data_ptr() if error_count is not None else None
    with torch.cuda.device(device):
        if num_tokens is None or int(num_tokens) == fmt.num_tokens:
            rc = _lib.lib().origami_restore_layer_to_paged(
                packed.data_ptr(), packed.numel(), ctypes.byref(pl), ctypes.byref(tab), ctypes.byref(desc),
                ids.data_ptr(), ids.numel(), fmt.num_tokens, err, _stream_handle(stream, device))
            what = "origami_restore_layer_to_paged"
        else:
            rc = _lib.lib().origami_restore_layer_prefix_to_paged(
                packed.data_ptr(), packed.numel(), ctypes.byref(pl), ctypes.byref(tab), ctypes.byref(desc),
                ids.data_ptr(), ids.numel(), fmt.num_tokens, int(num_tokens), err, _stream_handle(stream, device))
            what = "origami_restore_layer_prefix_to_paged"
    _lib.check(rc, what)


def _jobs(kv_layers, block_ids, device) -> tuple[_lib.PagedKV, ctypes.Array, list]:
    if len(kv_layers) != len(block_ids) or not kv_layers:
        raise ValueError("one block table per job is required")
    descs = [paged_desc(t) for t in kv_layers]
    d0 = descs[0]
    for d in descs[1:]:
        if (d.layout, d.num_blocks, d.block_size, d.num_heads, d.head_dim) != (
                d0.layout, d0.num_blocks, d0.block_size, d0.num_heads, d0.head_dim):
            raise ValueError("batched jobs must share the cache geometry")
    ids = [block_ids_tensor(b, device) for b in block_ids]
    arr = (_lib.LayerJob * len(descs))(*[_lib.LayerJob(d.d_data, i.data_ptr(), i.numel()) for d, i in zip(descs, ids)])
    return d0, arr, ids


def job_stride(fmt: LayerFormat) -> int:
    """Byte stride of consecutive jobs in a batched packed buffer (16-byte multiple)."""
    return (fmt.packed_bytes + 15) // 16 * 16


def alloc_jobs_packed(fmt: LayerFormat, num_jobs: int, device) -> torch.Tensor:
    return torch.empty((num_jobs * job_stride(fmt),), dtype=torch.uint8, device=device)


def restore_layers(packed: torch.Tensor, fmt: LayerFormat, kv_layers, block_ids, *,
                   stream: torch.cuda.Stream | None = None, error_count: torch.Tensor | None = None) -> None:
    """Restore len(kv_layers) jobs (layers / requests sharing fmt) in as few launches as
    possible; job j's chunks start at packed[j * job_stride(fmt)]."""
    device = kv_layers[0].device
    d0, arr, _ids = _jobs(kv_layers, block_ids, device)
    if d0.num_heads != fmt.num_heads or d0.head_dim != fmt.head_dim:
        raise ValueError("layer format heads / head_dim do not match the cache")
    pl = planes_desc(fmt)
    tab = _table(fmt, device)
    with torch.cuda.device(device):
        rc = _lib.lib().origami_restore_layers_to_paged(
            packed.data_ptr(), packed.numel(), job_stride(fmt), ctypes.byref(pl), ctypes.byref(tab), ctypes.byref(d0),
            arr, len(arr), fmt.num_tokens, error_count.data_ptr() if error_count is not None else None,
            _stream_handle(stream, device))
    _lib.check(rc, "origami_restore_layers_to_paged")


def pack_layers(kv_layers, block_ids, fmt: LayerFormat, out: torch.Tensor, *,
                stream: torch.cuda.Stream | None = None, error_count: torch.Tensor | None = None) -> torch.Tensor:
    """Pack len(kv_layers) jobs sharing fmt into `out` (job j at j * job_stride(fmt))."""
    device = kv_layers[0].device
    d0, arr, _ids = _jobs(kv_layers, block_ids, device)
    if d0.num_heads != fmt.num_heads or d0.head_dim != fmt.head_dim:
        raise ValueError("layer format heads / head_dim do not match the cache")
    pl = planes_desc(fmt)
    tab = _table(fmt, device)
    with torch.cuda.device(device):
        rc = _lib.lib().origami_pack_layers_from_paged(
            ctypes.byref(d0), arr, len(arr), fmt.num_tokens, ctypes.byref(pl), ctypes.byref(tab), out.data_ptr(),
            out.numel(), job_stride(fmt), error_count.data_ptr() if error_count is not None else None,
            _stream_handle(stream, device))
    _lib.check(rc, "origami_pack_layers_from_paged")
    return out


def gather_blocks(kv_layer: torch.Tensor, block_ids, *, out: torch.Tensor | None = None,
                  stream: torch.cuda.Stream | None = None, error_count: torch.Tensor | None = None) -> torch.Tensor:
    """index_select along the block dimension; returns the gathered blocks."""
    device = kv_layer.device
    desc = paged_desc(kv_layer)
    ids = block_ids_tensor(block_ids, device)
    n = ids.numel()
    shape = (2, n) + tuple(kv_layer.shape[2:]) if desc.layout == _lib.ORIGAMI_KV_FIRST else (n, 2) + tuple(
        kv_layer.shape[2:])
    if out is None:
        out = torch.empty(shape, dtype=kv_layer.dtype, device=device)
    nbytes = out.numel() * out.element_size()
    with torch.cuda.device(device):
        rc = _lib.lib().origami_gather_blocks(ctypes.byref(desc), ids.data_ptr(), n, out.data_ptr(), nbytes,
                                              error_count.data_ptr() if error_count is not None else None,
                                              _stream_handle(stream, device))
    _lib.check(rc, "origami_gather_blocks")
    return out


def scatter_blocks(value: torch.Tensor, kv_layer: torch.Tensor, block_ids, *,
                   stream: torch.cuda.Stream | None = None, error_count: torch.Tensor | None = None) -> None:
    """index_copy_ of gathered blocks (or their raw bytes) back into the cache."""
    device = kv_layer.device
    desc = paged_desc(kv_layer)
    ids = block_ids_tensor(block_ids, device)
    if not value.is_cuda or value.device != device or not value.is_contiguous():
        raise ValueError("value must be a contiguous tensor on the cache's device")
    nbytes = value.numel() * value.element_size()
    with torch.cuda.device(device):
        rc = _lib.lib().origami_scatter_blocks(value.data_ptr(), nbytes, ctypes.byref(desc), ids.data_ptr(),
                                               ids.numel(), error_count.data_ptr() if error_count is not None else None,
                                               _stream_handle(stream, device))
    _lib.check(rc, "origami_scatter_blocks")


def fused_kernel_name(fmt: LayerFormat, restore: bool = True) -> str:
    """Name of the kernel the fused op launches for this format (the dispatch rules of
    csrc/abi.cu, the packed buffer assumed 16-byte aligned): for the plane presets with
    contiguous runs, the row kernels at head_dim 128 / 256 (restore for every preset, pack
    for byte planes with ragged runs), else TMA tensor-map kernels for 16-byte aligned runs and bulk-copy
    kernels for byte-aligned runs; generic tile kernels otherwise."""
    presets = {(8, 0): (8, 8), (7, 15, 0): (8, 1, 7), (10, 8, 0): (6, 2, 8)}
    D, T = fmt.head_dim, fmt.num_tokens
    tt = 8 * (2048 // D)
    preset = presets.get(tuple(fmt.planes.shifts)) == tuple(fmt.planes.bits) and D in (64, 128, 256)
    aligned = preset and all((T * b) % 128 == 0 and (tt * b) % 128 == 0 for b in fmt.planes.bits)
    ragged = preset and not aligned and all((T * b) % 8 == 0 for b in fmt.planes.bits)
    if (aligned or ragged) and D in (128, 256) and (restore or (ragged and tuple(fmt.planes.bits) == (8, 8))):
        return "restore_rows" if restore else "pack_rows"
    if aligned:
        return "restore_tma" if restore else "pack_tma"
    if ragged:
        return "restore_bulk" if restore else "pack_bulk"
    return "restore_tiles" if restore else "pack_tiles"


def raw_chunk_bounds(total_bytes: int, chunk_bytes: int = 1 << 20) -> np.ndarray:
    """Byte bounds of the reference's raw-bytes chunks: the planner over a
    [1, 1, total_bytes] symbol tensor yields contiguous slices (chunking.py:95-121)."""
    from origami_b200.lossless.chunking import plan_head_channel_chunks

    plan = plan_head_channel_chunks(layer_index=0, num_heads=1, head_dim=int(total_bytes), token_count=1,
                                    bytes_per_symbol=1, min_bytes=chunk_bytes, target_bytes=chunk_bytes,
                                    max_bytes=chunk_bytes)
    return np.asarray([0] + [c.layout.channel_end for c in plan], dtype=np.int64)


def split_raw(gathered: torch.Tensor, bounds: Sequence[int]) -> list[torch.Tensor]:
    flat = gathered.reshape(-1).view(torch.uint8)
    return [flat[int(a):int(b)] for a, b in zip(bounds[:-1], bounds[1:])]
