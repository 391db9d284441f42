"""Drop-in for the reference's ``lossless/native_gpu.py`` canonical bitpack ops.

Same entry points and argument meaning as the reference (lossless/native_gpu.py:35-146
and the extension export unpack_canonical_storage_chunks_cuda,
bitpack_layout_cuda.cpp:316-400), served by liborigami_b200.so. Differences that keep
results identical but remove the reference's stalls:

* chunk tables are built once on the host, validated there and uploaded with one
  pinned non-blocking copy (the reference copies them back with three ``.cpu()``
  calls, cpp:156, 350-351);
* host chunks are concatenated in pinned memory and sent in one copy instead of one
  copy per chunk (native_gpu.py:92-110);
* everything is enqueued on the current stream, nothing synchronises.
"""
from __future__ import annotations

from typing import Any, Iterable, Sequence

import numpy as np
import torch

from origami_b200 import _lib
from origami_b200.lossless import native_cpu


def _cuda_required() -> None:
    if not torch.cuda.is_available():
        raise RuntimeError("Origami CUDA bitpack extension requires CUDA")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _np_ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def upload_i64(values: np.ndarray, device: torch.device) -> torch.Tensor:
    """One pinned, non-blocking host->device copy of an int64 table."""
    host = torch.from_numpy(np.ascontiguousarray(values, dtype=np.int64)).pin_memory()
    return host.to(device, non_blocking=True)


def _host_i64(values: torch.Tensor | Sequence[int] | np.ndarray) -> np.ndarray:
    if isinstance(values, torch.Tensor):
        values = values.detach().to("cpu", torch.int64)
        return np.ascontiguousarray(values.numpy(), dtype=np.int64)
    return np.ascontiguousarray(np.asarray(values, dtype=np.int64))


def _specs_np(chunk_specs: torch.Tensor | Iterable[Iterable[int]]) -> np.ndarray:
    if isinstance(chunk_specs, torch.Tensor):
        specs = _host_i64(chunk_specs)
    else:
        rows = [list(r) for r in chunk_specs]
        specs = np.asarray(rows, dtype=np.int64) if rows else np.empty((0, 6), dtype=np.int64)
    if specs.size == 0:
        return np.empty((0, 6), dtype=np.int64)
    return np.ascontiguousarray(specs.reshape(-1, 6))


def _bits_list(bits: int | Sequence[int], n: int) -> np.ndarray:
    if isinstance(bits, (int, np.integer)):
        return np.full(n, int(bits), dtype=np.int64)
    out = np.asarray([int(b) for b in bits], dtype=np.int64)
    if len(out) != n:
        raise ValueError("bits_per_chunk length must match chunk_specs")
    return out


def spec_symbol_counts(specs: np.ndarray) -> np.ndarray:
    return (specs[:, 1] - specs[:, 0]) * (specs[:, 3] - specs[:, 2]) * (specs[:, 5] - specs[:, 4])


class _Extension:
    """The reference extension's tensor-level surface (bitpack_layout_cuda.cpp:894-903)."""

    def unpack_canonical_storage_chunks_cuda(
        self,
        flat_chunks: torch.Tensor,
        chunk_offsets: torch.Tensor,
        bits_per_chunk: torch.Tensor,
        source_shape: torch.Tensor,
        axis_positions: torch.Tensor,
        token_count: int,
        num_heads: int,
        head_dim: int,
        chunk_specs: torch.Tensor,
    ) -> torch.Tensor:
        if not flat_chunks.is_cuda or not flat_chunks.is_contiguous():
            raise RuntimeError("flat_chunks must be a contiguous CUDA tensor")
        if flat_chunks.dtype != torch.uint8:
            raise RuntimeError("flat_chunks must be uint8")
        device = flat_chunks.device
        h_specs = _specs_np(chunk_specs)
        h_offsets = _host_i64(chunk_offsets)
        h_bits = _host_i64(bits_per_chunk)
        if len(h_offsets) != len(h_specs) + 1:
            raise RuntimeError("chunk_offsets length must be chunk count + 1")
        if len(h_bits) != len(h_specs):
            raise RuntimeError("bits_per_chunk length must equal chunk count")
        return unpack_flat(flat_chunks, h_offsets, h_bits, h_specs, _host_i64(source_shape),
                           _host_i64(axis_positions), int(token_count), int(num_heads), int(head_dim),
                           d_tables=(chunk_offsets, bits_per_chunk, chunk_specs) if chunk_offsets.is_cuda else None,
                           device=device)

    def pack_canonical_storage_chunks_cuda(
        self,
        symbols: torch.Tensor,
        chunk_offsets: torch.Tensor,
        bits_per_chunk: torch.Tensor,
        source_shape: torch.Tensor,
        axis_positions: torch.Tensor,
        token_count: int,
        num_heads: int,
        head_dim: int,
        chunk_specs: torch.Tensor,
    ) -> torch.Tensor:
        if not symbols.is_cuda or not symbols.is_contiguous() or symbols.dtype != torch.uint8:
            raise RuntimeError("symbols must be a contiguous uint8 CUDA tensor")
        return pack_flat(symbols, _host_i64(chunk_offsets), _host_i64(bits_per_chunk), _specs_np(chunk_specs),
                         _host_i64(source_shape), _host_i64(axis_positions), int(token_count), int(num_heads),
                         int(head_dim), device=symbols.device)


    # The quantized restore exports (cpp:897-901) keep the reference's positional
    # signatures; origami_b200.quant holds the checks and the library calls.
    def cachegen_unpack_dequantize_cuda(self, *args: Any) -> torch.Tensor:
        from origami_b200 import quant

        return quant.cachegen_unpack_dequantize_cuda(*args)

    def cachegen_unpack_dequantize_to_kv_cache_cuda(self, *args: Any) -> None:
        from origami_b200 import quant

        quant.cachegen_unpack_dequantize_to_kv_cache_cuda(*args)

    def kivi_dequantize_to_kv_cache_cuda(self, *args: Any) -> None:
        from origami_b200 import quant

        quant.kivi_dequantize_to_kv_cache_cuda(*args)

    def fused_prefix_attention_cuda(self, *args: Any, **kwargs: Any) -> None:
        from origami_b200 import attention

        attention.fused_prefix_attention_cuda(*args, **kwargs)


_EXT = _Extension()


def load_bitpack_cuda_extension() -> Any:
    """Return the extension object (the reference JIT-builds; this loads the prebuilt
    in-tree library and raises when it or CUDA is missing)."""
    _cuda_required()
    _lib.lib()
    return _EXT


def available() -> bool:
    if not torch.cuda.is_available():
        return False
    try:
        load_bitpack_cuda_extension()
        return True
    except Exception:
        return False


def _tables(device, h_offsets, h_bits, h_specs, d_tables):
    if d_tables is not None:
        d_off, d_bits, d_specs = (t.to(device=device, dtype=torch.int64).contiguous() for t in d_tables)
    else:
        d_off, d_bits, d_specs = (upload_i64(a, device) for a in (h_offsets, h_bits, h_specs))
    return d_off, d_bits, d_specs


def unpack_flat(flat: torch.Tensor, h_offsets: np.ndarray, h_bits: np.ndarray, h_specs: np.ndarray,
                shape: np.ndarray, axes: np.ndarray, token_count: int, num_heads: int, head_dim: int, *,
                d_tables=None, device: torch.device) -> torch.Tensor:
    L = _lib.lib()
    numel = int(np.prod(shape)) if len(shape) else 0
    out = torch.empty((numel,), dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        d_off, d_bits, d_specs = _tables(device, h_offsets, h_bits, h_specs, d_tables)
        rc = L.origami_unpack_canonical_storage_chunks(
            _ptr(flat), flat.numel(), _ptr(d_off), _ptr(d_bits), _ptr(d_specs),
            _np_ptr(h_offsets), _np_ptr(h_bits), _np_ptr(h_specs), len(h_specs),
            _np_ptr(shape), len(shape), _np_ptr(axes), token_count, num_heads, head_dim,
            _ptr(out), numel, _stream(device))
    _lib.check(rc, "origami_unpack_canonical_storage_chunks")
    return out


def pack_flat(symbols: torch.Tensor, h_offsets: np.ndarray, h_bits: np.ndarray, h_specs: np.ndarray,
              shape: np.ndarray, axes: np.ndarray, token_count: int, num_heads: int, head_dim: int, *,
              device: torch.device) -> torch.Tensor:
    """Pack symbols into one flat chunk buffer laid out by h_offsets."""
    L = _lib.lib()
    total = int(h_offsets[-1]) if len(h_offsets) else 0
    storage = torch.empty(((total + 15) // 16 * 16,), dtype=torch.uint8, device=device)
    flat = storage[:total]
    with torch.cuda.device(device):
        d_off, d_bits, d_specs = _tables(device, h_offsets, h_bits, h_specs, None)
        rc = L.origami_pack_canonical_storage_chunks(
            _ptr(symbols), symbols.numel(), _ptr(d_off), _ptr(d_bits), _ptr(d_specs),
            _np_ptr(h_offsets), _np_ptr(h_bits), _np_ptr(h_specs), len(h_specs),
            _np_ptr(shape), len(shape), _np_ptr(axes), token_count, num_heads, head_dim,
            _ptr(storage), total, _stream(device))
    _lib.check(rc, "origami_pack_canonical_storage_chunks")
    return flat


def _flat_chunks(chunks: list[torch.Tensor], device: torch.device) -> tuple[torch.Tensor, np.ndarray]:
    flats = [c.detach().reshape(-1).to(torch.uint8) for c in chunks]
    sizes = [int(f.numel()) for f in flats]
    offsets = np.concatenate([[0], np.cumsum(sizes, dtype=np.int64)]).astype(np.int64)
    total = int(offsets[-1])
    if not flats:
        return torch.empty((0,), dtype=torch.uint8, device=device), offsets
    if all(f.device == device for f in flats):
        return (torch.cat(flats) if len(flats) > 1 else flats[0].contiguous()), offsets
    host = torch.empty((total,), dtype=torch.uint8, pin_memory=True)
    for f, a, b in zip(flats, offsets[:-1], offsets[1:]):
        host[int(a):int(b)].copy_(f.cpu())
    return host.to(device, non_blocking=True), offsets


def unpack_canonical_storage_chunks(
    chunks: Iterable[torch.Tensor],
    bits: int | Sequence[int],
    source_shape: Sequence[int],
    source_layout: Sequence[str],
    chunk_specs: torch.Tensor | Iterable[Iterable[int]],
    *,
    device: torch.device | str | None = None,
) -> torch.Tensor:
    """Same contract as the reference (native_gpu.py:113-146): uint8 tensor in source
    layout, zero where no chunk writes."""
    _cuda_required()
    target = torch.device(device or "cuda")
    if target.index is None:
        target = torch.device("cuda", torch.cuda.current_device())
    token_count, num_heads, head_dim, shape, layout = native_cpu.canonical_axis_sizes(source_shape, source_layout)
    specs = _specs_np(chunk_specs)
    bits_arr = _bits_list(bits, len(specs))
    flat, offsets = _flat_chunks(list(chunks), target)
    if len(offsets) != len(specs) + 1:
        raise RuntimeError("Origami native layout metadata chunk count does not match payload chunks")
    return unpack_flat(flat, offsets, bits_arr, specs, np.asarray(shape, dtype=np.int64),
                       np.asarray(native_cpu.axis_positions(layout), dtype=np.int64),
                       token_count, num_heads, head_dim, device=target)


def pack_canonical_storage_chunks(
    symbols: torch.Tensor,
    bits: int | Sequence[int],
    source_shape: Sequence[int],
    source_layout: Sequence[str],
    chunk_specs: torch.Tensor | Iterable[Iterable[int]],
    *,
    device: torch.device | str | None = None,
) -> list[torch.Tensor]:
    """Inverse of unpack_canonical_storage_chunks: one packed uint8 tensor per spec,
    on the symbols' device (CPU symbols are packed on the GPU and copied back)."""
    _cuda_required()
    token_count, num_heads, head_dim, shape, layout = native_cpu.canonical_axis_sizes(source_shape, source_layout)
    specs = _specs_np(chunk_specs)
    bits_arr = _bits_list(bits, len(specs))
    if bits_arr.size and (bits_arr.min() < 1 or bits_arr.max() > 8):
        raise ValueError("origami_bits must be in the range 1..8")
    home = symbols.device
    target = home if home.type == "cuda" else torch.device(device or "cuda")
    if target.index is None:
        target = torch.device("cuda", torch.cuda.current_device())
    flat_symbols = symbols.detach().reshape(-1).to(torch.uint8)
    if flat_symbols.numel() != int(np.prod(shape)):
        raise ValueError("Origami quantizer symbol count must equal origami_symbol_shape product")
    if flat_symbols.device != target:
        flat_symbols = flat_symbols.contiguous().pin_memory().to(target, non_blocking=True)
    flat_symbols = flat_symbols.contiguous()
    sizes = (spec_symbol_counts(specs) * bits_arr + 7) // 8
    offsets = np.concatenate([[0], np.cumsum(sizes, dtype=np.int64)]).astype(np.int64)
    flat = pack_flat(flat_symbols, offsets, bits_arr, specs, np.asarray(shape, dtype=np.int64),
                     np.asarray(native_cpu.axis_positions(layout), dtype=np.int64),
                     token_count, num_heads, head_dim, device=target)
    if home.type != "cuda":
        host = torch.empty((flat.numel(),), dtype=torch.uint8, pin_memory=True)
        host.copy_(flat, non_blocking=True)
        torch.cuda.current_stream(target).synchronize()
        flat = host
    return [flat[int(a):int(b)] for a, b in zip(offsets[:-1], offsets[1:])]


def cachegen_unpack_dequantize(
    bytestream: torch.Tensor,
    offsets: torch.Tensor,
    bits_per_layer: torch.Tensor,
    key_bins: torch.Tensor,
    value_bins: torch.Tensor,
    max_key: torch.Tensor,
    max_value: torch.Tensor,
    *,
    tokens: int,
    heads: int,
    head_dim: int,
) -> torch.Tensor:
    """native_gpu.py:149-175 of the reference."""
    ext = load_bitpack_cuda_extension()
    dev = bytestream.device
    return ext.cachegen_unpack_dequantize_cuda(
        bytestream.reshape(-1).contiguous(),
        offsets.to(device=dev, dtype=torch.int64).contiguous(),
        bits_per_layer.to(device=dev, dtype=torch.int64).contiguous(),
        key_bins.to(device=dev, dtype=torch.int64).contiguous(),
        value_bins.to(device=dev, dtype=torch.int64).contiguous(),
        max_key.contiguous(),
        max_value.contiguous(),
        int(tokens),
        int(heads),
        int(head_dim),
    )


def cachegen_unpack_dequantize_to_kv_cache(
    bytestream: torch.Tensor,
    *,
    key_offset: int,
    key_bytes: int,
    value_offset: int,
    value_bytes: int,
    key_bits: int,
    value_bits: int,
    key_bins: int,
    value_bins: int,
    max_key: torch.Tensor,
    max_value: torch.Tensor,
    kv_cache: torch.Tensor,
    block_ids: torch.Tensor,
    tokens: int,
    heads: int,
    head_dim: int,
) -> None:
    """native_gpu.py:178-215 of the reference (called by cachegen_adapter.py:770)."""
    ext = load_bitpack_cuda_extension()
    ext.cachegen_unpack_dequantize_to_kv_cache_cuda(
        bytestream.reshape(-1).contiguous(),
        int(key_offset),
        int(key_bytes),
        int(value_offset),
        int(value_bytes),
        int(key_bits),
        int(value_bits),
        int(key_bins),
        int(value_bins),
        max_key.contiguous(),
        max_value.contiguous(),
        kv_cache,
        block_ids.to(device=kv_cache.device, dtype=torch.int64).contiguous(),
        int(tokens),
        int(heads),
        int(head_dim),
    )


def kivi_dequantize_to_kv_cache(
    bytestream: torch.Tensor,
    *,
    key_offset: int,
    key_bytes: int,
    value_offset: int,
    value_bytes: int,
    bits: int,
    group_size: int,
    sink_tokens: int,
    key_scale: torch.Tensor,
    key_zero: torch.Tensor,
    value_scale: torch.Tensor,
    value_zero: torch.Tensor,
    key_sink: torch.Tensor,
    value_sink: torch.Tensor,
    kv_cache: torch.Tensor,
    block_ids: torch.Tensor,
    tokens: int,
    heads: int,
    head_dim: int,
) -> None:
    """native_gpu.py:218-260 of the reference (called by kivi_adapter.py:643)."""
    ext = load_bitpack_cuda_extension()
    ext.kivi_dequantize_to_kv_cache_cuda(
        bytestream.reshape(-1).contiguous(),
        int(key_offset),
        int(key_bytes),
        int(value_offset),
        int(value_bytes),
        int(bits),
        int(group_size),
        int(sink_tokens),
        key_scale.contiguous(),
        key_zero.contiguous(),
        value_scale.contiguous(),
        value_zero.contiguous(),
        key_sink.contiguous(),
        value_sink.contiguous(),
        kv_cache,
        block_ids.to(device=kv_cache.device, dtype=torch.int64).contiguous(),
        int(tokens),
        int(heads),
        int(head_dim),
    )


def _fp16_blob_view(bytestream: torch.Tensor, metadata: dict[str, Any], name: str) -> torch.Tensor:
    """An fp16 metadata tensor stored inside the artifact's bytestream (native_gpu.py:264-276)."""
    offset = int(metadata[f"{name}_offset"])
    numel = int(metadata[f"{name}_numel"])
    byte_count = numel * 2
    if offset < 0 or offset + byte_count > int(bytestream.numel()):
        raise ValueError(f"{name} range exceeds the Origami artifact")
    if offset % 2:
        raise ValueError(f"{name} must be aligned for float16 access")
    return bytestream.narrow(0, offset, byte_count).view(torch.float16)


def _fused_prefix_attention(bytestream: torch.Tensor, *, codec: int, metadata: dict[str, Any],
                            key_scale: torch.Tensor, key_zero: torch.Tensor, value_scale: torch.Tensor,
                            value_zero: torch.Tensor, key_sink: torch.Tensor, value_sink: torch.Tensor,
                            query: torch.Tensor, kv_cache: torch.Tensor, block_table: torch.Tensor,
                            query_start_position: int, sequence_length: int, softmax_scale: float,
                            output: torch.Tensor) -> None:
    """native_gpu.py:279-343 of the reference: artifact checks, then the fused kernel."""
    if bytestream.device != query.device or query.device != kv_cache.device:
        raise ValueError("compressed payload, query, and KV cache must share a device")
    if query.ndim != 3 or output.shape != query.shape:
        raise ValueError("query and output must be matching rank-3 tensors")
    if kv_cache.ndim != 5 or int(kv_cache.shape[0]) != 2:
        raise ValueError("fused attention requires NHD KV cache shape [2, blocks, block, heads, dim]")
    if int(metadata["head_dim"]) != int(query.shape[2]):
        raise ValueError("artifact head_dim does not match query")
    if int(metadata["num_heads"]) != int(kv_cache.shape[3]):
        raise ValueError("artifact KV head count does not match KV cache")
    if int(kv_cache.shape[4]) != int(query.shape[2]):
        raise ValueError("KV cache head_dim does not match query")
    declared_bytes = int(metadata.get("symbol_byte_count", bytestream.numel()))
    if declared_bytes != int(bytestream.numel()):
        raise ValueError("artifact byte count does not match compressed payload")
    if int(query_start_position) < int(metadata["token_count"]):
        raise ValueError("query starts inside the compressed prefix")
    ext = load_bitpack_cuda_extension()
    ext.fused_prefix_attention_cuda(
        bytestream.reshape(-1).contiguous(), int(metadata["key_stream_offset"]), int(metadata["key_stream_bytes"]),
        int(metadata["value_stream_offset"]), int(metadata["value_stream_bytes"]), int(codec), int(metadata["bits"]),
        int(metadata.get("group_size", 1)), int(metadata.get("sink_tokens", 0)), key_scale.contiguous(),
        key_zero.contiguous(), value_scale.contiguous(), value_zero.contiguous(), key_sink.contiguous(),
        value_sink.contiguous(), query.contiguous(), kv_cache,
        block_table.to(device=kv_cache.device, dtype=torch.int32).contiguous(), int(metadata["token_count"]),
        int(query_start_position), int(sequence_length), float(softmax_scale), output)


def kivi_fused_prefix_attention(bytestream: torch.Tensor, *, metadata: dict[str, Any], query: torch.Tensor,
                                kv_cache: torch.Tensor, block_table: torch.Tensor, query_start_position: int,
                                sequence_length: int, softmax_scale: float, output: torch.Tensor) -> None:
    """native_gpu.py:346-383 of the reference: a structured KIVI artifact (codec 0)."""
    if str(metadata.get("format")) != "kivi_structured_blob":
        raise ValueError("KIVI fused attention requires a structured KIVI artifact")
    if tuple(metadata.get("key_order", ())) != ("head_dim", "layer", "head", "token") or tuple(
            metadata.get("value_order", ())) != ("head", "layer", "head_dim", "token"):
        raise ValueError("KIVI artifact has an unsupported packed layout")
    _fused_prefix_attention(
        bytestream, codec=0, metadata=metadata,
        key_scale=_fp16_blob_view(bytestream, metadata, "key_scale"),
        key_zero=_fp16_blob_view(bytestream, metadata, "key_zero"),
        value_scale=_fp16_blob_view(bytestream, metadata, "value_scale"),
        value_zero=_fp16_blob_view(bytestream, metadata, "value_zero"),
        key_sink=_fp16_blob_view(bytestream, metadata, "key_sink"),
        value_sink=_fp16_blob_view(bytestream, metadata, "value_sink"),
        query=query, kv_cache=kv_cache, block_table=block_table, query_start_position=query_start_position,
        sequence_length=sequence_length, softmax_scale=softmax_scale, output=output)


def kvquant_fused_prefix_attention(bytestream: torch.Tensor, *, metadata: dict[str, Any], query: torch.Tensor,
                                   kv_cache: torch.Tensor, block_table: torch.Tensor, query_start_position: int,
                                   sequence_length: int, softmax_scale: float, output: torch.Tensor) -> None:
    """native_gpu.py:386-420 of the reference: a structured KVQuant artifact (codec 1)."""
    if str(metadata.get("format")) != "kvquant_structured_blob":
        raise ValueError("KVQuant fused attention requires a structured artifact")
    if tuple(metadata.get("key_order", ())) != ("head_dim", "layer", "head", "token") or tuple(
            metadata.get("value_order", ())) != ("layer", "head", "token", "head_dim"):
        raise ValueError("KVQuant artifact has an unsupported packed layout")
    empty = torch.empty((0,), dtype=torch.float16, device=bytestream.device)
    _fused_prefix_attention(
        bytestream, codec=1, metadata=metadata,
        key_scale=_fp16_blob_view(bytestream, metadata, "key_scale"),
        key_zero=_fp16_blob_view(bytestream, metadata, "key_min"),
        value_scale=_fp16_blob_view(bytestream, metadata, "value_scale"),
        value_zero=_fp16_blob_view(bytestream, metadata, "value_min"),
        key_sink=empty, value_sink=empty, query=query, kv_cache=kv_cache, block_table=block_table,
        query_start_position=query_start_position, sequence_length=sequence_length, softmax_scale=softmax_scale,
        output=output)
