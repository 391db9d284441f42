"""Fused dequantize-to-cache ops of the reference's lossy restore paths, served by
liborigami_b200.so (kernels: csrc/quant_kernels.cuh).

* ``cachegen_unpack_dequantize_to_kv_cache_cuda``: CacheGen streams -> paged cache
  (reference bitpack_layout_cuda.cpp:475-580, called by
  quantization/cachegen_adapter.py:770);
* ``cachegen_unpack_dequantize_cuda``: CacheGen streams of several layers -> an fp16
  [layers, 2, heads, tokens, head_dim] tensor (cpp:402-473);
* ``kivi_dequantize_to_kv_cache_cuda``: KIVI streams + scale/zero/sink tensors -> paged
  cache (cpp:583-700, called by quantization/kivi_adapter.py:643).

Same arguments, checks (in the same order) and error messages as the reference extension,
raised as RuntimeError; results are bit-identical to the reference kernels. Work goes to
the current stream of the cache's device; nothing synchronises. ``error_count`` (an int32
CUDA tensor, optional) receives one count per (kv, token, head) row whose block id lies
outside the cache; the reference skips those rows silently.
"""
from __future__ import annotations

import torch

from origami_b200 import _lib

_DTYPE = {torch.float16: _lib.ORIGAMI_DTYPE_F16, torch.bfloat16: _lib.ORIGAMI_DTYPE_BF16,
          torch.float32: _lib.ORIGAMI_DTYPE_F32}


def _check_cuda_contiguous(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _check_i64(t: torch.Tensor, name: str) -> None:
    if t.dtype != torch.int64:
        raise RuntimeError(f"{name} must be int64")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _check_bits(bits: int) -> None:
    if not 1 <= int(bits) <= 8:
        raise RuntimeError("Origami CUDA bitpack supports only 1..8 bit symbols")


def _paged(kv_cache: torch.Tensor, heads: int, head_dim: int) -> _lib.PagedKV:
    """Layout detection of cpp:517-546: [num_blocks, 2, ...] is tried first."""
    if kv_cache.dim() != 5:
        raise RuntimeError("kv_cache must have rank 5")
    if kv_cache.size(1) == 2:
        layout, nb = _lib.ORIGAMI_BLOCKS_FIRST, kv_cache.size(0)
    elif kv_cache.size(0) == 2:
        layout, nb = _lib.ORIGAMI_KV_FIRST, kv_cache.size(1)
    else:
        raise RuntimeError("kv_cache must be [num_blocks,2,block,heads,dim] or [2,num_blocks,block,heads,dim]")
    if kv_cache.size(3) != heads or kv_cache.size(4) != head_dim:
        raise RuntimeError("kv_cache head shape mismatch")
    if kv_cache.size(2) <= 0:
        raise RuntimeError("kv_cache block size must be positive")
    return _lib.PagedKV(kv_cache.data_ptr(), layout, 2, int(nb), int(kv_cache.size(2)), int(heads), int(head_dim))


def _blocks(kv_cache: torch.Tensor, block_ids: torch.Tensor, tokens: int) -> None:
    if block_ids.numel() <= 0:
        raise RuntimeError("block_ids must be non-empty")
    if tokens > block_ids.numel() * kv_cache.size(2):
        raise RuntimeError("tokens exceed destination block capacity")


def _err_ptr(error_count: torch.Tensor | None) -> int | None:
    if error_count is None:
        return None
    if not error_count.is_cuda or error_count.dtype not in (torch.int32, torch.uint32) or error_count.numel() < 1:
        raise RuntimeError("error_count must be a CUDA int32 tensor")
    return error_count.data_ptr()


def cachegen_unpack_dequantize_to_kv_cache_cuda(
    bytestream: torch.Tensor, key_offset: int, key_bytes: int, value_offset: int, value_bytes: int, key_bits: int,
    value_bits: int, key_bins: int, value_bins: int, max_key: torch.Tensor, max_value: torch.Tensor,
    kv_cache: torch.Tensor, block_ids: torch.Tensor, tokens: int, heads: int, head_dim: int, *,
    error_count: torch.Tensor | None = None,
) -> None:
    for t, n in ((bytestream, "bytestream"), (max_key, "max_key"), (max_value, "max_value"),
                 (kv_cache, "kv_cache"), (block_ids, "block_ids")):
        _check_cuda_contiguous(t, n)
    if bytestream.dtype != torch.uint8:
        raise RuntimeError("bytestream must be uint8")
    if kv_cache.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("kv_cache must be float16 or bfloat16")
    _check_i64(block_ids, "block_ids")
    if max_key.dtype != max_value.dtype:
        raise RuntimeError("max_key and max_value must have the same dtype")
    if max_key.dtype not in (torch.float16, torch.float32):
        raise RuntimeError("max tensors must be float16 or float32")
    _check_bits(key_bits)
    _check_bits(value_bits)
    if tokens <= 0 or heads <= 0 or head_dim <= 0:
        raise RuntimeError("tokens, heads, and head_dim must be positive")
    if key_bins <= 1 or value_bins <= 1:
        raise RuntimeError("CacheGen bins must be greater than one")
    if key_offset < 0 or key_bytes < 0 or value_offset < 0 or value_bytes < 0:
        raise RuntimeError("invalid CacheGen stream offsets")
    if key_offset + key_bytes > bytestream.numel() or value_offset + value_bytes > bytestream.numel():
        raise RuntimeError("CacheGen stream ranges exceed bytestream length")
    if max_key.numel() < tokens or max_value.numel() < tokens:
        raise RuntimeError("max tensors must contain at least tokens values")
    kv = _paged(kv_cache, heads, head_dim)
    _blocks(kv_cache, block_ids, tokens)
    device = kv_cache.device
    with torch.cuda.device(device):
        rc = _lib.lib().origami_cachegen_unpack_dequantize_to_kv_cache(
            bytestream.data_ptr(), bytestream.numel(), int(key_offset), int(key_bytes), int(value_offset),
            int(value_bytes), int(key_bits), int(value_bits), int(key_bins), int(value_bins), max_key.data_ptr(),
            max_key.numel(), max_value.data_ptr(), max_value.numel(), _DTYPE[max_key.dtype], kv,
            _DTYPE[kv_cache.dtype], block_ids.data_ptr(), block_ids.numel(), int(tokens), _err_ptr(error_count),
            torch.cuda.current_stream(device).cuda_stream)
    _lib.check(rc, "origami_cachegen_unpack_dequantize_to_kv_cache")


def cachegen_unpack_dequantize_cuda(
    bytestream: torch.Tensor, offsets: torch.Tensor, bits_per_layer: torch.Tensor, key_bins: torch.Tensor,
    value_bins: torch.Tensor, max_key: torch.Tensor, max_value: torch.Tensor, tokens: int, heads: int, head_dim: int,
) -> torch.Tensor:
    for t, n in ((bytestream, "bytestream"), (offsets, "offsets"), (bits_per_layer, "bits_per_layer"),
                 (key_bins, "key_bins"), (value_bins, "value_bins"), (max_key, "max_key"),
                 (max_value, "max_value")):
        _check_cuda_contiguous(t, n)
    if bytestream.dtype != torch.uint8:
        raise RuntimeError("bytestream must be uint8")
    for t, n in ((offsets, "offsets"), (bits_per_layer, "bits_per_layer"), (key_bins, "key_bins"),
                 (value_bins, "value_bins")):
        _check_i64(t, n)
    if max_key.dtype != max_value.dtype:
        raise RuntimeError("max_key and max_value must have the same dtype")
    if max_key.dtype not in (torch.float16, torch.float32):
        raise RuntimeError("max tensors must be float16 or float32")
    if bits_per_layer.numel() % 2 != 0:
        raise RuntimeError("bits_per_layer length must be even")
    layers = bits_per_layer.numel() // 2
    if key_bins.numel() != layers:
        raise RuntimeError("key_bins length must match layers")
    if value_bins.numel() != layers:
        raise RuntimeError("value_bins length must match layers")
    if offsets.numel() != bits_per_layer.numel() + 1:
        raise RuntimeError("offsets length must be bits_per_layer length + 1")
    if max_key.numel() != layers * tokens:
        raise RuntimeError("max_key must have layers * tokens values")
    if max_value.numel() != layers * tokens:
        raise RuntimeError("max_value must have layers * tokens values")
    if tokens <= 0 or heads <= 0 or head_dim <= 0:
        raise RuntimeError("tokens, heads, and head_dim must be positive")
    # The reference copies bits_per_layer to the host to check it (cpp:442-447); so do we,
    # together with the offsets (validated here, so the kernel never reads outside the
    # bytestream).
    h_bits = bits_per_layer.to("cpu")
    h_off = offsets.to("cpu")
    for b in h_bits.tolist():
        _check_bits(b)
    device = bytestream.device
    out = torch.empty((layers, 2, heads, tokens, head_dim), dtype=torch.float16, device=device)
    with torch.cuda.device(device):
        rc = _lib.lib().origami_cachegen_unpack_dequantize(
            bytestream.data_ptr(), bytestream.numel(), offsets.data_ptr(), h_off.data_ptr(), offsets.numel(),
            bits_per_layer.data_ptr(), h_bits.data_ptr(), bits_per_layer.numel(), key_bins.data_ptr(),
            key_bins.numel(), value_bins.data_ptr(), value_bins.numel(), max_key.data_ptr(), max_key.numel(),
            max_value.data_ptr(), max_value.numel(), _DTYPE[max_key.dtype], int(tokens), int(heads), int(head_dim),
            out.data_ptr(), out.numel() * 2, torch.cuda.current_stream(device).cuda_stream)
    _lib.check(rc, "origami_cachegen_unpack_dequantize")
    return out


def kivi_dequantize_to_kv_cache_cuda(
    bytestream: torch.Tensor, key_offset: int, key_bytes: int, value_offset: int, value_bytes: int, bits: int,
    group_size: int, sink_tokens: int, key_scale: torch.Tensor, key_zero: torch.Tensor, value_scale: torch.Tensor,
    value_zero: torch.Tensor, key_sink: torch.Tensor, value_sink: torch.Tensor, kv_cache: torch.Tensor,
    block_ids: torch.Tensor, tokens: int, heads: int, head_dim: int, *, error_count: torch.Tensor | None = None,
) -> None:
    metas = (key_scale, key_zero, value_scale, value_zero, key_sink, value_sink)
    for t, n in ((bytestream, "bytestream"), (key_scale, "key_scale"), (key_zero, "key_zero"),
                 (value_scale, "value_scale"), (value_zero, "value_zero"), (key_sink, "key_sink"),
                 (value_sink, "value_sink"), (kv_cache, "kv_cache"), (block_ids, "block_ids")):
        _check_cuda_contiguous(t, n)
    if bytestream.dtype != torch.uint8:
        raise RuntimeError("bytestream must be uint8")
    if kv_cache.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("kv_cache must be float16 or bfloat16")
    _check_i64(block_ids, "block_ids")
    if any(m.dtype != key_scale.dtype for m in metas):
        raise RuntimeError("KIVI metadata tensors must have the same dtype")
    if key_scale.dtype not in (torch.float16, torch.float32):
        raise RuntimeError("KIVI metadata tensors must be float16 or float32")
    _check_bits(bits)
    if group_size <= 0:
        raise RuntimeError("KIVI group_size must be positive")
    if sink_tokens < 0 or sink_tokens > tokens:
        raise RuntimeError("KIVI sink_tokens must be in [0, tokens]")
    if tokens <= 0 or heads <= 0 or head_dim <= 0:
        raise RuntimeError("tokens, heads, and head_dim must be positive")
    if key_offset < 0 or key_bytes < 0 or value_offset < 0 or value_bytes < 0:
        raise RuntimeError("invalid KIVI stream offsets")
    if key_offset + key_bytes > bytestream.numel() or value_offset + value_bytes > bytestream.numel():
        raise RuntimeError("KIVI stream ranges exceed bytestream length")
    body = tokens - sink_tokens
    channels = heads * head_dim
    key_groups = (body + group_size - 1) // group_size
    value_groups = (channels + group_size - 1) // group_size
    if key_scale.numel() < key_groups * channels or key_zero.numel() < key_groups * channels:
        raise RuntimeError("KIVI key metadata is too small")
    if value_scale.numel() < body * value_groups or value_zero.numel() < body * value_groups:
        raise RuntimeError("KIVI value metadata is too small")
    if key_sink.numel() < sink_tokens * channels or value_sink.numel() < sink_tokens * channels:
        raise RuntimeError("KIVI sink metadata is too small")
    kv = _paged(kv_cache, heads, head_dim)
    _blocks(kv_cache, block_ids, tokens)
    import ctypes

    numel = (ctypes.c_int64 * 6)(*[m.numel() for m in metas])
    device = kv_cache.device
    with torch.cuda.device(device):
        rc = _lib.lib().origami_kivi_dequantize_to_kv_cache(
            bytestream.data_ptr(), bytestream.numel(), int(key_offset), int(key_bytes), int(value_offset),
            int(value_bytes), int(bits), int(group_size), int(sink_tokens), *[m.data_ptr() for m in metas],
            ctypes.cast(numel, ctypes.c_void_p), _DTYPE[key_scale.dtype], kv, _DTYPE[kv_cache.dtype],
            block_ids.data_ptr(), block_ids.numel(), int(tokens), _err_ptr(error_count),
            torch.cuda.current_stream(device).cuda_stream)
    _lib.check(rc, "origami_kivi_dequantize_to_kv_cache")
