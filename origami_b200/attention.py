"""Fused attention over a quantized prefix and a paged suffix, served by liborigami_b200.so
(kernel: csrc/attention_kernels.cuh, tcgen05 tensor cores).

``fused_prefix_attention_cuda`` keeps the positional signature, the checks (in the same
order) and the messages of the reference export (bitpack_layout_cuda.cpp:716-890), raised
as RuntimeError. The output matches the reference kernel within the reference test's
tolerance (test_origami_fused_attention.py:123: 1.5e-2 for fp16, 3e-2 for bf16): keys and
values are dequantized in fp32 exactly as the reference does, then rounded to the query
type for the tensor cores, and the probabilities are rounded to the query type for the
P.V product; accumulation is fp32. Work goes to the current stream of the query's device.

Two keyword arguments have no reference counterpart: ``workspace`` (uint8 CUDA tensor of at
least ``workspace_bytes(...)`` bytes, zero before its first use and left zero by the
kernel; allocated zeroed per call when omitted) and ``error_flags`` (int32 CUDA tensor; bit
31 is set if a bounded wait inside the kernel ran out).
"""
from __future__ import annotations

import ctypes

import torch

from origami_b200 import _lib
from origami_b200.quant import _check_cuda_contiguous

_QDTYPE = {torch.float16: _lib.ORIGAMI_DTYPE_F16, torch.bfloat16: _lib.ORIGAMI_DTYPE_BF16}


def workspace_bytes(query_tokens: int, query_heads: int, kv_heads: int, query_start_position: int,
                    sequence_length: int, device: torch.device | None = None) -> int:
    """Workspace the kernel needs for these shapes on `device` (0 when unsplit)."""
    out = ctypes.c_int64(0)
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        rc = _lib.lib().origami_fused_prefix_attention_workspace(int(query_tokens), int(query_heads), int(kv_heads),
                                                                 int(query_start_position), int(sequence_length),
                                                                 ctypes.byref(out))
    _lib.check(rc, "origami_fused_prefix_attention_workspace")
    return int(out.value)


def _paged(kv_cache: torch.Tensor) -> _lib.PagedKV:
    """cpp:793-818: the FlashAttention layout [2, blocks, ...] is tried before
    [blocks, 2, ...] (the reverse of the dequantize-to-cache ops); an unknown layout is
    passed on for the library to report in the reference's check order."""
    if kv_cache.size(0) == 2:
        layout, nb = _lib.ORIGAMI_KV_FIRST, kv_cache.size(1)
    elif kv_cache.size(1) == 2:
        layout, nb = _lib.ORIGAMI_BLOCKS_FIRST, kv_cache.size(0)
    else:
        layout, nb = -1, 0
    return _lib.PagedKV(kv_cache.data_ptr(), layout, 2, int(nb), int(kv_cache.size(2)), int(kv_cache.size(3)),
                        int(kv_cache.size(4)))


def fused_prefix_attention_cuda(bytestream: torch.Tensor, key_offset: int, key_bytes: int, value_offset: int,
                                value_bytes: int, codec: int, bits: int, group_size: int, sink_tokens: int,
                                key_scale: torch.Tensor, key_zero: torch.Tensor, value_scale: torch.Tensor,
                                value_zero: torch.Tensor, key_sink: torch.Tensor, value_sink: torch.Tensor,
                                query: torch.Tensor, kv_cache: torch.Tensor, block_table: torch.Tensor,
                                prefix_tokens: int, query_start_position: int, sequence_length: int,
                                softmax_scale: float, output: torch.Tensor, *,
                                workspace: torch.Tensor | None = None,
                                error_flags: torch.Tensor | None = None) -> None:
    for t, name in ((bytestream, "bytestream"), (key_scale, "key_scale"), (key_zero, "key_zero"),
                    (value_scale, "value_scale"), (value_zero, "value_zero"), (key_sink, "key_sink"),
                    (value_sink, "value_sink"), (query, "query"), (kv_cache, "kv_cache"),
                    (block_table, "block_table"), (output, "output")):
        _check_cuda_contiguous(t, name)
    if bytestream.dtype != torch.uint8:
        raise RuntimeError("bytestream must be uint8")
    if query.dim() != 3:
        raise RuntimeError("query must have shape [query_tokens, query_heads, head_dim]")
    if output.shape != query.shape:
        raise RuntimeError("output must have the same shape as query")
    if query.dtype not in _QDTYPE:
        raise RuntimeError("query must be float16 or bfloat16")
    if output.dtype != query.dtype:
        raise RuntimeError("output dtype must match query dtype")
    if kv_cache.dtype not in _QDTYPE:
        raise RuntimeError("kv_cache must be float16 or bfloat16")
    if block_table.dtype != torch.int32:
        raise RuntimeError("block_table must be int32")
    if block_table.dim() != 1:
        raise RuntimeError("block_table must be one-dimensional")
    if kv_cache.dim() != 5:
        raise RuntimeError("kv_cache must have rank 5")
    device = bytestream.device
    for t in (key_scale, key_zero, value_scale, value_zero, key_sink, value_sink, query, kv_cache, block_table, output):
        if t.device != device:
            raise RuntimeError("all fused-attention tensors must be on the same CUDA device")
    for t in (key_scale, key_zero, value_scale, value_zero, key_sink, value_sink):
        if t.dtype != torch.float16:
            raise RuntimeError("compressed metadata tensors must be float16")
    qt, qh, hd = (int(x) for x in query.shape)
    paged = _paged(kv_cache)
    kv_heads = int(kv_cache.size(3))
    with torch.cuda.device(device):
        need = 0
        if paged.layout >= 0 and hd == 128 and qt > 0 and qh > 0 and kv_heads > 0 and qh % kv_heads == 0 and \
                prefix_tokens <= query_start_position and query_start_position + qt <= sequence_length:
            need = workspace_bytes(qt, qh, kv_heads, query_start_position, sequence_length, device)
        if need > 0 and workspace is None:
            workspace = torch.zeros(need, dtype=torch.uint8, device=device)
        if workspace is not None and (not workspace.is_cuda or workspace.dtype != torch.uint8):
            raise RuntimeError("workspace must be a CUDA uint8 tensor")
        if error_flags is not None and (not error_flags.is_cuda or error_flags.dtype not in (torch.int32, torch.uint32)):
            raise RuntimeError("error_flags must be a CUDA int32 tensor")
        numel = (ctypes.c_int64 * 6)(*[int(t.numel()) for t in (key_scale, key_zero, value_scale, value_zero,
                                                               key_sink, value_sink)])
        rc = _lib.lib().origami_fused_prefix_attention(
            bytestream.data_ptr(), bytestream.numel(), int(key_offset), int(key_bytes), int(value_offset),
            int(value_bytes), int(codec), int(bits), int(group_size), int(sink_tokens), key_scale.data_ptr(),
            key_zero.data_ptr(), value_scale.data_ptr(), value_zero.data_ptr(), key_sink.data_ptr(),
            value_sink.data_ptr(), numel, _lib.ORIGAMI_DTYPE_F16, query.data_ptr(), _QDTYPE[query.dtype], qt, qh, hd,
            ctypes.byref(paged), _QDTYPE[kv_cache.dtype], block_table.data_ptr(), block_table.numel(),
            int(prefix_tokens), int(query_start_position), int(sequence_length), float(softmax_scale),
            output.data_ptr(), workspace.data_ptr() if workspace is not None else None,
            workspace.numel() if workspace is not None else 0,
            error_flags.data_ptr() if error_flags is not None else None,
            torch.cuda.current_stream(device).cuda_stream)
    _lib.check(rc, "origami_fused_prefix_attention")
