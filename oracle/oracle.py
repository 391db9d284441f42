"""TEST INFRASTRUCTURE ONLY — numpy front end of the CPU oracle (oracle.c).

Used by tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg as the
parity checker. The product (``origami_b200``) never imports this module.

Also holds a pure-Python restatement of the reference symbol reader
(``csrc/origami/bitpack_layout_cuda.cu:70-89``) for tiny cross-checks of the C code.
"""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
from pathlib import Path
from typing import Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liborigami_oracle.so"

_I64P = ctypes.POINTER(ctypes.c_int64)
_I32P = ctypes.POINTER(ctypes.c_int32)
_U8P = ctypes.POINTER(ctypes.c_uint8)
_U16P = ctypes.POINTER(ctypes.c_uint16)
_lib = None


def build() -> Path:
    """Compile oracle.c into _build/ (gcc with OpenMP)."""
    cc = shutil.which("gcc-13") or shutil.which("gcc") or "cc"
    LIB_PATH.parent.mkdir(parents=True, exist_ok=True)
    cmd = [cc, "-O2", "-fopenmp", "-fPIC", "-std=c11", "-ffp-contract=off", "-shared", "-o", str(LIB_PATH),
           str(HERE / "oracle.c"), "-lm"]
    subprocess.run(cmd, check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (HERE / "oracle.c").stat().st_mtime:
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.oracle_set_threads.argtypes = [ctypes.c_int]
        L.oracle_max_threads.restype = ctypes.c_int
        L.oracle_unpack_canonical.argtypes = [_U8P, _I64P, _I64P, _I64P, ctypes.c_int64, _I64P, ctypes.c_int, _I64P, _U8P]
        L.oracle_pack_canonical.argtypes = [_U8P, _I64P, _I64P, _I64P, ctypes.c_int64, _I64P, ctypes.c_int, _I64P, _U8P]
        geom = [ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]
        L.oracle_gather_blocks.argtypes = [_U8P] + geom + [ctypes.c_int, _I64P, ctypes.c_int64, _U8P]
        L.oracle_scatter_blocks.argtypes = [_U8P] + geom + [ctypes.c_int, _I64P, ctypes.c_int64, _U8P]
        L.oracle_pack_layer.argtypes = [_U16P] + geom + [_I64P, ctypes.c_int64, ctypes.c_int, _I32P, _I32P, _I64P,
                                                         ctypes.c_int64, _I64P, _U8P]
        L.oracle_restore_layer.argtypes = [_U8P, ctypes.c_int, _I32P, _I32P, _I64P, ctypes.c_int64, _I64P, _U16P] + geom + [
            _I64P, ctypes.c_int64]
        vp, i64, i = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.oracle_cachegen_to_cache.restype = i64
        L.oracle_cachegen_to_cache.argtypes = [vp, i64, i64, i64, i64, i64, i, i, i64, i64, vp, vp, i, vp, i, i, i64,
                                               vp, i64, i64, i64, i64, i64]
        L.oracle_cachegen_unpack.argtypes = [vp, i64, vp, vp, vp, vp, vp, vp, i, vp, i64, i64, i64, i64]
        L.oracle_kivi_to_cache.restype = i64
        L.oracle_kivi_to_cache.argtypes = [vp, i64, i64, i64, i64, i64, i, i64, i64, vp, vp, vp, vp, vp, vp, i, vp, i,
                                           i, i64, vp, i64, i64, i64, i64, i64]
        L.oracle_fused_prefix_attention.argtypes = [vp, i64, i64, i64, i64, i, i, i64, i64, vp, vp, vp, vp, vp, vp,
                                                    vp, i, vp, i, i, i64, i64, i64, vp, i64, i64, i64, i64, i64,
                                                    ctypes.c_float, vp]
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def _i64(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.int64))


AXIS_NAMES = {"token": 0, "head": 1, "head_dim": 2, "layer": 3}


def axis_positions(layout: Sequence[str]) -> list[int]:
    """[token, head, head_dim, layer or -1] positions (lossless/native_cpu.py:123-130)."""
    lay = list(layout)
    return [lay.index("token"), lay.index("head"), lay.index("head_dim"),
            lay.index("layer") if "layer" in lay else -1]


def packed_bytes(symbols: int, bits: int) -> int:
    return (int(symbols) * int(bits) + 7) // 8


def spec_symbols(spec: Sequence[int]) -> int:
    h0, h1, c0, c1, t0, t1 = (int(v) for v in spec)
    return (h1 - h0) * (c1 - c0) * (t1 - t0)


def chunk_offsets(specs: np.ndarray, bits: Sequence[int]) -> np.ndarray:
    sizes = [packed_bytes(spec_symbols(s), b) for s, b in zip(specs, bits)]
    return _i64(np.concatenate([[0], np.cumsum(sizes, dtype=np.int64)]))


# --------------------------------------------------------------------------------------
# canonical ops
# --------------------------------------------------------------------------------------
def unpack_canonical(flat: np.ndarray, offsets, bits, specs, shape, layout) -> np.ndarray:
    flat = np.ascontiguousarray(flat, dtype=np.uint8)
    offsets, bits, specs = _i64(offsets), _i64(bits), _i64(specs).reshape(-1, 6)
    shape_a = _i64(shape)
    axes = _i64(axis_positions(layout))
    out = np.empty(int(np.prod(shape_a)), dtype=np.uint8)
    lib().oracle_unpack_canonical(_p(flat, _U8P), _p(offsets, _I64P), _p(bits, _I64P), _p(specs, _I64P), len(specs),
                                  _p(shape_a, _I64P), len(shape_a), _p(axes, _I64P), _p(out, _U8P))
    return out


def pack_canonical(symbols: np.ndarray, bits, specs, shape, layout) -> tuple[np.ndarray, np.ndarray]:
    """Returns (flat chunk bytes, offsets[num_chunks + 1])."""
    symbols = np.ascontiguousarray(symbols, dtype=np.uint8).reshape(-1)
    specs = _i64(specs).reshape(-1, 6)
    bits = _i64([bits] * len(specs) if np.isscalar(bits) else bits)
    offsets = chunk_offsets(specs, bits)
    shape_a = _i64(shape)
    axes = _i64(axis_positions(layout))
    flat = np.zeros(int(offsets[-1]), dtype=np.uint8)
    lib().oracle_pack_canonical(_p(symbols, _U8P), _p(offsets, _I64P), _p(bits, _I64P), _p(specs, _I64P), len(specs),
                                _p(shape_a, _I64P), len(shape_a), _p(axes, _I64P), _p(flat, _U8P))
    return flat, offsets


# --------------------------------------------------------------------------------------
# paged cache ops; cache arrays are uint16 views [2, NB, bs, H, D] (layout 0) or
# [NB, 2, bs, H, D] (layout 1)
# --------------------------------------------------------------------------------------
def _geom(cache: np.ndarray, layout: int):
    if layout == 0:
        _, NB, bs, H, D = cache.shape
    else:
        NB, _, bs, H, D = cache.shape
    return int(NB), int(bs), int(H), int(D)


def gather_blocks(cache: np.ndarray, layout: int, ids) -> np.ndarray:
    cache = np.ascontiguousarray(cache)
    NB, bs, H, D = _geom(cache, layout)
    ids = _i64(ids)
    shape = (2, len(ids), bs, H, D) if layout == 0 else (len(ids), 2, bs, H, D)
    out = np.empty(shape, dtype=cache.dtype)
    rc = lib().oracle_gather_blocks(_p(cache.view(np.uint8), _U8P), layout, NB, bs, H, D, cache.itemsize,
                                    _p(ids, _I64P), len(ids), _p(out.view(np.uint8), _U8P))
    if rc != 0:
        raise ValueError("block id out of range")
    return out


def scatter_blocks(value: np.ndarray, cache: np.ndarray, layout: int, ids) -> None:
    assert cache.flags.c_contiguous
    value = np.ascontiguousarray(value, dtype=cache.dtype)
    NB, bs, H, D = _geom(cache, layout)
    ids = _i64(ids)
    rc = lib().oracle_scatter_blocks(_p(value.view(np.uint8), _U8P), layout, NB, bs, H, D, cache.itemsize,
                                     _p(ids, _I64P), len(ids), _p(cache.view(np.uint8), _U8P))
    if rc != 0:
        raise ValueError("block id out of range")


def layer_offsets(specs, plane_bits: Sequence[int]) -> np.ndarray:
    specs = _i64(specs).reshape(-1, 6)
    bits = []
    for _kv in range(2):
        for b in plane_bits:
            bits.extend([int(b)] * len(specs))
    all_specs = np.concatenate([specs] * (2 * len(plane_bits)))
    return chunk_offsets(all_specs, bits)


def pack_layer(cache: np.ndarray, layout: int, ids, num_tokens: int, shifts, bits, specs) -> tuple[np.ndarray, np.ndarray]:
    cache = np.ascontiguousarray(cache, dtype=np.uint16)
    NB, bs, H, D = _geom(cache, layout)
    ids = _i64(ids)
    specs = _i64(specs).reshape(-1, 6)
    offsets = layer_offsets(specs, bits)
    sh = np.ascontiguousarray(shifts, dtype=np.int32)
    bi = np.ascontiguousarray(bits, dtype=np.int32)
    packed = np.zeros(int(offsets[-1]), dtype=np.uint8)
    rc = lib().oracle_pack_layer(_p(cache, _U16P), layout, NB, bs, H, D, _p(ids, _I64P), int(num_tokens), len(bi),
                                 _p(sh, _I32P), _p(bi, _I32P), _p(specs, _I64P), len(specs), _p(offsets, _I64P),
                                 _p(packed, _U8P))
    if rc != 0:
        raise ValueError("oracle_pack_layer failed")
    return packed, offsets


def restore_layer(packed: np.ndarray, shifts, bits, specs, cache: np.ndarray, layout: int, ids, num_tokens: int) -> None:
    assert cache.flags.c_contiguous and cache.dtype == np.uint16
    NB, bs, H, D = _geom(cache, layout)
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    specs = _i64(specs).reshape(-1, 6)
    offsets = layer_offsets(specs, bits)
    sh = np.ascontiguousarray(shifts, dtype=np.int32)
    bi = np.ascontiguousarray(bits, dtype=np.int32)
    ids = _i64(ids)
    rc = lib().oracle_restore_layer(_p(packed, _U8P), len(bi), _p(sh, _I32P), _p(bi, _I32P), _p(specs, _I64P),
                                    len(specs), _p(offsets, _I64P), _p(cache, _U16P), layout, NB, bs, H, D,
                                    _p(ids, _I64P), int(num_tokens))
    if rc != 0:
        raise ValueError("oracle_restore_layer failed")


# --------------------------------------------------------------------------------------
# pure-Python restatement for tiny cross-checks (bitpack_layout_cuda.cu:70-128)
# --------------------------------------------------------------------------------------
def unpack_symbol_py(src: bytes, symbol_index: int, bits: int) -> int:
    if bits == 8:
        return src[symbol_index]
    bit_pos = symbol_index * bits
    byte_idx, shift = bit_pos >> 3, bit_pos & 7
    packed = src[byte_idx] if byte_idx < len(src) else 0
    if byte_idx + 1 < len(src):
        packed |= src[byte_idx + 1] << 8
    return (packed >> shift) & ((1 << bits) - 1)


def unpack_canonical_py(flat: bytes, offsets, bits, specs, shape, layout) -> np.ndarray:
    shape = [int(s) for s in shape]
    out = np.zeros(shape, dtype=np.uint8)
    axes = axis_positions(layout)
    for k, spec in enumerate(specs):
        h0, h1, c0, c1, t0, t1 = (int(v) for v in spec)
        src = bytes(flat[int(offsets[k]):int(offsets[k + 1])])
        local = 0
        for h in range(h0, h1):
            for c in range(c0, c1):
                for t in range(t0, t1):
                    coord = [0] * len(shape)
                    coord[axes[0]], coord[axes[1]], coord[axes[2]] = t, h, c
                    out[tuple(coord)] = unpack_symbol_py(src, local, int(bits[k]))
                    local += 1
    return out.reshape(-1)


if os.environ.get("ORIGAMI_ORACLE_THREADS"):
    set_threads(int(os.environ["ORIGAMI_ORACLE_THREADS"]))


# ---------------------------------------------------------------------------------------
# Quantized restore paths (restatements of bitpack_layout_cuda.cu:141-185, 348-423,
# 577-683). Float tensors are numpy float16 / float32 arrays; caches are uint16 arrays
# holding fp16 or bf16 bit patterns, [num_blocks, 2, bs, H, D] (blocks_first) or
# [2, num_blocks, bs, H, D].
# ---------------------------------------------------------------------------------------
def _meta(a: np.ndarray) -> tuple[np.ndarray, int]:
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        return a, 1
    if a.dtype == np.float32:
        return a, 0
    raise TypeError("metadata must be float16 or float32")


def _cache_geom(cache: np.ndarray, blocks_first: bool):
    assert cache.dtype == np.uint16 and cache.ndim == 5 and cache.flags["C_CONTIGUOUS"]
    nb = cache.shape[0] if blocks_first else cache.shape[1]
    return nb, cache.shape[2], cache.shape[3], cache.shape[4]


def cachegen_to_cache(bytestream, key_offset, key_bytes, value_offset, value_bytes, key_bits, value_bits, key_bins,
                      value_bins, max_key, max_value, cache: np.ndarray, blocks_first: bool, block_ids, tokens: int,
                      out_is_bf16: bool) -> int:
    """Writes `cache` in place; returns the (kv, token, head) rows skipped for bad ids."""
    bs_ = np.ascontiguousarray(bytestream, dtype=np.uint8)
    mk, mh = _meta(max_key)
    mv, mh2 = _meta(max_value)
    assert mh == mh2
    ids = _i64(block_ids)
    nb, bsz, H, D = _cache_geom(cache, blocks_first)
    return int(lib().oracle_cachegen_to_cache(
        bs_.ctypes.data, len(bs_), key_offset, key_bytes, value_offset, value_bytes, key_bits, value_bits, key_bins, value_bins,
        mk.ctypes.data, mv.ctypes.data, mh, cache.ctypes.data, int(out_is_bf16), int(blocks_first), nb,
        ids.ctypes.data, len(ids), bsz, tokens, H, D))


def cachegen_unpack(bytestream, offsets, bits, key_bins, value_bins, max_key, max_value, tokens: int, heads: int,
                    head_dim: int) -> np.ndarray:
    """fp16 bit patterns [layers, 2, heads, tokens, head_dim]."""
    bs_ = np.ascontiguousarray(bytestream, dtype=np.uint8)
    off, b, kb, vb = _i64(offsets), _i64(bits), _i64(key_bins), _i64(value_bins)
    mk, mh = _meta(max_key)
    mv, _ = _meta(max_value)
    layers = len(b) // 2
    out = np.zeros((layers, 2, heads, tokens, head_dim), dtype=np.uint16)
    lib().oracle_cachegen_unpack(bs_.ctypes.data, len(bs_), off.ctypes.data, b.ctypes.data, kb.ctypes.data, vb.ctypes.data,
                                 mk.ctypes.data, mv.ctypes.data, mh, out.ctypes.data, layers, tokens, heads, head_dim)
    return out


def kivi_to_cache(bytestream, key_offset, key_bytes, value_offset, value_bytes, bits, group_size, sink_tokens,
                  key_scale, key_zero, value_scale, value_zero, key_sink, value_sink, cache: np.ndarray,
                  blocks_first: bool, block_ids, tokens: int, out_is_bf16: bool) -> int:
    """Writes `cache` in place; returns the (kv, token, head) rows skipped for bad ids."""
    bs_ = np.ascontiguousarray(bytestream, dtype=np.uint8)
    metas = [_meta(m) for m in (key_scale, key_zero, value_scale, value_zero, key_sink, value_sink)]
    half = metas[0][1]
    assert all(m[1] == half for m in metas)
    ids = _i64(block_ids)
    nb, bsz, H, D = _cache_geom(cache, blocks_first)
    return int(lib().oracle_kivi_to_cache(
        bs_.ctypes.data, len(bs_), key_offset, key_bytes, value_offset, value_bytes, bits, group_size, sink_tokens,
        *[m[0].ctypes.data for m in metas], half, cache.ctypes.data, int(out_is_bf16), int(blocks_first), nb,
        ids.ctypes.data, len(ids), bsz, tokens, H, D))


def fused_prefix_attention(bytestream, key_offset, key_bytes, value_offset, value_bytes, codec, bits, group_size,
                           sink_tokens, key_scale, key_zero, value_scale, value_zero, key_sink, value_sink,
                           query: np.ndarray, query_bf16: bool, kv_cache: np.ndarray, cache_bf16: bool,
                           blocks_first: bool, block_table, prefix_tokens: int, query_start: int, sequence_length: int,
                           softmax_scale: float) -> np.ndarray:
    """The reference fused prefix attention (cu:873-1091) on the CPU: query and kv_cache
    hold fp16 / bf16 bit patterns (uint16), metadata is float16; returns the output bit
    patterns, shaped like query."""
    bs_ = np.ascontiguousarray(bytestream, dtype=np.uint8)
    metas = [np.ascontiguousarray(m, dtype=np.float16) for m in (key_scale, key_zero, value_scale, value_zero,
                                                                 key_sink, value_sink)]
    q = np.ascontiguousarray(query, dtype=np.uint16)
    cache = np.ascontiguousarray(kv_cache, dtype=np.uint16)
    table = np.ascontiguousarray(block_table, dtype=np.int32)
    nb, bsz, H, D = _cache_geom(cache, blocks_first)
    assert D == 128 and q.ndim == 3 and q.shape[2] == 128
    out = np.zeros_like(q)
    lib().oracle_fused_prefix_attention(
        bs_.ctypes.data, key_offset, key_bytes, value_offset, value_bytes, int(codec), int(bits), group_size,
        sink_tokens, *[m.ctypes.data for m in metas], q.ctypes.data, int(query_bf16), cache.ctypes.data,
        int(cache_bf16), int(blocks_first), nb, bsz, H, table.ctypes.data, prefix_tokens, query_start,
        sequence_length, q.shape[0], q.shape[1], float(softmax_scale), out.ctypes.data)
    return out
