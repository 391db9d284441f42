"""ctypes binding of liborigami_b200.so (declarations: include/origami_b200.h).

The library is the only compute path of this package: when it is missing or cannot be
loaded every op raises, there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "liborigami_b200.so"

ORIGAMI_OK = 0
ORIGAMI_KV_FIRST = 0
ORIGAMI_BLOCKS_FIRST = 1
MAX_PLANES = 8

_c_i64p = ctypes.POINTER(ctypes.c_int64)
_vp = ctypes.c_void_p


class PagedKV(ctypes.Structure):
    _fields_ = [
        ("d_data", _vp),
        ("layout", ctypes.c_int32),
        ("elem_bytes", ctypes.c_int32),
        ("num_blocks", ctypes.c_int64),
        ("block_size", ctypes.c_int64),
        ("num_heads", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
    ]


class Planes(ctypes.Structure):
    _fields_ = [
        ("num_planes", ctypes.c_int32),
        ("shift", ctypes.c_int32 * MAX_PLANES),
        ("bits", ctypes.c_int32 * MAX_PLANES),
    ]


class ChunkTable(ctypes.Structure):
    _fields_ = [
        ("d_specs", _vp),
        ("d_offsets", _vp),
        ("h_specs", _vp),
        ("h_offsets", _vp),
        ("num_specs", ctypes.c_int64),
    ]


class LayerJob(ctypes.Structure):
    _fields_ = [
        ("d_kv_cache", _vp),
        ("d_block_ids", _vp),
        ("num_block_ids", ctypes.c_int64),
    ]


class OrigamiError(RuntimeError):
    """A liborigami_b200 entry point returned an error status."""


_lock = threading.Lock()
_lib = None


def _declare(L: ctypes.CDLL) -> None:
    i32, i64 = ctypes.c_int32, ctypes.c_int64
    L.origami_b200_version.restype = i32
    L.origami_last_error.restype = ctypes.c_char_p
    L.origami_packed_bytes.restype = i64
    L.origami_packed_bytes.argtypes = [i64, i32]
    canon = [_vp, i64, _vp, _vp, _vp, _vp, _vp, _vp, i64, _vp, i32, _vp, i64, i64, i64, _vp, i64, _vp]
    L.origami_unpack_canonical_storage_chunks.argtypes = canon
    L.origami_unpack_canonical_storage_chunks.restype = i32
    L.origami_pack_canonical_storage_chunks.argtypes = canon
    L.origami_pack_canonical_storage_chunks.restype = i32
    P = ctypes.POINTER
    L.origami_pack_layer_from_paged.argtypes = [P(PagedKV), _vp, i64, i64, P(Planes), P(ChunkTable), _vp, i64, _vp, _vp]
    L.origami_pack_layer_from_paged.restype = i32
    L.origami_restore_layer_to_paged.argtypes = [_vp, i64, P(Planes), P(ChunkTable), P(PagedKV), _vp, i64, i64, _vp, _vp]
    L.origami_restore_layer_to_paged.restype = i32
    L.origami_restore_layer_prefix_to_paged.argtypes = [_vp, i64, P(Planes), P(ChunkTable), P(PagedKV), _vp, i64,
                                                        i64, i64, _vp, _vp]
    L.origami_restore_layer_prefix_to_paged.restype = i32
    L.origami_restore_layers_to_paged.argtypes = [_vp, i64, i64, P(Planes), P(ChunkTable), P(PagedKV), P(LayerJob),
                                                  i32, i64, _vp, _vp]
    L.origami_restore_layers_to_paged.restype = i32
    L.origami_pack_layers_from_paged.argtypes = [P(PagedKV), P(LayerJob), i32, i64, P(Planes), P(ChunkTable), _vp,
                                                 i64, i64, _vp, _vp]
    L.origami_pack_layers_from_paged.restype = i32
    L.origami_gather_blocks.argtypes = [P(PagedKV), _vp, i64, _vp, i64, _vp, _vp]
    L.origami_gather_blocks.restype = i32
    L.origami_scatter_blocks.argtypes = [_vp, i64, P(PagedKV), _vp, i64, _vp, _vp]
    L.origami_scatter_blocks.restype = i32
    L.origami_cachegen_unpack_dequantize_to_kv_cache.argtypes = [
        _vp, i64, i64, i64, i64, i64, i64, i64, i64, i64, _vp, i64, _vp, i64, i32, P(PagedKV), i32, _vp, i64, i64,
        _vp, _vp]
    L.origami_cachegen_unpack_dequantize_to_kv_cache.restype = i32
    L.origami_cachegen_unpack_dequantize.argtypes = [
        _vp, i64, _vp, _vp, i64, _vp, _vp, i64, _vp, i64, _vp, i64, _vp, i64, _vp, i64, i32, i64, i64, i64, _vp, i64,
        _vp]
    L.origami_cachegen_unpack_dequantize.restype = i32
    L.origami_kivi_dequantize_to_kv_cache.argtypes = [
        _vp, i64, i64, i64, i64, i64, i64, i64, i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, i32, P(PagedKV), i32, _vp,
        i64, i64, _vp, _vp]
    L.origami_kivi_dequantize_to_kv_cache.restype = i32
    L.origami_fused_prefix_attention.argtypes = [
        _vp, i64, i64, i64, i64, i64, i64, i64, i64, i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, i32, _vp, i32, i64, i64,
        i64, P(PagedKV), i32, _vp, i64, i64, i64, i64, ctypes.c_double, _vp, _vp, i64, _vp, _vp]
    L.origami_fused_prefix_attention.restype = i32
    L.origami_fused_prefix_attention_workspace.argtypes = [i64, i64, i64, i64, i64, _vp]
    L.origami_fused_prefix_attention_workspace.restype = i32
    L.origami_fused_prefix_attention_noalloc.argtypes = [
        _vp, i64, i64, i64, i64, i64, i64, i64, i64, i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, i32, _vp, i32, i64, i64,
        i64, P(PagedKV), i32, _vp, i64, i64, i64, i64, ctypes.c_double, _vp, _vp, _vp]
    L.origami_fused_prefix_attention_noalloc.restype = i32
    L.origami_selftest_wait_timeout.argtypes = [_vp, i32, _vp]
    L.origami_selftest_wait_timeout.restype = i32
    L.origami_origqz1_parse.argtypes = [_vp, i64, _vp, i64, _vp, _vp, _vp, _vp]
    L.origami_origqz1_parse.restype = i32
    L.origami_deflate_bound.argtypes = [i64]
    L.origami_deflate_bound.restype = i64
    L.origami_deflate_chunks.argtypes = [_vp, _vp, _vp, i64, i32, _vp, i64, _vp, _vp, i32]
    L.origami_deflate_chunks.restype = i32
    L.origami_inflate_chunks.argtypes = [_vp, _vp, _vp, i64, _vp, i64, _vp, _vp, i32]
    L.origami_inflate_chunks.restype = i32


def lib() -> ctypes.CDLL:
    """Load the CUDA library; raise loudly when it is absent."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise OrigamiError(
                        f"{LIB_PATH.name} is not built; run `python -m origami_b200.build` "
                        "(origami_b200 has no CPU fallback)"
                    )
                L = ctypes.CDLL(str(LIB_PATH))
                _declare(L)
                _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != ORIGAMI_OK:
        msg = lib().origami_last_error().decode(errors="replace")
        raise OrigamiError(f"{what} failed ({rc}): {msg}")


EXPORTS = (
    "origami_b200_version",
    "origami_last_error",
    "origami_packed_bytes",
    "origami_unpack_canonical_storage_chunks",
    "origami_pack_canonical_storage_chunks",
    "origami_pack_layer_from_paged",
    "origami_restore_layer_to_paged",
    "origami_restore_layer_prefix_to_paged",
    "origami_restore_layers_to_paged",
    "origami_pack_layers_from_paged",
    "origami_gather_blocks",
    "origami_scatter_blocks",
    "origami_cachegen_unpack_dequantize_to_kv_cache",
    "origami_cachegen_unpack_dequantize",
    "origami_kivi_dequantize_to_kv_cache",
    "origami_fused_prefix_attention",
    "origami_fused_prefix_attention_workspace",
    "origami_fused_prefix_attention_noalloc",
    "origami_origqz1_parse",
    "origami_deflate_bound",
    "origami_deflate_chunks",
    "origami_inflate_chunks",
    "origami_selftest_wait_timeout",
)

ORIGAMI_DTYPE_F16 = 1
ORIGAMI_DTYPE_BF16 = 2
ORIGAMI_DTYPE_F32 = 3
