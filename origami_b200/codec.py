"""Host codec of the save / restore path, on liborigami_b200.so (csrc/host_codec.cpp).

* ``deflate_chunks`` / ``inflate_chunks``: the reference CPU codec's zlib raw deflate
  (level 1, window bits -15; lossless/cpu_qat.py:64-84) over many chunks at once, on all
  host threads, reading and writing caller buffers in place. Inflate writes each chunk at
  its own offset of one (pinned) buffer, the restore pipeline's staging, so nothing is
  concatenated or bounced through pageable memory on the way to the GPU.
* ``parse_origqz1``: the ORIGQZ1 bundle header (the reference's qat_bundle.dz) with the
  reference parser's checks (qat_deflate.cpp:1804-1860).

The ctypes calls release the GIL, so the codec runs beside Python threads.
"""
from __future__ import annotations

import ctypes
from typing import Any

import numpy as np
import torch

from origami_b200 import _lib


class DzRecord(ctypes.Structure):
    _fields_ = [("raw_len", ctypes.c_uint32), ("comp_len", ctypes.c_uint32), ("comp_offset", ctypes.c_int64),
                ("output_offset", ctypes.c_int64)]


DZ_DTYPE = np.dtype([("raw_len", "<u4"), ("comp_len", "<u4"), ("comp_offset", "<i8"), ("output_offset", "<i8")])


def _buffer(x: Any, writable: bool = False) -> tuple[int, int, Any]:
    """(address, byte length, keep-alive) of a host byte buffer: a CPU tensor, a numpy
    array, bytes / bytearray / memoryview."""
    if isinstance(x, torch.Tensor):
        if x.device.type != "cpu" or not x.is_contiguous():
            raise ValueError("host codec buffers must be contiguous CPU tensors")
        return x.data_ptr(), x.numel() * x.element_size(), x
    if isinstance(x, np.ndarray):
        if not x.flags["C_CONTIGUOUS"] or (writable and not x.flags["WRITEABLE"]):
            raise ValueError("host codec buffers must be contiguous (and writable for outputs)")
        return x.ctypes.data, x.nbytes, x
    a = np.frombuffer(x, dtype=np.uint8)
    if writable and not a.flags["WRITEABLE"]:
        raise ValueError("output buffer is read-only")
    return a.ctypes.data, a.nbytes, a


def _i64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


def deflate_bound(n: int) -> int:
    return int(_lib.lib().origami_deflate_bound(int(n)))


def deflate_chunks(data, offsets, lengths, *, level: int = 1, threads: int = 0):
    """Compress chunks data[offsets[i], +lengths[i]); returns (buffer, comp_offsets,
    comp_lengths): chunk i's stream is buffer[comp_offsets[i], +comp_lengths[i])."""
    off, ln = _i64(offsets), _i64(lengths)
    L = _lib.lib()
    slots = np.asarray([deflate_bound(int(n)) for n in ln], dtype=np.int64)
    dst_off = np.zeros(len(ln), dtype=np.int64)
    if len(ln):
        dst_off[1:] = np.cumsum(slots)[:-1]
    out = np.empty(int(slots.sum()), dtype=np.uint8)
    comp = np.zeros(len(ln), dtype=np.int64)
    src_ptr, _, keep = _buffer(data)
    rc = L.origami_deflate_chunks(src_ptr, off.ctypes.data, ln.ctypes.data, len(ln), int(level), out.ctypes.data,
                                  out.nbytes, dst_off.ctypes.data, comp.ctypes.data, int(threads))
    del keep
    _lib.check(rc, "origami_deflate_chunks")
    return out, dst_off, comp


def inflate_chunks(src, src_offsets, src_lengths, dst, dst_offsets, dst_lengths, *, threads: int = 0) -> None:
    """Decompress chunk i of `src` into dst[dst_offsets[i], +dst_lengths[i]) (exact size)."""
    so, sl, do, dl = _i64(src_offsets), _i64(src_lengths), _i64(dst_offsets), _i64(dst_lengths)
    sp, sn, k1 = _buffer(src)
    dp, dn, k2 = _buffer(dst, writable=True)
    if len(so) and int((so + sl).max()) > sn:
        raise ValueError("compressed chunk range exceeds the source buffer")
    rc = _lib.lib().origami_inflate_chunks(sp, so.ctypes.data, sl.ctypes.data, len(so), dp, dn, do.ctypes.data,
                                           dl.ctypes.data, int(threads))
    del k1, k2
    _lib.check(rc, "origami_inflate_chunks")


def parse_origqz1(bundle) -> dict[str, Any]:
    """Header of an ORIGQZ1 bundle: chunk_bytes, raw_bytes, payload_offset and the records
    (numpy structured array: raw_len, comp_len, comp_offset, output_offset)."""
    L = _lib.lib()
    ptr, n, keep = _buffer(bundle)
    count, cb, raw, off = (ctypes.c_int64() for _ in range(4))
    rc = L.origami_origqz1_parse(ptr, n, None, 0, ctypes.byref(count), ctypes.byref(cb), ctypes.byref(raw),
                                 ctypes.byref(off))
    if rc != _lib.ORIGAMI_OK:
        _lib.check(rc, "origami_origqz1_parse")
    recs = np.zeros(count.value, dtype=DZ_DTYPE)
    rc = L.origami_origqz1_parse(ptr, n, recs.ctypes.data, len(recs), ctypes.byref(count), ctypes.byref(cb),
                                 ctypes.byref(raw), ctypes.byref(off))
    del keep
    _lib.check(rc, "origami_origqz1_parse")
    return {"chunk_bytes": cb.value, "raw_bytes": raw.value, "payload_offset": off.value, "records": recs}
