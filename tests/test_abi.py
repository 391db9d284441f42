"""The C-ABI library loads without a GPU, exports every symbol the header declares,
and its host-side validation (no CUDA call is reached) rejects bad arguments with the
reference's messages."""
import ctypes
import re

import numpy as np
import pytest

from conftest import REPO
from origami_b200 import _lib


def header_functions():
    text = (REPO / "include" / "origami_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(origami_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_header_symbols():
    L = _lib.lib()
    names = header_functions()
    assert len(names) >= 9
    for name in names:
        assert hasattr(L, name), name
    assert set(names) == set(_lib.EXPORTS)
    assert L.origami_b200_version() >= 1
    assert L.origami_packed_bytes(37, 3) == (37 * 3 + 7) // 8
    assert L.origami_packed_bytes(0, 8) == 0


def _canon(L, specs, offsets, bits, shape, axes, T, H, D, flat_bytes=1 << 20, out_bytes=None):
    specs = np.ascontiguousarray(specs, dtype=np.int64).reshape(-1, 6)
    offsets = np.ascontiguousarray(offsets, dtype=np.int64)
    bits = np.ascontiguousarray(bits, dtype=np.int64)
    shape = np.ascontiguousarray(shape, dtype=np.int64)
    axes = np.ascontiguousarray(axes, dtype=np.int64)
    numel = int(np.prod(shape)) if out_bytes is None else out_bytes
    fake = 1 << 12  # never dereferenced: validation fails first
    rc = L.origami_unpack_canonical_storage_chunks(
        fake, flat_bytes, fake, fake, fake, offsets.ctypes.data, bits.ctypes.data, specs.ctypes.data, len(specs),
        shape.ctypes.data, len(shape), axes.ctypes.data, T, H, D, fake, numel, None)
    return rc, L.origami_last_error().decode()


@pytest.mark.parametrize("mutate, message", [
    (lambda a: a.update(specs=[[0, 3, 0, 4, 0, 5]]), "invalid head range"),
    (lambda a: a.update(specs=[[0, 2, 2, 2, 0, 5]]), "invalid channel range"),
    (lambda a: a.update(specs=[[0, 2, 0, 4, 0, 6]]), "invalid token range"),
    (lambda a: a.update(bits=[9]), "only 1..8 bit symbols"),
    (lambda a: a.update(offsets=[0, 11]), "byte size mismatch"),
    (lambda a: a.update(shape=[5, 2]), "rank 3 or rank 4"),
    (lambda a: a.update(shape=[5, 3, 4]), "head axis size must match"),
    (lambda a: a.update(axes=[0, 1, 2, 5]), "layer axis must be -1"),
    (lambda a: a.update(shape=[5, 2, 4, 2], axes=[0, 1, 2, 3]), "layer axis size 1"),
    (lambda a: a.update(out_bytes=7), "layout needs"),
])
def test_canonical_validation(mutate, message):
    args = dict(specs=[[0, 2, 0, 4, 0, 5]], offsets=[0, 40], bits=[8], shape=[5, 2, 4], axes=[0, 1, 2, -1],
                out_bytes=None)
    mutate(args)
    rc, msg = _canon(_lib.lib(), args["specs"], args["offsets"], args["bits"], args["shape"], args["axes"], 5, 2, 4,
                     out_bytes=args["out_bytes"])
    assert rc == -1, msg
    assert message in msg


def _layer_call(L, planes, specs, offsets, T=64, bs=16, H=2, D=16, nids=4, align=0):
    fake = 1 << 12
    kv = _lib.PagedKV(fake + align, 0, 2, 8, bs, H, D)
    pl = _lib.Planes()
    pl.num_planes = len(planes)
    for i, (s, b) in enumerate(planes):
        pl.shift[i], pl.bits[i] = s, b
    specs = np.ascontiguousarray(specs, dtype=np.int64).reshape(-1, 6)
    offsets = np.ascontiguousarray(offsets, dtype=np.int64)
    tab = _lib.ChunkTable(fake, fake, specs.ctypes.data, offsets.ctypes.data, len(specs))
    rc = L.origami_restore_layer_to_paged(fake, 1 << 20, ctypes.byref(pl), ctypes.byref(tab), ctypes.byref(kv), fake,
                                          nids, T, None, None)
    return rc, L.origami_last_error().decode()


def test_layer_validation():
    L = _lib.lib()
    good_specs = [[0, 1, 0, 16, 0, 64], [1, 2, 0, 16, 0, 64]]
    n = 64 * 16
    offs = np.arange(9) * n  # 2 kv * 2 planes * 2 specs, 8-bit
    cases = [
        (dict(planes=[(8, 8)]), "cover all 16"),
        (dict(planes=[(8, 8), (0, 9)]), "bits must be 1..8"),
        (dict(planes=[(8, 8), (4, 8)]), "overlaps"),
        (dict(specs=[[0, 1, 0, 16, 0, 64]]), "exactly once"),
        (dict(specs=[[0, 1, 0, 16, 0, 32], [1, 2, 0, 16, 0, 64]]), "span tokens"),
        (dict(nids=3), "block table"),
        (dict(offsets=np.arange(9) * (n - 1)), "offsets give"),
        (dict(align=8), "16-byte aligned"),
        (dict(D=12, specs=[[0, 2, 0, 12, 0, 64]]), "multiple of 8"),
    ]
    for kw, message in cases:
        args = dict(planes=[(8, 8), (0, 8)], specs=good_specs, offsets=offs)
        args.update(kw)
        rc, msg = _layer_call(L, **args)
        assert rc != 0 and message in msg, (kw, msg)
