"""Host codec boundary: raw DEFLATE level 1 identical to the reference's zlib backend."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from origami_b200.lossless.cpu_qat import CpuLosslessCodec


def test_zlib_matches_reference_fixture():
    z = np.load(GOLDEN / "zlib_case.npz")
    raw, comp, sizes = z["raw"], z["compressed"], z["comp_sizes"]
    codec = CpuLosslessCodec("zlib")
    chunks = [torch.from_numpy(raw[i].copy()) for i in range(raw.shape[0])]
    mine = codec.compress_many(chunks)
    bounds = np.concatenate([[0], np.cumsum(sizes)])
    theirs = [torch.from_numpy(comp[a:b].copy()) for a, b in zip(bounds[:-1], bounds[1:])]
    for m, t in zip(mine, theirs):
        assert torch.equal(m, t)  # same zlib build, same stream
    back = codec.decompress_many(theirs, [raw.shape[1]] * raw.shape[0])
    for b, c in zip(back, chunks):
        assert torch.equal(b, c)


def test_codec_errors_like_reference():
    with pytest.raises(RuntimeError):
        CpuLosslessCodec("qat")
    assert CpuLosslessCodec("qat", allow_zlib_fallback=True).backend == "zlib"
    with pytest.raises(ValueError):
        CpuLosslessCodec("lz4")
    codec = CpuLosslessCodec("zlib")
    with pytest.raises(RuntimeError):
        codec.decompress(codec.compress(torch.arange(100, dtype=torch.uint8)), output_bytes=99)
    raw = CpuLosslessCodec("raw")
    with pytest.raises(RuntimeError):
        raw.decompress_many([torch.zeros(3, dtype=torch.uint8)], [4])
