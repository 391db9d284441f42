"""The reference's lossless raw-bytes layout (RawBytesTensorAdapter + planner)."""
import json

import numpy as np

from conftest import GOLDEN
from origami_b200.layer import raw_chunk_bounds


def test_raw_symbols_are_gathered_block_bytes():
    z = np.load(GOLDEN / "raw_bytes_case.npz")
    meta = json.loads(str(z["meta"]))
    blocks = z["blocks_u16"]
    assert meta["origami_symbol_shape"] == [1, 1, blocks.nbytes]
    assert meta["origami_bits"] == 8 and meta["shape"] == list(blocks.shape)
    np.testing.assert_array_equal(z["symbols"], blocks.view(np.uint8).reshape(-1))


def test_raw_chunk_bounds_match_reference_plan():
    z = np.load(GOLDEN / "raw_bytes_case.npz")
    specs = z["chunk_specs"]
    n = z["symbols"].size
    bounds = raw_chunk_bounds(n, 4096)
    assert bounds.tolist() == [0] + specs[:, 3].tolist()
    assert (specs[:, 2] == bounds[:-1]).all()
