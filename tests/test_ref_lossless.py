"""The CPU baseline's restatement of the reference's raw-bytes lossless restore
(oracle/ref_lossless.py) against the reference's own outputs."""
import json

import numpy as np
import torch

from conftest import GOLDEN
import ref_lossless as rl


def test_zlib_streams_match_the_reference_codec():
    z = np.load(GOLDEN / "zlib_case.npz")
    comp = z["compressed"]
    offs = np.concatenate([[0], np.cumsum(z["comp_sizes"])])
    for i, raw in enumerate(z["raw"]):
        want = comp[offs[i]:offs[i + 1]].tobytes()
        assert rl.zlib_compress(raw) == want
        np.testing.assert_array_equal(rl.zlib_decompress(want, raw.size).numpy(), raw)


def test_raw_symbols_and_slices_match_the_reference_adapter_and_planner():
    z = np.load(GOLDEN / "raw_bytes_case.npz")
    meta = json.loads(str(z["meta"]))
    blocks = torch.from_numpy(z["blocks_u16"].view(np.int16)).view(torch.bfloat16)
    symbols, mine = rl.raw_quantize(blocks)
    np.testing.assert_array_equal(symbols.numpy(), z["symbols"])
    for key in ("format", "shape", "byte_count", "origami_bits", "origami_symbol_shape", "origami_symbol_layout"):
        assert mine[key] == meta[key], key
    specs = z["chunk_specs"]
    assert rl.slice_bounds(symbols.numel(), 4096) == [0] + specs[:, 3].tolist()
    back = rl.raw_dequantize(symbols, mine)
    assert torch.equal(back.view(torch.int16), blocks.view(torch.int16))


def test_assign_blocks_is_the_inverse_of_the_reference_selection():
    z = np.load(GOLDEN / "select_blocks.npz")
    ids = z["ids"].tolist()
    for cache_key, sel_key in (("cache", "selected"), ("cache_blocks_first", "selected_blocks_first")):
        cache = torch.from_numpy(z[cache_key].copy())
        fresh = torch.zeros_like(cache)
        rl.assign_blocks(fresh, ids, torch.from_numpy(z[sel_key]))
        dim = 1 if cache.shape[0] == 2 else 0
        assert torch.equal(torch.index_select(fresh, dim, torch.tensor(ids)), torch.from_numpy(z[sel_key]))


def test_save_restore_round_trip():
    g = torch.Generator().manual_seed(3)
    cache = torch.randint(-32768, 32767, (2, 12, 16, 2, 64), generator=g, dtype=torch.int16).view(torch.bfloat16)
    ids = [7, 2, 9, 4]
    saved = rl.save_layer(cache, ids, chunk_bytes=5000)
    assert sum(saved.sizes) == 2 * len(ids) * 16 * 2 * 64 * 2
    fresh = torch.zeros_like(cache)
    rl.restore_layer(saved, fresh, ids)
    t = torch.tensor(ids)
    assert torch.equal(fresh[:, t].view(torch.int16), cache[:, t].view(torch.int16))
    untouched = [b for b in range(12) if b not in ids]
    assert not fresh[:, untouched].view(torch.int16).any()
