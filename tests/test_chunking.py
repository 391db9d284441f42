"""Planner and layout helpers against fixtures produced by the reference itself."""
import json

import pytest

from conftest import GOLDEN
from origami_b200.lossless import native_cpu
from origami_b200.lossless.chunking import plan_head_channel_chunks


def test_planner_matches_reference():
    cases = json.loads((GOLDEN / "planner_cases.json").read_text())
    assert len(cases) > 300
    for case in cases:
        got = plan_head_channel_chunks(**case["args"])
        rows = [[c.chunk_id, c.layout.layer_index, c.layout.head_start, c.layout.head_end, c.layout.channel_start,
                 c.layout.channel_end, c.layout.token_start, c.layout.token_end, c.layout.unpacked_bytes] for c in got]
        assert rows == case["chunks"], case["args"]


def test_layout_helpers_match_reference():
    for case in json.loads((GOLDEN / "layout_cases.json").read_text()):
        lay = case["layout"]
        if "error" in case:
            with pytest.raises(ValueError) as exc:
                native_cpu.normalize_symbol_layout(lay)
            assert str(exc.value) == case["error"]
            continue
        assert native_cpu.normalize_symbol_layout(lay) == case["normalized"]
        assert native_cpu.axis_positions(lay) == case["axis_positions"]
        for s in case["sizes"]:
            if "error" in s:
                with pytest.raises(ValueError) as exc:
                    native_cpu.canonical_axis_sizes(s["shape"], lay)
                assert str(exc.value) == s["error"]
            else:
                assert list(native_cpu.canonical_axis_sizes(s["shape"], lay)) == s["result"]
