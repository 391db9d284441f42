"""bundle_v1 artifacts and the host codec against fixtures written by the reference's own
LocalFileOrigamiStore (tests/golden/bundle_v1_*, made by make_golden.py)."""
from __future__ import annotations

import shutil
import struct
import zlib
from pathlib import Path

import numpy as np
import pytest
import torch

from origami_b200 import LayerFormat, codec
from origami_b200.bundle import BundleStore, QatBundle, safe_key
from origami_b200.metadata import ChunkLayout, ChunkRecord, LayerPayload, OrigamiPayload

GOLDEN = Path(__file__).resolve().parent / "golden"
LAYERS = ("model.layers.0.self_attn.attn", "model.layers.1.self_attn.attn")
FILES = ("manifest.json", "payload.bin", "qat_bundle.dz")


def _inputs(case):
    z = np.load(GOLDEN / f"bundle_v1_{case}" / "inputs.npz")
    layers = LAYERS if case == "zlib" else LAYERS[:1]
    return {name: (z[f"{name}/raw"], z[f"{name}/offsets"]) for name in layers}


def _fmt(li):
    return LayerFormat(100, 2, 16, chunk_min_bytes=1000, chunk_target_bytes=1000, chunk_max_bytes=1000,
                       layer_index=li)


def _write_ours(tmp_path, case, via_packed_layers):
    store = BundleStore(tmp_path)
    key = f"req-7:{case}/bundle"
    inputs = _inputs(case)
    meta = {"model": "synthetic", "layers": len(inputs)}
    if via_packed_layers:
        store.put_packed_layers(cache_key=key, request_id="req-7", token_count=100, quantizer="origami_planes",
                                quantizer_config_hash="cafe01", metadata=meta, codec_name=case,
                                layers=[(name, _fmt(li), raw) for li, (name, (raw, _)) in enumerate(inputs.items())])
    else:
        payload = OrigamiPayload(cache_key=key, request_id="req-7", quantizer="origami_planes",
                                 quantizer_config_hash="cafe01", token_start=0, token_count=100, metadata=meta)
        for li, (name, (raw, offsets)) in enumerate(inputs.items()):
            fmt = _fmt(li)
            chunks = []
            for k, layout in enumerate(fmt.chunk_layouts()):
                data = raw[offsets[k]:offsets[k + 1]]
                comp = data
                if case != "raw":  # the reference codec's stream (cpu_qat.py:64-74)
                    c = zlib.compressobj(level=1, wbits=-15)
                    comp = np.frombuffer(c.compress(data.tobytes()) + c.flush(), dtype=np.uint8)
                chunks.append(ChunkRecord(k, layout, case, torch.from_numpy(comp.copy()), int(comp.size),
                                          int(data.size)))
            payload.layer_payloads[name] = LayerPayload(name, "origami_planes", fmt.metadata(), chunks[::-1])
        store.put(payload)
    return store, key


@pytest.mark.parametrize("case", ["zlib", "raw"])
@pytest.mark.parametrize("via_packed_layers", [False, True])
def test_writer_reproduces_reference_bundle(tmp_path, case, via_packed_layers):
    store, key = _write_ours(tmp_path, case, via_packed_layers)
    ref = GOLDEN / f"bundle_v1_{case}"
    ours = store.bundle_dir(key)
    assert ours.name == safe_key(key)
    for f in FILES:
        if (ref / f).exists():
            assert (ours / f).read_bytes() == (ref / f).read_bytes(), f
        else:
            assert not (ours / f).exists(), f


@pytest.mark.parametrize("case", ["zlib", "raw"])
def test_reader_and_native_inflate_recover_the_chunks(tmp_path, case):
    key = f"req-7:{case}/bundle"
    shutil.copytree(GOLDEN / f"bundle_v1_{case}", tmp_path / safe_key(key))
    store = BundleStore(tmp_path)
    payload = store.get(key)
    assert payload.metadata["artifact_format"] == "bundle_v1"
    assert payload.token_count == 100 and payload.quantizer_config_hash == "cafe01"
    for li, (name, (raw, offsets)) in enumerate(_inputs(case).items()):
        lp = payload.layer_payloads[name]
        fmt = _fmt(li)
        assert [c.layout for c in lp.chunks] == fmt.chunk_layouts()
        assert lp.quant_metadata["format"] == "origami_planes_v1"
        for k, c in enumerate(lp.chunks):
            want = raw[offsets[k]:offsets[k + 1]]
            got = c.compressed.numpy() if case == "raw" else np.frombuffer(
                zlib.decompress(c.compressed.numpy().tobytes(), wbits=-15), dtype=np.uint8)
            np.testing.assert_array_equal(got, want)


def test_origqz1_window_inflates_into_pinned_layout(tmp_path):
    key = "req-7:zlib/bundle"
    shutil.copytree(GOLDEN / "bundle_v1_zlib", tmp_path / safe_key(key))
    store = BundleStore(tmp_path)
    qb = store.open_qat_bundle(key)
    assert qb.raw_bytes == sum(int(o[-1]) for _, o in _inputs("zlib").values())
    for li, (name, (raw, offsets)) in enumerate(_inputs("zlib").items()):
        out = np.full(int(offsets[-1]), 0xAB, dtype=np.uint8)
        qb.inflate_layer_into(name, _fmt(li), out, threads=4)
        np.testing.assert_array_equal(out, raw)


def test_origqz1_parser_checks():
    good = (GOLDEN / "bundle_v1_zlib" / "qat_bundle.dz").read_bytes()
    head = codec.parse_origqz1(good)
    assert head["payload_offset"] == 24 + 8 * len(head["records"])
    assert int(head["records"]["comp_len"].sum()) + head["payload_offset"] == len(good)
    bad = [
        (good[:20], "too small"),
        (b"ORIGQZ2\0" + good[8:], "invalid ORIGQZ1 bundle magic"),
        (good[:8] + struct.pack("<I", 0) + good[12:], "chunk_bytes must be positive"),
        (good[:12] + struct.pack("<I", 0) + good[16:], "chunk_count must be positive"),
        (good[:12] + struct.pack("<I", 10 ** 6) + good[16:], "record table exceeds bundle size"),
        (good[:16] + struct.pack("<Q", 5) + good[24:], "raw size mismatch"),
        (good + b"\0", "compressed payload size mismatch"),
        (good[:24] + struct.pack("<II", 10 ** 9, 5) + good[32:], "invalid ORIGQZ1 raw chunk length"),
    ]
    for blob, msg in bad:
        with pytest.raises(RuntimeError, match=msg):
            codec.parse_origqz1(blob)


def test_native_codec_matches_zlib_and_checks_lengths():
    rng = np.random.default_rng(3)
    data = (rng.normal(0, 9, 300_000).astype(np.int64) & 0xFF).astype(np.uint8)
    offs = np.array([0, 1000, 1000, 250_000], dtype=np.int64)
    lens = np.array([1000, 0, 249_000, 50_000], dtype=np.int64)
    buf, co, cl = codec.deflate_chunks(data, offs, lens, threads=3)
    for i in range(len(offs)):
        c = zlib.compressobj(level=1, wbits=-15, strategy=zlib.Z_DEFAULT_STRATEGY)
        want = c.compress(data[offs[i]:offs[i] + lens[i]].tobytes()) + c.flush()
        assert bytes(buf[co[i]:co[i] + cl[i]]) == want
    out = np.zeros(300_000, dtype=np.uint8)
    codec.inflate_chunks(buf, co, cl, out, offs, lens)
    np.testing.assert_array_equal(out, data)
    with pytest.raises(RuntimeError, match="decoded 249000 bytes, expected 248999"):
        codec.inflate_chunks(buf, co[2:3], cl[2:3], out, offs[2:3], lens[2:3] - 1)
    with pytest.raises(RuntimeError, match="exceeds"):
        codec.inflate_chunks(buf, co, cl, out[:1000], offs, lens)
    with pytest.raises(RuntimeError, match="inflate of chunk 0 failed"):
        codec.inflate_chunks(np.full(64, 0xFF, np.uint8), [0], [64], out, [0], [10])


def test_restore_staging_from_pinned_payload(tmp_path):
    """Save side -> bundle -> restore staging, host only: packed layers in (pinned) host
    memory are deflated in one parallel pass and come back bit-exact into a staging
    buffer at their packed offsets."""
    store = BundleStore(tmp_path)
    fmts = [LayerFormat(333, 4, 64, chunk_min_bytes=1 << 14, chunk_target_bytes=1 << 14, chunk_max_bytes=1 << 14,
                        layer_index=i) for i in range(3)]
    rng = np.random.default_rng(9)
    packed = [torch.from_numpy((rng.normal(0, 30, f.packed_bytes).astype(np.int64) & 0xFF).astype(np.uint8))
              for f in fmts]
    store.put_packed_layers(cache_key="k", request_id="r", token_count=333,
                            layers=[(f"layer{i}", f, p) for i, (f, p) in enumerate(zip(fmts, packed))])
    qb = store.open_qat_bundle("k")
    assert isinstance(qb, QatBundle)
    for i, f in enumerate(fmts):
        out = torch.empty(f.packed_bytes, dtype=torch.uint8)
        qb.inflate_layer_into(f"layer{i}", f, out)
        assert torch.equal(out, packed[i])
    got = store.get("k")
    assert [c.layout for c in got.layer_payloads["layer1"].chunks] == fmts[1].chunk_layouts()
    assert got.layer_payloads["layer2"].chunks[0].layout == ChunkLayout(2, *fmts[2].specs[0].tolist(),
                                                                        int(fmts[2].offsets[1]))
