"""Generate golden fixtures from the reference Origami code (run where it is checked out).

    python tests/golden/make_golden.py [/path/to/reference]

Imports the reference's own Python modules (planner, raw-bytes adapter, zlib codec,
layout helpers) through a package-path shim, runs them on seeded inputs and writes:

  planner_cases.json   plan_head_channel_chunks outputs over a grid of shapes
                       (lossless/chunking.py:22-123)
  layout_cases.json    normalize_symbol_layout / canonical_axis_sizes / axis_positions
                       results and error messages (lossless/native_cpu.py:81-130)
  raw_bytes_case.npz   RawBytesTensorAdapter.quantize of a seeded bf16 block tensor
                       (quantization/raw_tensor.py:100-122) and the chunk bounds the
                       planner gives its [1, 1, N] symbols
  zlib_case.npz        CpuLosslessCodec('zlib') compress of seeded bytes
                       (lossless/cpu_qat.py:64-84), with the input
  select_blocks.npz    the worker's _select_blocks (index_select) on a seeded cache
                       (worker.py:1881-1897)
  bundle_v1_zlib/, bundle_v1_raw/
                       bundle_v1 directories (manifest.json, payload.bin and, for the
                       deflate codec, the ORIGQZ1 qat_bundle.dz) written by the reference's
                       LocalFileOrigamiStore (store.py:706-867) from seeded chunks, with
                       the chunk inputs (inputs.npz)

The reference GPU unpack kernel cannot run here; tests/golden/make_ref_vectors.py
produces its vectors on a B200 from the compiled reference extension.
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
V1 = "vllm/distributed/kv_transfer/kv_connector/v1"
PKG = "vllm.distributed.kv_transfer.kv_connector.v1.origami"


def import_reference(root: str):
    os.environ["ORIGAMI_LIGHT_IMPORT"] = "1"
    import vllm.distributed.kv_transfer.kv_connector.v1 as v1  # installed vLLM provides the parents

    v1.__path__.insert(0, str(Path(root) / V1))
    import importlib

    mods = {
        "chunking": importlib.import_module(f"{PKG}.lossless.chunking"),
        "native_cpu": importlib.import_module(f"{PKG}.lossless.native_cpu"),
        "cpu_qat": importlib.import_module(f"{PKG}.lossless.cpu_qat"),
        "raw_tensor": importlib.import_module(f"{PKG}.quantization.raw_tensor"),
        "worker": importlib.import_module(f"{PKG}.worker"),
    }
    return mods


PLANNER_GRID = []
for H in (1, 2, 4, 8):
    for D in (64, 128):
        for T in (1, 7, 16, 100, 1024, 4096, 8192, 37123, 32768):
            for (mn, tg, mx) in ((1 << 20, 1 << 20, 1 << 20), (64 << 10, 64 << 10, 64 << 10),
                                 (4 << 20, 4 << 20, 4 << 20), (256 << 10, 1 << 20, 2 << 20),
                                 (1 << 10, 3000, 5000)):
                PLANNER_GRID.append((H, D, T, mn, tg, mx))
PLANNER_GRID += [(1, 1 << 22, 1, 1 << 20, 1 << 20, 1 << 20), (1, 3 * (1 << 20) + 5, 1, 1 << 20, 1 << 20, 1 << 20),
                 (3, 96, 555, 1000, 2000, 4000), (8, 128, 0, 1 << 20, 1 << 20, 1 << 20)]


def main(root: str) -> None:
    import torch

    m = import_reference(root)
    plan = m["chunking"].plan_head_channel_chunks
    cases = []
    for (H, D, T, mn, tg, mx) in PLANNER_GRID:
        chunks = plan(layer_index=5, num_heads=H, head_dim=D, token_count=T, bytes_per_symbol=1, min_bytes=mn,
                      target_bytes=tg, max_bytes=mx)
        cases.append({
            "args": {"layer_index": 5, "num_heads": H, "head_dim": D, "token_count": T, "bytes_per_symbol": 1,
                     "min_bytes": mn, "target_bytes": tg, "max_bytes": mx},
            "chunks": [[c.chunk_id, c.layout.layer_index, c.layout.head_start, c.layout.head_end,
                        c.layout.channel_start, c.layout.channel_end, c.layout.token_start, c.layout.token_end,
                        c.layout.unpacked_bytes] for c in chunks],
        })
    (HERE / "planner_cases.json").write_text(json.dumps(cases, separators=(",", ":")))

    nc = m["native_cpu"]
    layouts = [["token", "head", "head_dim"], ["head", "token", "head_dim"], ["head", "head_dim", "token"],
               ["layer", "head", "head_dim", "token"], ["Tokens", "KV_HEADS", "channel"], ["seq", "dim", "heads", "layers"],
               ["token", "head"], ["token", "token", "head_dim"], ["token", "head", "head_dim", "bogus"]]
    shapes = {3: [[5, 2, 8], [0, 2, 8]], 4: [[1, 2, 8, 5], [2, 2, 8, 5]]}
    lcases = []
    for lay in layouts:
        entry = {"layout": lay}
        try:
            entry["normalized"] = nc.normalize_symbol_layout(lay)
            entry["axis_positions"] = nc.axis_positions(lay)
        except Exception as exc:  # noqa: BLE001
            entry["error"] = str(exc)
        sizes = []
        for shape in shapes.get(len(lay), []):
            try:
                t, h, d, sh, ly = nc.canonical_axis_sizes(shape, lay)
                sizes.append({"shape": shape, "result": [t, h, d, sh, ly]})
            except Exception as exc:  # noqa: BLE001
                sizes.append({"shape": shape, "error": str(exc)})
        entry["sizes"] = sizes
        lcases.append(entry)
    (HERE / "layout_cases.json").write_text(json.dumps(lcases, indent=1))

    g = torch.Generator().manual_seed(7)
    blocks = torch.randn((2, 3, 16, 2, 64), generator=g).to(torch.bfloat16)
    q = m["raw_tensor"].RawBytesTensorAdapter().quantize(blocks)
    n = int(q.symbols.numel())
    rb = plan(layer_index=0, num_heads=1, head_dim=n, token_count=1, bytes_per_symbol=1, min_bytes=4096,
              target_bytes=4096, max_bytes=4096)
    np.savez_compressed(
        HERE / "raw_bytes_case.npz",
        blocks_u16=blocks.view(torch.int16).numpy().view(np.uint16),
        symbols=q.symbols.numpy(),
        meta=json.dumps(q.metadata),
        chunk_specs=np.asarray([[c.layout.head_start, c.layout.head_end, c.layout.channel_start, c.layout.channel_end,
                                 c.layout.token_start, c.layout.token_end] for c in rb], dtype=np.int64),
    )

    data = torch.randint(0, 256, (3, 40000), generator=g, dtype=torch.uint8)
    data[1, :20000] = 7  # compressible part
    codec = m["cpu_qat"].CpuLosslessCodec(backend="zlib")
    comp = codec.compress_many([data[i] for i in range(3)])
    np.savez_compressed(HERE / "zlib_case.npz", raw=data.numpy(),
                        compressed=np.concatenate([c.numpy() for c in comp]),
                        comp_sizes=np.asarray([c.numel() for c in comp], dtype=np.int64))

    W = m["worker"].OrigamiConnectorWorker
    cache = torch.randint(-30000, 30000, (2, 10, 4, 2, 8), generator=g, dtype=torch.int16)
    ids = (7, 2, 9, 2)
    sel = W._select_blocks(W.__new__(W), cache, ids)
    cache_bf = torch.randint(-30000, 30000, (10, 2, 4, 2, 8), generator=g, dtype=torch.int16)
    sel_bf = W._select_blocks(W.__new__(W), cache_bf, ids)
    np.savez_compressed(HERE / "select_blocks.npz", cache=cache.numpy(), ids=np.asarray(ids), selected=sel.numpy(),
                        cache_blocks_first=cache_bf.numpy(), selected_blocks_first=sel_bf.numpy())
    bundle_cases(m, root)
    print("golden fixtures written to", HERE)


BUNDLE_LAYERS = ("model.layers.0.self_attn.attn", "model.layers.1.self_attn.attn")


def bundle_inputs(case: str):
    """Seeded chunk inputs of a bundle case: per layer, the raw chunk bytes (a planes-format
    packed layer of 100 tokens x 2 heads x 16 channels cut by the planner with 1000-byte
    chunks, so chunk sizes differ) and the chunk layout rows."""
    sys.path.insert(0, str(HERE.parents[1]))
    from origami_b200 import LayerFormat

    rng = np.random.default_rng(1234 if case == "zlib" else 4321)
    layers = BUNDLE_LAYERS if case == "zlib" else BUNDLE_LAYERS[:1]
    out = {}
    for li, name in enumerate(layers):
        fmt = LayerFormat(100, 2, 16, chunk_min_bytes=1000, chunk_target_bytes=1000, chunk_max_bytes=1000,
                          layer_index=li)
        raw = (rng.normal(0, 12, fmt.packed_bytes).astype(np.int64) & 0xFF).astype(np.uint8)
        rows = [[l.layer_index, l.head_start, l.head_end, l.channel_start, l.channel_end, l.token_start,
                 l.token_end, l.unpacked_bytes] for l in fmt.chunk_layouts()]
        out[name] = (raw, np.asarray(fmt.offsets, dtype=np.int64), rows, fmt.metadata())
    return out


def bundle_cases(m, root: str) -> None:
    """bundle_v1 directories written by the reference's LocalFileOrigamiStore
    (store.py:706-867): a zlib payload of two layers (with ORIGQZ1 qat_bundle.dz) and a
    raw payload (no ORIGQZ1 file), plus the inputs that built them."""
    import importlib
    import shutil
    import tempfile

    import torch

    st = importlib.import_module(f"{PKG}.store")
    md = importlib.import_module(f"{PKG}.metadata")
    codec = m["cpu_qat"].CpuLosslessCodec("zlib")
    for case in ("zlib", "raw"):
        inputs = bundle_inputs(case)
        payload = md.OrigamiPayload(cache_key=f"req-7:{case}/bundle", request_id="req-7", quantizer="origami_planes",
                                    quantizer_config_hash="cafe01", token_start=0, token_count=100,
                                    metadata={"model": "synthetic", "layers": len(inputs)})
        store_arrays = {}
        for name, (raw, offsets, rows, meta) in inputs.items():
            chunks = []
            for k, row in enumerate(rows):
                data = torch.from_numpy(raw[offsets[k]:offsets[k + 1]].copy())
                comp = codec._zlib_compress(data) if case == "zlib" else data
                chunks.append(md.ChunkRecord(chunk_id=k, layout=md.ChunkLayout(*row), codec=case, compressed=comp,
                                             compressed_bytes=int(comp.numel()), unpacked_bytes=int(data.numel())))
            # insertion order of chunks is scrambled: the writer sorts them
            chunks = chunks[1::2] + chunks[0::2]
            payload.layer_payloads[name] = md.LayerPayload(layer_name=name, quantizer="origami_planes",
                                                           quant_metadata=meta, chunks=chunks)
            store_arrays[f"{name}/raw"] = raw
            store_arrays[f"{name}/offsets"] = offsets
        with tempfile.TemporaryDirectory() as tmp:
            st.LocalFileOrigamiStore(tmp).put(payload)
            src = Path(tmp) / st._safe_key(payload.cache_key)
            dst = HERE / f"bundle_v1_{case}"
            if dst.exists():
                shutil.rmtree(dst)
            shutil.copytree(src, dst)
        np.savez_compressed(HERE / f"bundle_v1_{case}" / "inputs.npz", **store_arrays)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ORIGAMI_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (or set ORIGAMI_REFERENCE_ROOT)")
    main(root)
