"""``bundle_v1`` artifacts, byte-compatible with the reference's LocalFileOrigamiStore
(store.py:176-923): a directory per cache key holding

* ``payload.bin``: every compressed chunk, grouped by uncompressed size (ascending), each
  group in (layer name, chunk id) order (store.py:728-811);
* ``qat_bundle.dz``: the ORIGQZ1 bundle, written when every chunk's codec is a deflate
  codec (store.py:45-48, 694-705, 760-772): "ORIGQZ1\\0", u32 chunk bytes (the largest
  raw chunk), u32 chunk count, u64 raw bytes, (u32 raw, u32 compressed) per chunk, then
  the compressed chunks in (layer name, chunk id) order;
* ``manifest.json``: per-layer chunk rows and size groups, request groups and the ORIGQZ1
  references (store.py:813-867), ``json.dump(..., ensure_ascii=False, indent=2)``.

The writer keeps the reference's key order and grouping so that the same payload gives
the same three files, byte for byte. Beyond the reference:

* ``put_packed_layers`` builds the payload straight from packed layers in pinned host
  memory (the save pipeline's output): all chunks of all layers are deflated at once by
  the native codec (origami_b200.codec) and written from views, no per-chunk copies;
* ``inflate_layer_into`` decodes one layer's chunks from the ORIGQZ1 bundle directly into
  a pinned staging buffer at their packed offsets, ready for the restore pipeline's
  host->device copy (the reference decompresses a window, concatenates it and copies it
  through pageable memory, worker.py:796-1049).
"""
from __future__ import annotations

import json
import struct
from dataclasses import asdict
from pathlib import Path
from typing import Any, Iterable

import numpy as np
import torch

from origami_b200 import codec
from origami_b200.metadata import ChunkLayout, ChunkRecord, LayerPayload, OrigamiPayload
from origami_b200.planes import LayerFormat

MAGIC = b"ORIGQZ1\0"


def safe_key(cache_key: str) -> str:
    """store.py:33-34."""
    return str(cache_key).replace("/", "_").replace(":", "_")


def codec_uses_qat_bundle(codec_name: str) -> bool:
    """store.py:45-47: every codec but raw / identity / nvcomp* is a raw-deflate stream."""
    normalized = str(codec_name).lower()
    return normalized not in {"raw", "identity"} and not normalized.startswith("nvcomp")


def _bytes_of(t: Any) -> memoryview:
    if isinstance(t, torch.Tensor):
        t = t.detach()
        if t.device.type != "cpu":
            t = t.cpu()
        return memoryview(t.to(torch.uint8).reshape(-1).contiguous().numpy())
    if isinstance(t, np.ndarray):
        return memoryview(np.ascontiguousarray(t).reshape(-1).view(np.uint8))
    return memoryview(t)


class _Slot:
    """One compressed chunk of a bundle and its place in payload.bin."""

    __slots__ = ("layer", "chunk", "data", "chunk_id", "raw", "size", "offset")

    def __init__(self, layer: str, chunk: ChunkRecord, data: memoryview):
        self.layer = layer
        self.chunk = chunk
        self.data = data
        self.chunk_id = int(chunk.chunk_id)
        self.raw = int(chunk.unpacked_bytes)
        self.size = data.nbytes
        self.offset = 0

    def chunk_row(self) -> dict[str, Any]:
        return {
            "chunk_id": self.chunk_id,
            "layout": asdict(self.chunk.layout),
            "codec": str(self.chunk.codec),
            "compressed_offset": self.offset,
            "compressed_bytes": self.size,
            "unpacked_bytes": self.raw,
        }


def _size_groups(run: list[_Slot], with_refs: bool) -> list[dict[str, Any]]:
    """Rows for the maximal runs of equal unpacked size in `run` (payload.bin order); each
    row's offset is its first chunk's."""
    rows: list[dict[str, Any]] = []
    i = 0
    while i < len(run):
        j = i
        while j < len(run) and run[j].raw == run[i].raw:
            j += 1
        part = run[i:j]
        row: dict[str, Any] = {"output_bytes": run[i].raw, "chunk_ids": [sl.chunk_id for sl in part]}
        if with_refs:
            row["refs"] = [{"layer_name": sl.layer, "chunk_id": sl.chunk_id} for sl in part]
        row["lengths"] = [sl.size for sl in part]
        row["compressed_offset"] = run[i].offset
        row["compressed_bytes"] = sum(sl.size for sl in part)
        rows.append(row)
        i = j
    return rows


class BundleStore:
    """bundle_v1 directories under `root` (LocalFileOrigamiStore's file layout)."""

    def __init__(self, root: str | Path):
        self.root = Path(root)
        self.root.mkdir(parents=True, exist_ok=True)

    def bundle_dir(self, cache_key: str) -> Path:
        return self.root / safe_key(cache_key)

    def manifest_path(self, cache_key: str) -> Path:
        return self.bundle_dir(cache_key) / "manifest.json"

    def payload_path(self, cache_key: str) -> Path:
        return self.bundle_dir(cache_key) / "payload.bin"

    def qat_bundle_path(self, cache_key: str) -> Path:
        return self.bundle_dir(cache_key) / "qat_bundle.dz"

    def contains(self, cache_key: str) -> bool:
        return self.manifest_path(cache_key).exists() and self.payload_path(cache_key).exists()

    # ---------------------------------------------------------------- writing
    def put(self, payload: OrigamiPayload) -> None:
        """Write `payload` as a bundle_v1 directory.

        The bundle is fixed by the format, in three steps:

        1. Canonical chunk order: layers by name, chunks of a layer by id.
        2. ``payload.bin`` holds the compressed chunks sorted by unpacked size, ascending;
           chunks of equal size keep the canonical order (so one layer's chunks of a size
           are adjacent). A chunk's offset is the sum of the sizes before it.
        3. ``qat_bundle.dz`` (only when every chunk is a raw-deflate stream) holds the
           ORIGQZ1 header, the (unpacked, compressed) size table and the chunks, all in
           canonical order.

        The manifest (key order fixed, ``json.dump(..., ensure_ascii=False, indent=2)``)
        describes both files: per layer its chunk rows (by id) and one row per unpacked
        size present in the layer; per size over all layers a request group; and the
        ORIGQZ1 summary with one reference per chunk in canonical order.
        """
        folder = self.bundle_dir(payload.cache_key)
        folder.mkdir(parents=True, exist_ok=True)
        slots = [_Slot(name, ch, _bytes_of(ch.compressed))
                 for name in sorted(payload.layer_payloads)
                 for ch in sorted(payload.layer_payloads[name].chunks, key=lambda c: int(c.chunk_id))]
        stream = sorted(slots, key=lambda sl: sl.raw)  # stable: equal sizes stay canonical
        cursor = 0
        for sl in stream:
            sl.offset = cursor
            cursor += sl.size
        with self.payload_path(payload.cache_key).open("wb") as fh:
            for sl in stream:
                fh.write(sl.data)

        deflate = all(codec_uses_qat_bundle(sl.chunk.codec) for sl in slots)
        qat_file = self.qat_bundle_path(payload.cache_key)
        qat_summary: dict[str, Any] = {}
        if deflate:
            widest = max((sl.raw for sl in slots), default=1)
            table = b"".join(struct.pack("<II", sl.raw, sl.size) for sl in slots)
            with qat_file.open("wb") as fh:
                fh.write(MAGIC + struct.pack("<IIQ", widest, len(slots), sum(sl.raw for sl in slots)) + table)
                for sl in slots:
                    fh.write(sl.data)
            qat_summary = {
                "format": "ORIGQZ1",
                "path": qat_file.name,
                "chunk_bytes": widest,
                "chunks": len(slots),
                "compressed_bytes": sum(sl.size for sl in slots),
                "unpacked_bytes": sum(sl.raw for sl in slots),
                "refs": [{"layer_name": sl.layer, "chunk_id": sl.chunk_id, "output_bytes": sl.raw} for sl in slots],
            }
        elif qat_file.exists():
            qat_file.unlink()

        layers = []
        for name in sorted(payload.layer_payloads):
            lp = payload.layer_payloads[name]
            mine = [sl for sl in slots if sl.layer == name]
            layers.append({
                "layer_name": lp.layer_name,
                "quantizer": lp.quantizer,
                "quant_metadata": lp.quant_metadata,
                "chunks": [sl.chunk_row() for sl in mine],
                "groups": _size_groups([sl for sl in stream if sl.layer == name], with_refs=False),
            })
        manifest = {
            "format": "bundle_v1",
            "cache_key": payload.cache_key,
            "request_id": payload.request_id,
            "quantizer": payload.quantizer,
            "quantizer_config_hash": payload.quantizer_config_hash,
            "token_start": int(payload.token_start),
            "token_count": int(payload.token_count),
            "metadata": dict(payload.metadata),
            "layers": layers,
            "request_groups": _size_groups(stream, with_refs=True),
            "qat_bundle": qat_summary,
        }
        with self.manifest_path(payload.cache_key).open("w", encoding="utf-8") as handle:
            json.dump(manifest, handle, ensure_ascii=False, indent=2, default=str)

    def put_packed_layers(self, *, cache_key: str, request_id: str, token_count: int,
                          layers: Iterable[tuple[str, LayerFormat, Any]], quantizer: str = "origami_planes",
                          quantizer_config_hash: str = "", token_start: int = 0,
                          metadata: dict[str, Any] | None = None, codec_name: str = "zlib", level: int = 1,
                          threads: int = 0, dtype: torch.dtype | None = None) -> OrigamiPayload:
        """Compress packed layers (name, format, packed host bytes: the save pipeline's
        pinned output) with the native codec in one parallel pass and write the bundle.
        Chunk ids, layouts and byte counts are the format's (the reference planner's)."""
        items = []
        bufs, offs, lens = [], [], []
        base = 0
        for name, fmt, host in layers:
            view = np.frombuffer(_bytes_of(host), dtype=np.uint8)[: fmt.packed_bytes]
            items.append((name, fmt, base))
            bufs.append(view)
            for k in range(len(fmt.offsets) - 1):
                offs.append(base + int(fmt.offsets[k]))
                lens.append(int(fmt.offsets[k + 1] - fmt.offsets[k]))
            base += fmt.packed_bytes
        flat = bufs[0] if len(bufs) == 1 else (np.concatenate(bufs) if bufs else np.zeros(0, np.uint8))
        if codec_name.lower() in ("raw", "identity"):
            comp_buf, comp_off, comp_len = flat, np.asarray(offs, np.int64), np.asarray(lens, np.int64)
        else:
            comp_buf, comp_off, comp_len = codec.deflate_chunks(flat, offs, lens, level=level, threads=threads)
        comp_t = torch.from_numpy(comp_buf)
        payload = OrigamiPayload(cache_key=cache_key, request_id=request_id, quantizer=quantizer,
                                 quantizer_config_hash=quantizer_config_hash, token_start=token_start,
                                 token_count=token_count, metadata=dict(metadata or {}))
        k = 0
        for name, fmt, _ in items:
            chunks = []
            for cid, layout in enumerate(fmt.chunk_layouts()):
                o, n = int(comp_off[k]), int(comp_len[k])
                chunks.append(ChunkRecord(chunk_id=cid, layout=layout, codec=codec_name,
                                          compressed=comp_t[o:o + n], compressed_bytes=n,
                                          unpacked_bytes=int(lens[k])))
                k += 1
            payload.layer_payloads[name] = LayerPayload(layer_name=name, quantizer=quantizer,
                                                        quant_metadata=fmt.metadata(dtype), chunks=chunks)
        self.put(payload)
        return payload

    # ---------------------------------------------------------------- reading
    def read_manifest(self, cache_key: str) -> dict[str, Any]:
        path = self.manifest_path(cache_key)
        if not path.exists():
            raise KeyError(f"Origami bundle manifest not found: {cache_key}")
        with path.open("r", encoding="utf-8") as handle:
            manifest = json.load(handle)
        if manifest.get("format") != "bundle_v1":
            raise ValueError(f"Unsupported Origami artifact format: {manifest.get('format')!r}")
        return manifest

    def get(self, cache_key: str) -> OrigamiPayload:
        """store.py:204-214 / 881-923: the payload with every chunk's compressed bytes."""
        manifest = self.read_manifest(cache_key)
        data = self.payload_path(cache_key).read_bytes()
        payload = OrigamiPayload(
            cache_key=str(manifest["cache_key"]), request_id=str(manifest.get("request_id", "")),
            quantizer=str(manifest["quantizer"]), quantizer_config_hash=str(manifest.get("quantizer_config_hash", "")),
            token_start=int(manifest.get("token_start", 0)), token_count=int(manifest.get("token_count", 0)),
            metadata=dict(manifest.get("metadata") or {}))
        payload.metadata["artifact_format"] = "bundle_v1"
        for layer in manifest["layers"]:
            chunks = []
            for row in layer.get("chunks", []):
                off, n = int(row["compressed_offset"]), int(row["compressed_bytes"])
                chunks.append(ChunkRecord(
                    chunk_id=int(row["chunk_id"]), layout=ChunkLayout(**row["layout"]),
                    codec=str(row.get("codec", "qat")),
                    compressed=torch.frombuffer(bytearray(data[off:off + n]), dtype=torch.uint8),
                    compressed_bytes=n, unpacked_bytes=int(row["unpacked_bytes"])))
            payload.layer_payloads[str(layer["layer_name"])] = LayerPayload(
                layer_name=str(layer["layer_name"]), quantizer=str(layer["quantizer"]),
                quant_metadata=dict(layer.get("quant_metadata") or {}),
                chunks=sorted(chunks, key=lambda c: int(c.chunk_id)))
        return payload

    def open_qat_bundle(self, cache_key: str) -> "QatBundle":
        return QatBundle(self.qat_bundle_path(cache_key), self.read_manifest(cache_key))


class QatBundle:
    """A loaded ORIGQZ1 bundle with the manifest's (layer, chunk) references: the restore
    side's source of compressed chunk windows."""

    def __init__(self, path: str | Path, manifest: dict[str, Any] | None = None):
        self.data = np.fromfile(path, dtype=np.uint8)
        head = codec.parse_origqz1(self.data)
        self.records = head["records"]
        self.chunk_bytes = head["chunk_bytes"]
        self.raw_bytes = head["raw_bytes"]
        self.index: dict[tuple[str, int], int] = {}
        refs = ((manifest or {}).get("qat_bundle") or {}).get("refs") or []
        if refs and len(refs) != len(self.records):
            raise ValueError("ORIGQZ1 record count does not match the manifest references")
        for i, ref in enumerate(refs):
            if int(ref["output_bytes"]) != int(self.records[i]["raw_len"]):
                raise ValueError(f"ORIGQZ1 record {i} length does not match the manifest")
            self.index[(str(ref["layer_name"]), int(ref["chunk_id"]))] = i

    def layer_records(self, layer_name: str, num_chunks: int) -> np.ndarray:
        return np.asarray([self.index[(layer_name, c)] for c in range(num_chunks)], dtype=np.int64)

    def inflate_layer_into(self, layer_name: str, fmt: LayerFormat, out: torch.Tensor | np.ndarray, *,
                           threads: int = 0) -> None:
        """Decode the layer's chunks into `out` (pinned staging) at the format's packed
        offsets, in parallel, straight from the bundle bytes."""
        n = len(fmt.offsets) - 1
        idx = self.layer_records(layer_name, n)
        rec = self.records[idx]
        if np.any(rec["raw_len"].astype(np.int64) != np.diff(fmt.offsets)):
            raise ValueError(f"{layer_name}: bundle chunk sizes differ from the layer format")
        codec.inflate_chunks(self.data, rec["comp_offset"], rec["comp_len"], out, fmt.offsets[:-1],
                             np.diff(fmt.offsets), threads=threads)
