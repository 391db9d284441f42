"""Worker-side connector hooks on the B200 path.

Mirrors the hot-path methods of the reference OrigamiConnectorWorker
(O/worker.py:194-2499: register_kv_caches, start_load_kv, wait_for_layer_load,
save_kv_layer, wait_for_save, get_finished) for the lossless layouts, with the GPU
work done by this library:

save_kv_layer  : an event on the model's stream orders the pack after the layer's KV
                 writes; pack_layer (gather + plane split + bitpack) runs on a save
                 stream into a device slot, the chunks go D2H into pinned memory, and a
                 host thread compresses them with the host codec (zlib / raw).
start_load_kv  : per request, a host thread decompresses each layer's chunks directly
                 into a pinned staging buffer (no cat, no pageable copy) and enqueues it
                 on the RestorePipeline (copy stream -> ring slot -> restore kernel ->
                 per-layer event).
wait_for_layer_load : each pending request's layer event is published when the
                 layer is enqueued; the model's current stream waits on it (a host wait
                 only while the codec has not yet decoded that layer).

Layout policies: 'byte' / 'bit' (plane format origami_planes_v1) and 'raw' (the
reference's raw-bytes layout: gathered blocks in 1 MiB chunks, RawBytesTensorAdapter
metadata, quantization/raw_tensor.py:100-122).
"""
from __future__ import annotations

import hashlib
import json
import threading
import zlib
from concurrent.futures import Future, ThreadPoolExecutor
from typing import Any

import numpy as np
import torch

from origami_b200.layer import gather_blocks, raw_chunk_bounds
from origami_b200.metadata import (ChunkLayout, ChunkRecord, LayerPayload, OrigamiConnectorMetadata, OrigamiPayload,
                                   OrigamiRestoreRequest, OrigamiSaveRequest)
from origami_b200.pipeline import RestorePipeline, SavePipeline
from origami_b200.planes import FORMAT_NAME, LayerFormat, PlaneSpec, plane_spec

NATIVE_LAYOUT_KEY = "origami_native_layout"


def _layer_index(layer_name: str) -> int:
    digits = ""
    for ch in reversed(layer_name):
        if ch.isdigit():
            digits = ch + digits
        elif digits:
            break
    return int(digits) if digits else 0


class InMemoryStore:
    """Process-local artifact store (the reference's InMemoryOrigamiStore, store.py:153-173)."""

    def __init__(self):
        self._data: dict[str, OrigamiPayload] = {}
        self._lock = threading.Lock()

    def put(self, payload: OrigamiPayload) -> None:
        with self._lock:
            self._data[payload.cache_key] = payload

    def get(self, cache_key: str) -> OrigamiPayload:
        with self._lock:
            if cache_key not in self._data:
                raise KeyError(f"Origami artifact {cache_key!r} not found")
            return self._data[cache_key]

    def contains(self, cache_key: str) -> bool:
        with self._lock:
            return cache_key in self._data


class PinnedPool:
    """Reusable pinned host buffers; a buffer returns to the pool once the CUDA event
    guarding its last copy has completed."""

    def __init__(self):
        self._free: dict[int, list[torch.Tensor]] = {}
        self._pending: list[tuple[torch.cuda.Event, torch.Tensor]] = []
        self._lock = threading.Lock()

    def take(self, nbytes: int) -> torch.Tensor:
        size = max(16, (int(nbytes) + 4095) // 4096 * 4096)
        with self._lock:
            still = []
            for ev, buf in self._pending:
                if ev.query():
                    self._free.setdefault(buf.numel(), []).append(buf)
                else:
                    still.append((ev, buf))
            self._pending = still
            free = self._free.get(size)
            if free:
                return free.pop()
        return torch.empty((size,), dtype=torch.uint8, pin_memory=True)

    def release_after(self, buf: torch.Tensor, event: torch.cuda.Event | None) -> None:
        with self._lock:
            if event is None:
                self._free.setdefault(buf.numel(), []).append(buf)
            else:
                self._pending.append((event, buf))


class OrigamiB200Worker:
    def __init__(self, *, layout_policy: str = "byte", chunk_min_bytes: int = 1 << 20,
                 chunk_target_bytes: int = 1 << 20, chunk_max_bytes: int = 1 << 20, lossless_backend: str = "zlib",
                 threads: int = 8, pipeline_slots: int = 3, store: InMemoryStore | None = None,
                 device: torch.device | str | None = None):
        if lossless_backend not in {"zlib", "raw"}:
            raise ValueError(f"Unsupported Origami CPU lossless backend {lossless_backend!r}")
        if not chunk_min_bytes <= chunk_target_bytes <= chunk_max_bytes or chunk_min_bytes <= 0:
            raise ValueError("Origami chunk sizes must satisfy 0 < min <= target <= max")
        self.layout_policy = str(layout_policy).lower()
        self.chunk_sizes = (int(chunk_min_bytes), int(chunk_target_bytes), int(chunk_max_bytes))
        self.backend = lossless_backend
        self.store = store or InMemoryStore()
        self.device = torch.device(device or "cuda")
        self.pipeline_slots = int(pipeline_slots)
        self.kv_caches: dict[str, torch.Tensor] = {}
        self._executor = ThreadPoolExecutor(max_workers=max(1, threads))
        self._codec_pool = ThreadPoolExecutor(max_workers=max(1, threads))
        self._pinned = PinnedPool()
        self._formats: dict[tuple, LayerFormat] = {}
        self._restore_pipe: RestorePipeline | None = None
        self._save_pipe: SavePipeline | None = None
        self._pipe_lock = threading.Lock()
        self._retired: list = []
        self._metadata: OrigamiConnectorMetadata | None = None
        self._pending_layer_futures: dict[str, list[Future]] = {}
        self._pending_request_layer_futures: dict[str, list[Future]] = {}
        self._restore_futures: dict[Future, str] = {}
        self._save_futures: list[Future] = []
        self._save_payloads: dict[str, OrigamiPayload] = {}
        self.host_waits = 0  # wait_for_layer_load calls that found a layer still being decoded

    # ------------------------------------------------------------------ setup
    def register_kv_caches(self, kv_caches: dict[str, torch.Tensor]) -> None:
        for name, t in kv_caches.items():
            if t.dim() != 5 or not t.is_cuda:
                raise ValueError(f"KV cache {name!r} must be a 5-D CUDA tensor")
        self.kv_caches = dict(kv_caches)

    def _planes(self, dtype: torch.dtype) -> PlaneSpec:
        return plane_spec(self.layout_policy, dtype)

    def _format(self, T: int, H: int, D: int, planes: PlaneSpec, layer_index: int = 0) -> LayerFormat:
        key = (T, H, D, planes.name, self.chunk_sizes)
        fmt = self._formats.get(key)
        if fmt is None:
            fmt = LayerFormat(T, H, D, planes, *self.chunk_sizes)
            self._formats[key] = fmt
        return fmt

    @staticmethod
    def _geometry(kv_layer: torch.Tensor) -> tuple[int, int, int]:
        _, _, bs, h, d = kv_layer.shape  # [2, NB, bs, H, D] or [NB, 2, bs, H, D]
        return int(bs), int(h), int(d)

    def _raw_side_stream(self) -> torch.cuda.Stream:
        with self._pipe_lock:
            if getattr(self, "_raw_stream", None) is None:
                self._raw_stream = torch.cuda.Stream(self.device)
            return self._raw_stream

    def _pipes(self, nbytes: int) -> tuple[RestorePipeline, SavePipeline]:
        # A pipeline outgrown by a larger layer is retired, not freed: its ring slots may
        # still be read or written by work queued on its streams.
        with self._pipe_lock:
            if self._restore_pipe is None or self._restore_pipe.slots[0].buf.numel() < nbytes:
                if self._restore_pipe is not None:
                    self._retired.append(self._restore_pipe)
                self._restore_pipe = RestorePipeline(self.device, nbytes, self.pipeline_slots)
            if self._save_pipe is None or self._save_pipe.slots[0].buf.numel() < nbytes:
                if self._save_pipe is not None:
                    self._retired.append(self._save_pipe)
                self._save_pipe = SavePipeline(self.device, nbytes, self.pipeline_slots)
            return self._restore_pipe, self._save_pipe

    # ------------------------------------------------------------------ codec
    def _compress(self, data: np.ndarray) -> torch.Tensor:
        if self.backend == "raw":
            return torch.from_numpy(data.copy())
        c = zlib.compressobj(level=1, wbits=-15, strategy=zlib.Z_DEFAULT_STRATEGY)
        enc = c.compress(data.tobytes()) + c.flush()
        return torch.frombuffer(bytearray(enc), dtype=torch.uint8).clone()

    def _decompress_into(self, comp: torch.Tensor, out: np.ndarray) -> None:
        if self.backend == "raw":
            src = comp.numpy()
            if src.size != out.size:
                raise RuntimeError(f"Origami raw backend received {src.size} bytes, expected {out.size}")
            out[:] = src
            return
        d = zlib.decompressobj(wbits=-15)
        dec = d.decompress(comp.numpy().tobytes())
        if len(dec) != out.size:
            raise RuntimeError(f"Origami CPU lossless decoded {len(dec)} bytes, expected {out.size}")
        out[:] = np.frombuffer(dec, dtype=np.uint8)

    # ------------------------------------------------------------------ save
    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata: Any = None) -> None:
        del attn_metadata
        if self._metadata is None or not self._metadata.reqs_to_save:
            return
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(kv_layer.device))  # after the layer's KV writes
        for save in self._metadata.reqs_to_save.values():
            block_ids = save.block_ids_per_group[0] if save.block_ids_per_group else ()
            if not block_ids:
                continue
            self._save_futures.append(self._save_layer(save, layer_name, kv_layer, block_ids, ready))

    def _save_layer(self, save: OrigamiSaveRequest, layer_name: str, kv_layer: torch.Tensor, block_ids,
                    ready: torch.cuda.Event) -> Future:
        bs, H, D = self._geometry(kv_layer)
        T = int(save.num_tokens)
        ids = torch.tensor([int(b) for b in block_ids], dtype=torch.int64).pin_memory().to(self.device,
                                                                                              non_blocking=True)
        li = _layer_index(layer_name)
        if self.layout_policy == "raw":
            nb = len(block_ids)
            side = self._raw_side_stream()
            side.wait_event(ready)
            with torch.cuda.stream(side):
                gathered = gather_blocks(kv_layer, ids, stream=side)
                nbytes = gathered.numel() * gathered.element_size()
                host = self._pinned.take(nbytes)
                host[:nbytes].copy_(gathered.view(-1).view(torch.uint8), non_blocking=True)
                done = torch.cuda.Event()
                done.record(side)
            shape = list(gathered.shape)

            def finish_raw():
                done.synchronize()
                data = host[:nbytes].numpy()
                bounds = raw_chunk_bounds(nbytes)
                comps = list(self._codec_pool.map(lambda ab: self._compress(data[ab[0]:ab[1]]),
                                                  zip(bounds[:-1], bounds[1:])))
                self._pinned.release_after(host, None)
                chunks = []
                for k, (a, b, comp) in enumerate(zip(bounds[:-1], bounds[1:], comps)):
                    layout = ChunkLayout(li, 0, 1, int(a), int(b), save.token_start, save.token_start + T, int(b - a))
                    chunks.append(ChunkRecord(k, layout, self.backend, comp, int(comp.numel()), int(b - a)))
                specs = [[0, 1, int(a), int(b), 0, 1] for a, b in zip(bounds[:-1], bounds[1:])]
                meta = {"format": "raw_bytes", "dtype": str(kv_layer.dtype).replace("torch.", ""), "shape": shape,
                        "byte_count": nbytes, "origami_bits": 8, "origami_symbol_shape": [1, 1, nbytes],
                        "origami_symbol_layout": ["token", "head", "head_dim"], "num_blocks": nb,
                        NATIVE_LAYOUT_KEY: {"version": 2, "bits": 8, "source_shape": [1, 1, nbytes],
                                            "source_layout": ["token", "head", "head_dim"],
                                            "storage_layout": ["layer", "head", "head_dim", "token"],
                                            "token_count": 1, "num_heads": 1, "head_dim": nbytes,
                                            "symbol_count": nbytes, "layout_policy": "baseline", "bitpack": False,
                                            "chunk_specs": specs}}
                return save, LayerPayload(layer_name, "raw_bytes", meta, chunks)

            return self._executor.submit(finish_raw)

        fmt = self._format(T, H, D, self._planes(kv_layer.dtype), li)
        _, save_pipe = self._pipes(fmt.packed_bytes)
        host = self._pinned.take(fmt.packed_bytes)
        with self._pipe_lock:
            done = save_pipe.enqueue(kv_layer, ids, fmt, host, after=ready)

        def finish_planes():
            done.synchronize()
            data = host[: fmt.packed_bytes].numpy()
            offs = fmt.offsets
            comps = list(self._codec_pool.map(lambda k: self._compress(data[offs[k]:offs[k + 1]]),
                                              range(fmt.num_chunks)))
            self._pinned.release_after(host, None)
            chunks = []
            S = fmt.num_specs
            for k, comp in enumerate(comps):
                h0, h1, c0, c1, _t0, _t1 = (int(v) for v in fmt.specs[k % S])
                nbytes = int(offs[k + 1] - offs[k])
                layout = ChunkLayout(li, h0, h1, c0, c1, save.token_start, save.token_start + T, nbytes)
                chunks.append(ChunkRecord(k, layout, self.backend, comp, int(comp.numel()), nbytes))
            meta = {"format": FORMAT_NAME, "dtype": str(kv_layer.dtype).replace("torch.", ""),
                    "shape": [2, T, H, D], "token_count": T, "origami_bits": 8,
                    "chunk_bytes": list(self.chunk_sizes), NATIVE_LAYOUT_KEY: fmt.metadata(kv_layer.dtype)}
            return save, LayerPayload(layer_name, "origami_planes", meta, chunks)

        return self._executor.submit(finish_planes)

    def wait_for_save(self) -> None:
        for fut in self._save_futures:
            save, layer_payload = fut.result()
            payload = self._save_payloads.get(save.cache_key)
            if payload is None:
                cfg = json.dumps({"layout_policy": self.layout_policy, "chunks": self.chunk_sizes}, sort_keys=True)
                payload = OrigamiPayload(save.cache_key, save.request_id, layer_payload.quantizer,
                                         hashlib.sha256(cfg.encode()).hexdigest(), save.token_start, save.num_tokens)
                self._save_payloads[save.cache_key] = payload
            payload.layer_payloads[layer_payload.layer_name] = layer_payload
        for payload in self._save_payloads.values():
            self.store.put(payload)
        self._save_futures.clear()
        self._save_payloads.clear()

    # ------------------------------------------------------------------ restore
    def start_load_kv(self, metadata: OrigamiConnectorMetadata) -> None:
        """Queue every layer of every request to restore. A request thread decodes layer
        after layer into pinned staging (its chunks in parallel on the codec pool) and
        enqueues each on the restore pipeline as soon as it is decoded, so layer L + 1
        decodes while layer L is copied and restored; the layer's event is published the
        moment it is enqueued."""
        self._metadata = metadata
        for restore in metadata.reqs_to_restore.values():
            futs: dict[str, Future] = {}
            for layer_name in self.kv_caches:
                f: Future = Future()
                futs[layer_name] = f
                self._pending_layer_futures.setdefault(layer_name, []).append(f)
            self._pending_request_layer_futures[restore.request_id] = list(futs.values())
            rf = self._executor.submit(self._restore_request, restore, futs)
            self._restore_futures[rf] = restore.request_id

    def _restore_request(self, restore: OrigamiRestoreRequest, futs: dict[str, Future]) -> str:
        try:
            payload = self.store.get(restore.cache_key)
            ids_list = [int(b) for b in (restore.block_ids_per_group[0] if restore.block_ids_per_group else ())]
            ids_dev = torch.tensor(ids_list, dtype=torch.int64, device=self.device) if ids_list else None
            for layer_name, fut in futs.items():
                if fut.done():
                    continue
                try:
                    fut.set_result(self._restore_layer(payload, restore, layer_name, ids_list, ids_dev))
                except Exception as exc:  # noqa: BLE001
                    fut.set_exception(exc)
                    raise
            return restore.request_id
        except Exception as exc:
            for fut in futs.values():
                if not fut.done():
                    fut.set_exception(exc)
            raise

    def _restore_layer(self, payload: OrigamiPayload, restore: OrigamiRestoreRequest, layer_name: str,
                       ids_list: list[int], ids_dev: torch.Tensor | None) -> torch.cuda.Event | None:
        lp = payload.layer_payloads.get(layer_name)
        if lp is None:
            return None
        kv_cache = self.kv_caches[layer_name]
        bs, H, D = self._geometry(kv_cache)
        native = lp.quant_metadata.get(NATIVE_LAYOUT_KEY) or {}
        fmt_name = str(lp.quant_metadata.get("format"))
        want = int(restore.num_tokens)
        if fmt_name == "raw_bytes":
            nb = int(lp.quant_metadata["num_blocks"])
            nbytes = int(lp.quant_metadata["byte_count"])
            if len(ids_list) < nb:
                raise RuntimeError("Origami restore request has fewer blocks than the artifact")
            # a shorter request restores the whole blocks its tokens need (worker.py:1133-1139)
            use = min(nb, (want + bs - 1) // bs) if want > 0 else nb
            host = self._pinned.take(nbytes)
            data = host.numpy()
            bounds = [0] + [int(s[3]) for s in native["chunk_specs"]]
            list(self._codec_pool.map(lambda k: self._decompress_into(lp.chunks[k].compressed,
                                                                      data[bounds[k]:bounds[k + 1]]),
                                      range(len(lp.chunks))))
            restore_pipe, _ = self._pipes(nbytes)
            with self._pipe_lock:
                ev = restore_pipe.enqueue_raw(host, nbytes, lp.quant_metadata["shape"], kv_cache, ids_dev[:use], use)
            self._pinned.release_after(host, ev)
            return ev
        if fmt_name != FORMAT_NAME:
            raise RuntimeError(f"unsupported Origami payload format {fmt_name!r}")
        T = int(native["token_count"])
        if want <= 0 or want > T:
            want = T
        if int(native["num_heads"]) != H or int(native["head_dim"]) != D:
            raise RuntimeError("artifact heads / head_dim do not match the KV cache")
        planes = plane_spec(native["planes"], kv_cache.dtype)
        chunk_sizes = lp.quant_metadata.get("chunk_bytes", list(self.chunk_sizes))
        fmt = LayerFormat(T, H, D, planes, *chunk_sizes)
        if fmt.specs.tolist() != native["chunk_specs"] or len(lp.chunks) != fmt.num_chunks:
            raise RuntimeError("Origami native layout metadata chunk count does not match payload chunks")
        need = (want + bs - 1) // bs
        if len(ids_list) < need:
            raise RuntimeError("Origami restore request has fewer blocks than its tokens need")
        host = self._pinned.take(fmt.packed_bytes)
        data = host.numpy()
        offs = fmt.offsets
        list(self._codec_pool.map(lambda k: self._decompress_into(lp.chunks[k].compressed, data[offs[k]:offs[k + 1]]),
                                  range(fmt.num_chunks)))
        restore_pipe, _ = self._pipes(fmt.packed_bytes)
        with self._pipe_lock:
            ev = restore_pipe.enqueue(host, fmt, kv_cache, ids_dev[:need], num_tokens=want)
        self._pinned.release_after(host, ev)
        return ev

    def wait_for_layer_load(self, layer_name: str) -> None:
        """Order the model's current stream after this layer's restore. A layer that is
        already enqueued costs one stream->event wait and no host wait; only a layer whose
        chunks are still being decoded makes the caller wait for the codec (the reference
        waits on the layer's future every time, worker.py:553-572)."""
        stream = torch.cuda.current_stream(self.device)
        for fut in self._pending_layer_futures.pop(layer_name, []):
            if not fut.done():
                self.host_waits += 1
            ev = fut.result()
            if ev is not None:
                stream.wait_event(ev)

    def get_finished(self, finished_req_ids: set[str] | None = None) -> tuple[set[str], set[str]]:
        del finished_req_ids
        done_recv: set[str] = set()
        for rf in list(self._restore_futures):
            if not rf.done():
                continue
            req_id = self._restore_futures.pop(rf)
            rf.result()  # re-raise a failed restore
            layer_futs = self._pending_request_layer_futures.pop(req_id, [])
            for f in layer_futs:
                f.result()
            done_recv.add(req_id)
        return set(), done_recv

    def shutdown(self) -> None:
        self._executor.shutdown(wait=True)
        self._codec_pool.shutdown(wait=True)
