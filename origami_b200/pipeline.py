"""Layer-wise restore / save pipelines around the fused kernels.

RestorePipeline: packed layers live in pinned host memory (where the host codec
decompresses them). Each enqueued layer is copied host->device on a dedicated copy
stream into one slot of a small device ring (3 slots, the reference's
qat_pipeline_slots default, config.py:73), unpacked and scattered into the paged cache
on a restore stream that waits only for its own copy, and marked with a per-layer CUDA
event. The H2D copy of layer L+1 therefore overlaps the unpack/scatter of layer L and
whatever the model runs on its compute stream. ``wait_for_layer_load`` is a
stream->event wait, never a host block (the reference blocks on a future and then waits,
worker.py:553-572).

enqueue_from_bundle is the codec handoff: the host codec decodes a layer's chunks out of
the ORIGQZ1 bundle straight into a pinned staging slot (one of a ring as deep as the
device ring), which the copy stream then moves to the device; the reference instead
concatenates decoded chunks and copies them through pageable memory (worker.py:796-1049,
benchmark_utils.py:438).

SavePipeline: the mirror image: pack each layer on a save stream into a device slot
and copy it to pinned host memory on a copy stream, one event per layer for the host
codec to wait on.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from origami_b200 import _lib
from origami_b200.layer import cache_layout, pack_layer, restore_layer, scatter_blocks
from origami_b200.planes import LayerFormat


@dataclass
class _Slot:
    buf: torch.Tensor
    copied: torch.cuda.Event
    free: torch.cuda.Event
    used: bool = False


class RestorePipeline:
    """Streams are created at high priority by default: a restore gates the model's next
    layer, so its copy and kernel go ahead of work of normal priority when both wait."""

    def __init__(self, device: torch.device, slot_bytes: int, slots: int = 3, *, priority: int = -1):
        self.device = torch.device(device)
        self.copy_stream = torch.cuda.Stream(self.device, priority=priority)
        self.restore_stream = torch.cuda.Stream(self.device, priority=priority)
        n = (int(slot_bytes) + 15) // 16 * 16
        self.slots = [_Slot(torch.empty((n,), dtype=torch.uint8, device=self.device), torch.cuda.Event(),
                            torch.cuda.Event()) for _ in range(max(1, slots))]
        self._next = 0
        self.launches = 0

    def _upload(self, host: torch.Tensor, n: int) -> _Slot:
        """Copy n pinned bytes into the next ring slot on the copy stream; the restore
        stream waits for that copy only."""
        if host.device.type != "cpu" or not host.is_pinned():
            raise ValueError("host packed layer must be in pinned host memory")
        if host.numel() < n:
            raise ValueError("host packed layer is shorter than the layer format")
        slot = self.slots[self._next]
        self._next = (self._next + 1) % len(self.slots)
        if slot.buf.numel() < n:
            raise ValueError("pipeline slot smaller than the packed layer")
        if slot.used:
            self.copy_stream.wait_event(slot.free)  # previous user of the slot has been unpacked
        with torch.cuda.stream(self.copy_stream):
            slot.buf[:n].copy_(host[:n], non_blocking=True)
            slot.copied.record(self.copy_stream)
        self.restore_stream.wait_event(slot.copied)
        return slot

    def _done(self, slot: _Slot) -> torch.cuda.Event:
        self.launches += 1
        slot.free.record(self.restore_stream)
        slot.used = True
        ready = torch.cuda.Event()
        ready.record(self.restore_stream)
        return ready

    def enqueue(self, host_packed: torch.Tensor, fmt: LayerFormat, kv_layer: torch.Tensor, block_ids,
                error_count: torch.Tensor | None = None, *, num_tokens: int | None = None) -> torch.cuda.Event:
        """Queue one layer (or its first num_tokens tokens); returns the event that marks
        the layer as restored."""
        n = fmt.packed_bytes
        slot = self._upload(host_packed, n)
        restore_layer(slot.buf[:n], fmt, kv_layer, block_ids, stream=self.restore_stream, error_count=error_count,
                      num_tokens=num_tokens)
        return self._done(slot)

    def enqueue_raw(self, host_bytes: torch.Tensor, nbytes: int, shape, kv_layer: torch.Tensor, block_ids,
                    num_blocks: int, error_count: torch.Tensor | None = None) -> torch.cuda.Event:
        """Queue one raw-bytes layer (the gathered [2, n, bs, H, D] or [n, 2, bs, H, D]
        blocks): copy it into a ring slot and scatter its first num_blocks blocks into the
        cache by block table."""
        slot = self._upload(host_bytes, nbytes)
        value = slot.buf[:nbytes].view(kv_layer.dtype).view(list(shape))
        block_dim = 1 if cache_layout(kv_layer) == _lib.ORIGAMI_KV_FIRST else 0
        with torch.cuda.stream(self.restore_stream):
            if num_blocks < value.shape[block_dim]:
                value = value.narrow(block_dim, 0, num_blocks).contiguous()
            scatter_blocks(value, kv_layer, block_ids, stream=self.restore_stream, error_count=error_count)
        return self._done(slot)

    def enqueue_from_bundle(self, bundle, layer_name: str, fmt: LayerFormat, kv_layer: torch.Tensor, block_ids,
                            error_count: torch.Tensor | None = None, *, threads: int = 0) -> torch.cuda.Event:
        """Host codec -> H2D handoff: decode the layer's chunks from an ORIGQZ1 bundle
        (origami_b200.bundle.QatBundle) straight into a pinned staging slot at their packed
        offsets, then enqueue() it. The slot is reused once its previous copy has finished
        (the only host wait), so decoding layer L+1 overlaps the copy and restore of L."""
        staging = self._host_slot(fmt.packed_bytes)
        bundle.inflate_layer_into(layer_name, fmt, staging.buf[: fmt.packed_bytes], threads=threads)
        ready = self.enqueue(staging.buf, fmt, kv_layer, block_ids, error_count=error_count)
        staging.copied.record(self.copy_stream)
        staging.used = True
        return ready

    def _host_slot(self, n: int) -> _Slot:
        if not hasattr(self, "_host"):
            self._host, self._host_next = [], 0
        if len(self._host) < len(self.slots):
            size = max(n, self.slots[0].buf.numel())
            self._host.append(_Slot(torch.empty((size,), dtype=torch.uint8, pin_memory=True), torch.cuda.Event(),
                                    torch.cuda.Event()))
            slot = self._host[-1]
        else:
            slot = self._host[self._host_next]
            self._host_next = (self._host_next + 1) % len(self._host)
            if slot.used:
                slot.copied.synchronize()  # its bytes have reached the device
        if slot.buf.numel() < n:
            raise ValueError("pinned staging slot smaller than the packed layer")
        return slot

    @staticmethod
    def wait_for_layer_load(event: torch.cuda.Event, stream: torch.cuda.Stream | None = None) -> None:
        (stream or torch.cuda.current_stream()).wait_event(event)

    def synchronize(self) -> None:
        self.copy_stream.synchronize()
        self.restore_stream.synchronize()


class SavePipeline:
    def __init__(self, device: torch.device, slot_bytes: int, slots: int = 3):
        self.device = torch.device(device)
        self.save_stream = torch.cuda.Stream(self.device)
        self.copy_stream = torch.cuda.Stream(self.device)
        n = (int(slot_bytes) + 15) // 16 * 16
        self.slots = [_Slot(torch.empty((n,), dtype=torch.uint8, device=self.device), torch.cuda.Event(),
                            torch.cuda.Event()) for _ in range(max(1, slots))]
        self._next = 0
        self.launches = 0

    def enqueue(self, kv_layer: torch.Tensor, block_ids, fmt: LayerFormat, host_out: torch.Tensor,
                *, after: torch.cuda.Event | None = None,
                error_count: torch.Tensor | None = None) -> torch.cuda.Event:
        """Pack one layer into pinned `host_out`; returns the event after the D2H copy.

        `after` (optional) is the event the layer's KV is complete at (e.g. recorded on
        the model stream after attention wrote it)."""
        if not host_out.is_pinned():
            raise ValueError("host output must be pinned")
        n = fmt.packed_bytes
        slot = self.slots[self._next]
        self._next = (self._next + 1) % len(self.slots)
        if slot.used:
            self.save_stream.wait_event(slot.free)
        if after is not None:
            self.save_stream.wait_event(after)
        pack_layer(kv_layer, block_ids, fmt, out=slot.buf[:n], stream=self.save_stream, error_count=error_count)
        self.launches += 1
        slot.copied.record(self.save_stream)
        self.copy_stream.wait_event(slot.copied)
        with torch.cuda.stream(self.copy_stream):
            host_out[:n].copy_(slot.buf[:n], non_blocking=True)
        slot.free.record(self.copy_stream)
        slot.used = True
        done = torch.cuda.Event()
        done.record(self.copy_stream)
        return done
