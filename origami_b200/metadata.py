"""Chunk-table records of the Origami artifact.

Field-for-field the records of the reference connector (metadata.py:22-61 in the
reference's origami package), so payloads written by either side stay interchangeable.
"""
from __future__ import annotations

import sys

from dataclasses import dataclass, field
from typing import Any

import torch


@dataclass(frozen=True)
class ChunkLayout:
    layer_index: int
    head_start: int
    head_end: int
    channel_start: int
    channel_end: int
    token_start: int
    token_end: int
    unpacked_bytes: int

    def spec(self) -> list[int]:
        """The [h0, h1, c0, c1, t0, t1] spec row of this chunk (worker.py:2207-2216)."""
        return [self.head_start, self.head_end, self.channel_start, self.channel_end,
                self.token_start, self.token_end]


@dataclass
class ChunkRecord:
    chunk_id: int
    layout: ChunkLayout
    codec: str
    compressed: torch.Tensor
    compressed_bytes: int
    unpacked_bytes: int


@dataclass
class LayerPayload:
    layer_name: str
    quantizer: str
    quant_metadata: dict[str, Any]
    chunks: list[ChunkRecord] = field(default_factory=list)


@dataclass
class OrigamiPayload:
    cache_key: str
    request_id: str
    quantizer: str
    quantizer_config_hash: str
    token_start: int
    token_count: int
    layer_payloads: dict[str, LayerPayload] = field(default_factory=dict)
    metadata: dict[str, Any] = field(default_factory=dict)


@dataclass(frozen=True)
class OrigamiRestoreRequest:
    request_id: str
    cache_key: str
    block_ids_per_group: tuple[tuple[int, ...], ...]
    num_tokens: int
    lossless_path: str = "cpu"
    metric_request_id: str | None = None


@dataclass(frozen=True)
class OrigamiSaveRequest:
    request_id: str
    cache_key: str
    block_ids_per_group: tuple[tuple[int, ...], ...]
    num_tokens: int
    token_start: int = 0


_ConnectorMetadataBase: type = object
if "vllm" in sys.modules:  # inside a vLLM process: derive from its connector metadata base
    try:
        from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorMetadata as _ConnectorMetadataBase
    except Exception:  # noqa: BLE001
        _ConnectorMetadataBase = object


@dataclass
class OrigamiConnectorMetadata(_ConnectorMetadataBase):
    """What the scheduler side hands the worker each step (metadata.py:74-92): the
    requests to restore / save, the GPU lossless share, and the fused-attention requests
    with their query positions, counts, batch indices, codecs and prefix lengths."""

    reqs_to_restore: dict[str, OrigamiRestoreRequest] = field(default_factory=dict)
    reqs_to_save: dict[str, OrigamiSaveRequest] = field(default_factory=dict)
    gpu_lossless_ratio: int = 0
    fused_request_ids: tuple[str, ...] = ()
    fused_query_start_positions: dict[str, int] = field(default_factory=dict)
    fused_query_token_counts: dict[str, int] = field(default_factory=dict)
    fused_request_indices: dict[str, int] = field(default_factory=dict)
    fused_codecs: dict[str, str] = field(default_factory=dict)
    fused_prefix_lengths: dict[str, int] = field(default_factory=dict)
