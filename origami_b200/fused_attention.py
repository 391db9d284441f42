"""Compressed-prefix attention entry point of the connector (the reference's
origami/fused_attention.py:11-72): a GPU-resident quantized prefix of one layer and the
launch of the fused kernel for it."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch


@dataclass
class FusedLayerPayload:
    """GPU-resident compressed prefix for one Origami cache layer."""

    request_id: str
    cache_key: str
    layer_name: str
    quantizer: str
    symbols: torch.Tensor
    metadata: dict[str, Any]
    ready_event: torch.cuda.Event
    ref_count: int = 1

    @property
    def prefix_tokens(self) -> int:
        return int(self.metadata["token_count"])


def run_fused_prefix_attention(payload: FusedLayerPayload, *, query: torch.Tensor, kv_cache: torch.Tensor,
                               block_table: torch.Tensor, query_start_position: int, sequence_length: int,
                               softmax_scale: float, output: torch.Tensor) -> None:
    """Launch the fused online-softmax attention over the payload's quantized prefix and the
    paged suffix (fused_attention.py:29-72 of the reference)."""
    from origami_b200.lossless import native_gpu

    kwargs = dict(metadata=payload.metadata, query=query, kv_cache=kv_cache, block_table=block_table,
                  query_start_position=query_start_position, sequence_length=sequence_length,
                  softmax_scale=softmax_scale, output=output)
    if payload.quantizer == "kivi":
        native_gpu.kivi_fused_prefix_attention(payload.symbols, **kwargs)
        return
    if payload.quantizer == "kvquant":
        native_gpu.kvquant_fused_prefix_attention(payload.symbols, **kwargs)
        return
    raise ValueError(f"Unsupported Origami fused quantizer {payload.quantizer!r}")
