"""Head/channel chunk planner for codec-sized chunks.

Same plan as the reference planner (lossless/chunking.py:22-123): the plan decides the
chunk table of every artifact, so equal inputs must give equal chunks. A head is split
along channels into runs of about ``target_bytes`` (at least ``min_bytes``, at most
``max_bytes``); when a whole head is smaller than ``target_bytes``, adjacent whole heads
are grouped. Every chunk spans all ``token_count`` tokens.
"""
from __future__ import annotations

from dataclasses import dataclass

from origami_b200.metadata import ChunkLayout


@dataclass(frozen=True)
class PlannedChunk:
    chunk_id: int
    layout: ChunkLayout


def _span_bytes(tokens: int, channels: int, bytes_per_symbol: int) -> int:
    return max(0, int(tokens)) * max(0, int(channels)) * max(1, int(bytes_per_symbol))


def plan_head_channel_chunks(
    *,
    layer_index: int,
    num_heads: int,
    head_dim: int,
    token_count: int,
    bytes_per_symbol: int,
    min_bytes: int,
    target_bytes: int,
    max_bytes: int,
) -> list[PlannedChunk]:
    if num_heads <= 0 or head_dim <= 0 or token_count <= 0:
        return []
    per_channel = max(1, token_count * bytes_per_symbol)
    want_ch = max(1, target_bytes // per_channel)
    cap_ch = max(1, max_bytes // per_channel)
    floor_ch = max(1, min_bytes // per_channel)
    whole_head = _span_bytes(token_count, head_dim, bytes_per_symbol)

    plan: list[PlannedChunk] = []

    def emit(h0: int, h1: int, c0: int, c1: int) -> None:
        width = (h1 - h0) * (c1 - c0)
        plan.append(PlannedChunk(
            chunk_id=len(plan),
            layout=ChunkLayout(layer_index=layer_index, head_start=h0, head_end=h1,
                               channel_start=c0, channel_end=c1, token_start=0,
                               token_end=token_count,
                               unpacked_bytes=_span_bytes(token_count, width, bytes_per_symbol)),
        ))

    head = 0
    while head < num_heads:
        left = num_heads - head
        if whole_head < target_bytes and left > 1:
            # Group whole heads: as many as fit the target (and the cap), then grow
            # until the group reaches min_bytes.
            group = min(left, max(1, min(want_ch // head_dim, cap_ch // head_dim, left)))
            while group < left and _span_bytes(token_count, group * head_dim, bytes_per_symbol) < min_bytes:
                group += 1
            emit(head, head + group, 0, head_dim)
            head += group
            continue
        ch = 0
        while ch < head_dim:
            rest = head_dim - ch
            width = min(rest, max(1, min(want_ch, cap_ch)))
            if rest > width:
                width = min(max(width, floor_ch), rest)
            emit(head, head + 1, ch, ch + width)
            ch += width
        head += 1
    return plan
