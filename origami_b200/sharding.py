"""KV-head sharding across ranks (vLLM tensor parallelism).

Rank r of N owns heads [r*H/N, (r+1)*H/N) of every layer and restores only those into
its own head-sliced paged cache; its chunk plan is made with num_heads = H/N, so no
chunk straddles two ranks. No collective touches the data path.
"""
from __future__ import annotations

from origami_b200.planes import BYTE_PLANES, LayerFormat, PlaneSpec


def head_range(rank: int, world: int, num_heads: int) -> tuple[int, int]:
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if num_heads % world:
        raise ValueError(f"{num_heads} KV heads do not shard evenly over {world} ranks")
    per = num_heads // world
    return rank * per, (rank + 1) * per


def shard_format(rank: int, world: int, num_tokens: int, num_heads: int, head_dim: int,
                 planes: PlaneSpec = BYTE_PLANES, chunk_bytes: int = 1 << 20, layer_index: int = 0) -> LayerFormat:
    h0, h1 = head_range(rank, world, num_heads)
    return LayerFormat(num_tokens, h1 - h0, head_dim, planes, chunk_bytes, chunk_bytes, chunk_bytes, layer_index)
