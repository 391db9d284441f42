"""Seeded synthetic KV workloads with the shapes and value distributions of the
benchmark configurations (all inputs are synthetic; nothing is downloaded).

C1  CPU round trip   2 layers, 8 KV heads, D 128, block 16, 64 blocks, bf16
C2  restore          32 layers (Llama-3-8B KV), 8 heads, D 128, bf16, block 16,
                     one request of 32768 tokens, block table = seeded permutation
C3  ragged batch     16 requests, T ~ U[4096, 65536], Llama-3-8B KV, block 16,
                     interleaved block tables in a pool sized for 120 GB
C4  70B pipeline     80 layers, 8 heads, D 128, fp16, block 32, 4 x 131072 tokens
C5  save stress      Qwen2-7B KV (28 layers, 4 heads, D 128, bf16, block 16),
                     64 requests x 8192 tokens

Values: K and V ~ N(0, 1) (V ~ N(0, 0.5) in C2-C5) times a per-channel scale drawn
log-uniform in [0.1, 10]; in K, 4 channels per head are multiplied by 20 (outliers).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

SEED = 7


@dataclass(frozen=True)
class KVConfig:
    name: str
    layers: int
    heads: int
    head_dim: int
    block_size: int
    dtype: torch.dtype
    tokens: tuple[int, ...]  # tokens per request
    v_std: float = 1.0


C1 = KVConfig("C1", 2, 8, 128, 16, torch.bfloat16, (1024,), 1.0)
C2 = KVConfig("C2", 32, 8, 128, 16, torch.bfloat16, (32768,), 0.5)
C4 = KVConfig("C4", 80, 8, 128, 32, torch.float16, (131072,) * 4, 0.5)
C5 = KVConfig("C5", 28, 4, 128, 16, torch.bfloat16, (8192,) * 64, 0.5)


def c3_config(seed: int = SEED + 3) -> KVConfig:
    rng = np.random.default_rng(seed)
    toks = tuple(int(t) for t in rng.integers(4096, 65536 + 1, 16))
    return KVConfig("C3", 32, 8, 128, 16, torch.bfloat16, toks, 0.5)


def c3_pool_blocks(cfg: KVConfig, pool_bytes: float = 120e9) -> int:
    per_block = cfg.block_size * cfg.layers * 2 * cfg.heads * cfg.head_dim * 2
    return int(pool_bytes // per_block)


def channel_scales(heads: int, head_dim: int, seed: int, outliers: bool) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    scale = torch.exp(torch.empty(heads, head_dim).uniform_(np.log(0.1), np.log(10.0), generator=g))
    if outliers:
        for h in range(heads):
            idx = torch.randperm(head_dim, generator=g)[:4]
            scale[h, idx] *= 20.0
    return scale


def kv_values(tokens: int, heads: int, head_dim: int, dtype: torch.dtype, *, seed: int, v_std: float = 1.0,
              device: torch.device | str = "cpu") -> torch.Tensor:
    """[2, tokens, heads, head_dim] K/V values of one layer."""
    ks = channel_scales(heads, head_dim, seed, True).to(device)
    vs = channel_scales(heads, head_dim, seed + 1, False).to(device)
    g = torch.Generator(device=device).manual_seed(seed + 2)
    k = torch.randn((tokens, heads, head_dim), generator=g, device=device) * ks
    v = torch.randn((tokens, heads, head_dim), generator=g, device=device) * (vs * v_std)
    return torch.stack([k, v]).to(dtype)


def permuted_block_table(num_blocks: int, pool_blocks: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randperm(pool_blocks, generator=g)[:num_blocks].to(torch.int64)


def interleaved_block_tables(token_counts, block_size: int, pool_blocks: int, seed: int) -> list[torch.Tensor]:
    """Per-request block tables drawn from one shuffled pool, requests interleaved."""
    need = [(t + block_size - 1) // block_size for t in token_counts]
    if sum(need) > pool_blocks:
        raise ValueError("pool too small for the requests")
    g = torch.Generator().manual_seed(seed)
    pool = torch.randperm(pool_blocks, generator=g)[: sum(need)]
    owner = np.repeat(np.arange(len(need)), need)
    np.random.default_rng(seed).shuffle(owner)
    tables = [pool[torch.from_numpy(np.nonzero(owner == r)[0])] for r in range(len(need))]
    return [t.to(torch.int64) for t in tables]


def scatter_into_cache(cache: torch.Tensor, kv: torch.Tensor, block_ids: torch.Tensor, kv_first: bool = True) -> None:
    """Set-up helper: place [2, T, H, D] values into a paged cache through block ids."""
    T = kv.shape[1]
    if kv_first:
        _, NB, bs, H, D = cache.shape
        flat = cache.view(2, NB * bs, H, D)
    else:
        NB, _, bs, H, D = cache.shape
        flat = cache.permute(1, 0, 2, 3, 4).reshape(2, NB * bs, H, D)
    t = torch.arange(T, device=cache.device)
    rows = block_ids.to(cache.device)[t // bs] * bs + t % bs
    if kv_first:
        flat[:, rows] = kv.to(cache.device)
    else:
        view = cache.view(NB, 2, bs, H, D)
        for kvi in range(2):
            view[rows // bs, kvi, rows % bs] = kv[kvi].to(cache.device)


def tokens_from_cache(cache: torch.Tensor, block_ids: torch.Tensor, T: int, kv_first: bool = True) -> torch.Tensor:
    """Check helper: read [2, T, H, D] back out of a paged cache."""
    if kv_first:
        _, NB, bs, H, D = cache.shape
    else:
        NB, _, bs, H, D = cache.shape
    t = torch.arange(T, device=cache.device)
    blk = block_ids.to(cache.device)[t // bs]
    slot = t % bs
    if kv_first:
        return cache[:, blk, slot]
    return torch.stack([cache[blk, 0, slot], cache[blk, 1, slot]])
