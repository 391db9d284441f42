"""Seeded cases of the fused prefix attention (reference fused_prefix_attention_cuda,
bitpack_layout_cuda.cpp:716-890 / cu:873-1091), shared by the golden-vector generator
(make_ref_attention_vectors.py, run on a B200 against the reference extension), the CPU
oracle tests and the GPU tests.

Symbol streams are seeded random bytes (every byte pattern is a valid dense stream; 3-bit
symbols are nibble-packed and the mask drops each nibble's top bit). Scales and zeros put
dequantized values near [-1, 1]. Queries and caches are fp16 / bf16 bit patterns (uint16)
of N(0, 1) values. The bytestream is [pad][key stream][pad][value stream][pad], so the
streams start at odd offsets.
"""
from __future__ import annotations

import math

import numpy as np

D = 128


def _bits16(x: np.ndarray, bf16: bool) -> np.ndarray:
    x = x.astype(np.float32)
    if bf16:
        u = x.view(np.uint32).astype(np.uint64)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return x.astype(np.float16).view(np.uint16)


def packed_symbol_bytes(bits: int, symbols: int) -> int:
    return (symbols + 1) // 2 if bits == 3 else (symbols * bits + 7) // 8


def attention_case(name, seed, *, codec, bits, prefix, sink=0, group_size=1, kv_heads=2, query_heads=4,
                   query_tokens=1, query_start=None, seq_len=None, block_size=16, blocks_first=False,
                   query_bf16=False, cache_bf16=None, bad_blocks=False, spare_blocks=3):
    rng = np.random.default_rng(seed)
    cache_bf16 = query_bf16 if cache_bf16 is None else cache_bf16
    query_start = prefix if query_start is None else query_start
    seq_len = query_start + query_tokens if seq_len is None else seq_len
    C = kv_heads * D
    sink = sink if codec == 0 else 0
    body = prefix - sink if codec == 0 else prefix
    nbytes = packed_symbol_bytes(bits, body * C)
    pads = [int(x) for x in rng.integers(1, 9, 3)]
    key_offset = pads[0]
    value_offset = key_offset + nbytes + pads[1]
    stream = rng.integers(0, 256, value_offset + nbytes + pads[2], dtype=np.uint8)
    levels = (1 << bits) - 1

    def scale(shape):
        return (rng.uniform(0.5, 1.5, shape) * 2.0 / levels).astype(np.float16)

    def zero(shape):
        return rng.uniform(-1.2, -0.8, shape).astype(np.float16)

    if codec == 0:
        kg = (body + group_size - 1) // group_size
        vg = (C + group_size - 1) // group_size
        meta = dict(key_scale=scale((kg, C)), key_zero=zero((kg, C)), value_scale=scale((body, vg)),
                    value_zero=zero((body, vg)),
                    key_sink=rng.normal(0, 1, (sink, C)).astype(np.float16),
                    value_sink=rng.normal(0, 1, (sink, C)).astype(np.float16))
    else:
        meta = dict(key_scale=scale(C), key_zero=zero(C), value_scale=scale(prefix), value_zero=zero(prefix),
                    key_sink=np.zeros(0, np.float16), value_sink=np.zeros(0, np.float16))
    logical = (seq_len + block_size - 1) // block_size
    nb = logical + spare_blocks
    table = rng.permutation(nb)[:logical].astype(np.int32)
    if bad_blocks and logical >= 3:
        suffix_blocks = list(range(prefix // block_size + 1, logical))
        if suffix_blocks:
            table[suffix_blocks[0]] = -1
            table[suffix_blocks[-1]] = nb + 5
    shape = (nb, 2, block_size, kv_heads, D) if blocks_first else (2, nb, block_size, kv_heads, D)
    cache = _bits16(rng.normal(0, 1, shape), cache_bf16)
    query = _bits16(rng.normal(0, 1, (query_tokens, query_heads, D)), query_bf16)
    return dict(name=name, codec=codec, bits=bits, group_size=group_size, sink_tokens=sink, prefix_tokens=prefix,
                bytestream=stream, key_offset=key_offset, key_bytes=nbytes, value_offset=value_offset,
                value_bytes=nbytes, query=query, query_bf16=query_bf16, kv_cache=cache, cache_bf16=cache_bf16,
                blocks_first=blocks_first, block_table=table, query_start=query_start, sequence_length=seq_len,
                softmax_scale=1.0 / math.sqrt(D), **meta)


def cases() -> list[dict]:
    c = attention_case
    return [
        # the reference test's shapes: prefix 19, 2 KV heads, 4 query heads, one query token
        c("kivi_b2_f16_decode", 1, codec=0, bits=2, prefix=19, sink=3, group_size=7),
        c("kivi_b3_bf16_decode", 2, codec=0, bits=3, prefix=19, sink=3, group_size=7, query_bf16=True),
        c("kivi_b4_f16_q16", 3, codec=0, bits=4, prefix=19, sink=3, group_size=7, query_tokens=16),
        c("kivi_b8_bf16_decode", 4, codec=0, bits=8, prefix=19, sink=3, group_size=7, query_bf16=True),
        c("kvquant_b2_f16_decode", 5, codec=1, bits=2, prefix=19),
        c("kvquant_b3_bf16_decode", 6, codec=1, bits=3, prefix=19, query_bf16=True),
        c("kvquant_b4_f16_q16", 7, codec=1, bits=4, prefix=19, query_tokens=16),
        c("kvquant_b8_bf16_decode", 8, codec=1, bits=8, prefix=19, query_bf16=True),
        c("kivi_b4_f16_q128", 9, codec=0, bits=4, prefix=19, sink=3, group_size=7, query_tokens=128),
        # long prefixes: split key ranges, body octets, sink tokens, a suffix in the cache
        c("kivi_b2_long_decode", 10, codec=0, bits=2, prefix=1000, sink=32, group_size=32, kv_heads=8,
          query_heads=32, query_start=1199, seq_len=1200),
        c("kvquant_b4_ragged_gap", 11, codec=1, bits=4, prefix=777, kv_heads=4, query_heads=16, query_tokens=3,
          query_start=827, seq_len=850),
        c("kivi_b3_blocks_first_mixed_bad", 12, codec=0, bits=3, prefix=300, sink=8, group_size=16, kv_heads=2,
          query_heads=8, query_tokens=4, query_start=340, seq_len=400, blocks_first=True, query_bf16=True,
          cache_bf16=False, bad_blocks=True),
        c("kvquant_b8_mha_q5_bs32", 13, codec=1, bits=8, prefix=256, kv_heads=3, query_heads=3, query_tokens=5,
          block_size=32, cache_bf16=True),
        c("kivi_b4_gs1_p128", 14, codec=0, bits=4, prefix=128, sink=0, group_size=1, kv_heads=1, query_heads=2,
          query_tokens=9, query_start=160),
        c("kivi_b2_prefill_q40", 15, codec=0, bits=2, prefix=513, sink=16, group_size=64, kv_heads=2,
          query_heads=16, query_tokens=40, query_start=513),
        # decode shapes whose groups fit the symbol-operand kernel: key groups of 64 / 96 / 128
        # tokens (up to 3 per 128-key tile, boundaries off the tiles), value channel groups
        # within a head, sinks off the 8-key octets
        c("kivi_b2_g64_decode", 16, codec=0, bits=2, prefix=2000, sink=128, group_size=64, kv_heads=8,
          query_heads=32, query_start=2099, seq_len=2100, query_bf16=True),
        c("kivi_b4_g128_q4_ragged", 17, codec=0, bits=4, prefix=777, sink=5, group_size=128, kv_heads=2,
          query_heads=8, query_tokens=4, query_start=800, seq_len=820),
        c("kivi_b8_g64_blocks_first_mixed_bad", 18, codec=0, bits=8, prefix=300, sink=12, group_size=64,
          kv_heads=4, query_heads=4, query_tokens=3, query_start=330, seq_len=360, blocks_first=True,
          query_bf16=True, cache_bf16=False, bad_blocks=True),
        c("kivi_b3_g96_q2", 19, codec=0, bits=3, prefix=500, sink=7, group_size=96, kv_heads=3, query_heads=6,
          query_tokens=2, query_start=520, seq_len=540),
    ]


def _oracle_module():
    """oracle/oracle.py, whether oracle/ itself or the repository root is on sys.path."""
    import oracle

    if not hasattr(oracle, "fused_prefix_attention"):
        from oracle import oracle
    return oracle


def run_oracle(case: dict) -> np.ndarray:
    o = _oracle_module()
    return o.fused_prefix_attention(
        case["bytestream"], case["key_offset"], case["key_bytes"], case["value_offset"], case["value_bytes"],
        case["codec"], case["bits"], case["group_size"], case["sink_tokens"], case["key_scale"], case["key_zero"],
        case["value_scale"], case["value_zero"], case["key_sink"], case["value_sink"], case["query"],
        case["query_bf16"], case["kv_cache"], case["cache_bf16"], case["blocks_first"], case["block_table"],
        case["prefix_tokens"], case["query_start"], case["sequence_length"], case["softmax_scale"])


def to_float(bits16: np.ndarray, bf16: bool) -> np.ndarray:
    if bf16:
        return (bits16.astype(np.uint32) << 16).view(np.float32)
    return bits16.view(np.float16).astype(np.float32)
