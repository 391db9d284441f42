"""Seeded cases of the quantized restore ops (CacheGen and KIVI dequantize-to-cache, CacheGen
unpack), shared by the golden-vector generator (make_ref_quant_vectors.py, run on a B200
against the reference extension) and the tests.

Every case is a dict of numpy inputs plus scalar parameters. Caches are uint16 arrays of
fp16 / bf16 bit patterns filled with seeded noise, so rows an op must not touch are
checked too. Symbol streams are seeded random bytes: every byte pattern is a valid dense
LSB-first stream. The bytestream holds [pad][key stream][pad][value stream][pad], so the
streams start at odd offsets.
"""
from __future__ import annotations

import numpy as np


def _nbytes(symbols: int, bits: int) -> int:
    return (symbols * bits + 7) // 8


def _layout(rng, key_len: int, value_len: int):
    pads = [int(x) for x in rng.integers(1, 9, 3)]
    key_offset = pads[0]
    value_offset = key_offset + key_len + pads[1]
    total = value_offset + value_len + pads[2]
    return rng.integers(0, 256, total, dtype=np.uint8), key_offset, value_offset


def _cache(rng, nb: int, bs: int, H: int, D: int, blocks_first: bool) -> np.ndarray:
    shape = (nb, 2, bs, H, D) if blocks_first else (2, nb, bs, H, D)
    return rng.integers(0, 1 << 16, shape, dtype=np.uint16)


def _ids(rng, needed: int, nb: int, bad: bool) -> np.ndarray:
    ids = rng.permutation(nb)[:needed].astype(np.int64)
    if bad and needed >= 2:
        ids[1] = -1
        ids[-1] = nb
    return ids


def _meta(rng, shape, dtype, lo=-2.0, hi=2.0) -> np.ndarray:
    return rng.uniform(lo, hi, shape).astype(dtype)


def cachegen_cache_case(name, seed, T, H, D, bs, key_bits, value_bits, key_bins, value_bins, max_dtype, out_bf16,
                        blocks_first, spare_blocks=2, bad=False, trunc=(0, 0)):
    rng = np.random.default_rng(seed)
    C = H * D
    klen = max(_nbytes(T * C, key_bits) - trunc[0], 0)
    vlen = max(_nbytes(T * C, value_bits) - trunc[1], 0)
    stream, koff, voff = _layout(rng, klen, vlen)
    needed = (T + bs - 1) // bs
    nb = needed + spare_blocks
    return dict(kind="cg_cache", name=name, bytestream=stream, key_offset=koff, key_bytes=klen, value_offset=voff,
                value_bytes=vlen, key_bits=key_bits, value_bits=value_bits, key_bins=key_bins, value_bins=value_bins,
                max_key=np.exp(rng.normal(0, 1, T)).astype(max_dtype),
                max_value=np.exp(rng.normal(0, 1, T)).astype(max_dtype),
                cache=_cache(rng, nb, bs, H, D, blocks_first), blocks_first=blocks_first,
                block_ids=_ids(rng, needed, nb, bad), tokens=T, heads=H, head_dim=D, out_bf16=out_bf16)


def cachegen_unpack_case(name, seed, T, H, D, key_bits, value_bits, key_bins, value_bins, max_dtype, trunc=0,
                         trunc_stream=-1):
    """`trunc` bytes are cut from stream `trunc_stream` (default: the last one)."""
    rng = np.random.default_rng(seed)
    L = len(key_bits)
    bits = list(key_bits) + list(value_bits)
    cut = trunc_stream % len(bits)
    lens = [max(_nbytes(T * H * D, b) - (trunc if i == cut else 0), 0) for i, b in enumerate(bits)]
    offsets = [0]
    for n in lens:
        offsets.append(offsets[-1] + n + int(rng.integers(0, 5)))
    stream = rng.integers(0, 256, offsets[-1] + 3, dtype=np.uint8)
    # offsets[i + 1] - offsets[i] is the stream length the kernel sees (gaps included)
    return dict(kind="cg_unpack", name=name, bytestream=stream, offsets=np.asarray(offsets, np.int64),
                bits=np.asarray(bits, np.int64), key_bins=np.asarray(key_bins, np.int64),
                value_bins=np.asarray(value_bins, np.int64),
                max_key=np.exp(rng.normal(0, 1, L * T)).astype(max_dtype),
                max_value=np.exp(rng.normal(0, 1, L * T)).astype(max_dtype), tokens=T, heads=H, head_dim=D)


def kivi_case(name, seed, T, sink, H, D, bs, bits, group_size, meta_dtype, out_bf16, blocks_first, spare_blocks=2,
              bad=False, trunc=(0, 0)):
    rng = np.random.default_rng(seed)
    C = H * D
    body = T - sink
    klen = max(_nbytes(body * C, bits) - trunc[0], 0)
    vlen = max(_nbytes(body * C, bits) - trunc[1], 0)
    stream, koff, voff = _layout(rng, klen, vlen)
    key_groups = (body + group_size - 1) // group_size
    value_groups = (C + group_size - 1) // group_size
    needed = (T + bs - 1) // bs
    nb = needed + spare_blocks
    return dict(kind="kivi", name=name, bytestream=stream, key_offset=koff, key_bytes=klen, value_offset=voff,
                value_bytes=vlen, bits=bits, group_size=group_size, sink_tokens=sink,
                key_scale=_meta(rng, key_groups * C, meta_dtype, 0.001, 0.5),
                key_zero=_meta(rng, key_groups * C, meta_dtype),
                value_scale=_meta(rng, body * value_groups, meta_dtype, 0.001, 0.5),
                value_zero=_meta(rng, body * value_groups, meta_dtype),
                key_sink=_meta(rng, sink * C, meta_dtype, -8.0, 8.0),
                value_sink=_meta(rng, sink * C, meta_dtype, -8.0, 8.0),
                cache=_cache(rng, nb, bs, H, D, blocks_first), blocks_first=blocks_first,
                block_ids=_ids(rng, needed, nb, bad), tokens=T, heads=H, head_dim=D, out_bf16=out_bf16)


def cases() -> list[dict]:
    f16, f32 = np.float16, np.float32
    return [
        cachegen_cache_case("cg_small_f16", 101, 37, 2, 16, 16, 5, 4, 32, 16, f16, False, False),
        cachegen_cache_case("cg_bf16_f32max_blocks_first_bad_ids", 102, 50, 3, 8, 8, 3, 8, 12, 256, f32, True, True,
                            bad=True),
        cachegen_cache_case("cg_center_zero", 103, 20, 1, 24, 16, 1, 2, 2, 3, f16, False, False),
        cachegen_cache_case("cg_truncated_streams", 104, 40, 2, 32, 16, 7, 6, 100, 64, f16, True, False,
                            trunc=(11, 1)),
        cachegen_cache_case("cg_llama_shape", 105, 40, 8, 128, 16, 5, 4, 32, 16, f16, True, False),
        cachegen_cache_case("cg_odd_channels", 106, 33, 3, 10, 4, 4, 5, 16, 20, f32, False, True),
        cachegen_unpack_case("cgu_two_layers", 201, 20, 2, 16, [5, 4], [3, 8], [32, 12], [16, 256], f16),
        cachegen_unpack_case("cgu_f32_head_dim12_truncated", 202, 9, 3, 12, [6], [2], [64], [4], f32, trunc=5),
        # 8-bit streams cut short: the reference reads on into the bytes that follow
        cachegen_cache_case("cg_b8_short_key_stream", 107, 24, 2, 16, 16, 8, 8, 256, 200, f16, False, False,
                            trunc=(9, 0)),
        cachegen_unpack_case("cgu_b8_short_first_stream", 203, 10, 2, 8, [8], [8], [256], [130], f16, trunc=6,
                             trunc_stream=0),
        kivi_case("kivi_b2_tiled", 301, 150, 16, 2, 64, 16, 2, 32, f16, False, False),
        kivi_case("kivi_b4_ragged_sink_group", 302, 77, 5, 3, 16, 8, 4, 12, f32, True, True, bad=True),
        kivi_case("kivi_all_sink", 303, 40, 40, 1, 64, 16, 8, 64, f16, False, False),
        kivi_case("kivi_b3_no_sink", 304, 300, 0, 1, 128, 16, 3, 128, f16, True, False),
        kivi_case("kivi_b5_d256", 305, 70, 8, 2, 256, 32, 5, 64, f16, False, True),
        kivi_case("kivi_b8_group7_truncated", 306, 50, 16, 2, 64, 16, 8, 7, f32, False, False, trunc=(3, 0)),
        kivi_case("kivi_b1_d128_bad_ids", 307, 129, 8, 2, 128, 16, 1, 64, f16, True, True, bad=True),
    ]


def _oracle_module():
    """oracle/oracle.py, whether oracle/ itself or the repository root is on sys.path."""
    import oracle

    if not hasattr(oracle, "kivi_to_cache"):
        from oracle import oracle
    return oracle


def run_oracle(case: dict) -> np.ndarray:
    """The CPU oracle's output for a case (test infrastructure)."""
    oracle = _oracle_module()

    c = case
    if c["kind"] == "cg_cache":
        out = c["cache"].copy()
        oracle.cachegen_to_cache(c["bytestream"], c["key_offset"], c["key_bytes"], c["value_offset"],
                                 c["value_bytes"], c["key_bits"], c["value_bits"], c["key_bins"], c["value_bins"],
                                 c["max_key"], c["max_value"], out, c["blocks_first"], c["block_ids"], c["tokens"],
                                 c["out_bf16"])
        return out
    if c["kind"] == "cg_unpack":
        return oracle.cachegen_unpack(c["bytestream"], c["offsets"], c["bits"], c["key_bins"], c["value_bins"],
                                      c["max_key"], c["max_value"], c["tokens"], c["heads"], c["head_dim"])
    out = c["cache"].copy()
    oracle.kivi_to_cache(c["bytestream"], c["key_offset"], c["key_bytes"], c["value_offset"], c["value_bytes"],
                         c["bits"], c["group_size"], c["sink_tokens"], c["key_scale"], c["key_zero"],
                         c["value_scale"], c["value_zero"], c["key_sink"], c["value_sink"], out, c["blocks_first"],
                         c["block_ids"], c["tokens"], c["out_bf16"])
    return out
