"""CPU oracle of the quantized restore ops (CacheGen, KIVI) against the reference kernels'
own outputs (tests/golden/ref_quant_vectors.npz, made on a B200 by
make_ref_quant_vectors.py) and against an independent numpy restatement."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))

from quant_cases import _oracle_module, cases, run_oracle  # noqa: E402

oracle = _oracle_module()

VECTORS = GOLDEN / "ref_quant_vectors.npz"
CASES = cases()


def _f32(a: np.ndarray) -> np.ndarray:
    return a.astype(np.float32)


def _to_out(v: np.ndarray, bf16: bool) -> np.ndarray:
    """float32 -> fp16 / bf16 bit patterns, round to nearest even, NaN -> 0x7FFF."""
    v = v.astype(np.float32)
    if bf16:
        u = v.view(np.uint32).astype(np.uint64)
        out = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    else:
        with np.errstate(over="ignore"):
            out = v.astype(np.float16).view(np.uint16)
    out[np.isnan(v)] = 0x7FFF
    return out


def _symbols(stream: np.ndarray, nbytes: int, index: np.ndarray, bits: int) -> np.ndarray:
    """`stream` runs to the bytestream's end; 8-bit symbols may read all of it (the
    reference's unchecked src[index]), narrower ones only `nbytes`."""
    if bits == 8:
        nbytes = len(stream)
    padded = np.zeros(len(stream) + 2, dtype=np.uint16)
    padded[:nbytes] = stream[:nbytes]
    bit = index * bits
    byte = bit >> 3
    w = padded[np.minimum(byte, len(padded) - 2)] | (padded[np.minimum(byte + 1, len(padded) - 1)] << 8)
    w = np.where(byte < nbytes, w, 0)
    return ((w >> (bit & 7)) & ((1 << bits) - 1)).astype(np.uint32)


def _cache_rows(c):
    """(token, kv) -> cache row slices: yields token, kv, block, offset."""
    bs = c["cache"].shape[2]
    nb = c["cache"].shape[0] if c["blocks_first"] else c["cache"].shape[1]
    for t in range(c["tokens"]):
        blk = c["block_ids"][t // bs]
        if blk < 0 or blk >= nb:
            continue
        for kv in range(2):
            yield t, kv, blk, t % bs


def _put(cache, blocks_first, kv, blk, off, row):
    if blocks_first:
        cache[blk, kv, off] = row
    else:
        cache[kv, blk, off] = row


def numpy_restatement(c) -> np.ndarray:
    """The same ops written with numpy vector arithmetic (float32 throughout)."""
    H, D = c["heads"], c["head_dim"]
    C = H * D
    if c["kind"] == "cg_unpack":
        L = len(c["bits"]) // 2
        out = np.zeros((L, 2, H, c["tokens"], D), dtype=np.uint16)
        for s in range(2 * L):
            kv, layer = (1, s - L) if s >= L else (0, s)
            stream = c["bytestream"][c["offsets"][s]:]
            n = int(c["offsets"][s + 1] - c["offsets"][s])
            bins = (c["value_bins"] if kv else c["key_bins"])[layer]
            center = np.float32(bins // 2 - 1)
            mx = _f32((c["max_value"] if kv else c["max_key"])[layer * c["tokens"]:(layer + 1) * c["tokens"]])
            idx = np.arange(c["tokens"] * C, dtype=np.int64)
            sym = _symbols(stream, n, idx, int(c["bits"][s])).astype(np.float32)
            with np.errstate(divide="ignore", invalid="ignore"):
                q = (sym - center) / center
            v = (q.reshape(c["tokens"], C) * mx[:, None]).reshape(c["tokens"], H, D).transpose(1, 0, 2)
            out[layer, kv] = _to_out(v, False)
        return out
    cache = c["cache"].copy()
    if c["kind"] == "cg_cache":
        for t, kv, blk, off in _cache_rows(c):
            stream = c["bytestream"][c["value_offset"] if kv else c["key_offset"]:]
            n = c["value_bytes"] if kv else c["key_bytes"]
            bits = c["value_bits"] if kv else c["key_bits"]
            center = np.float32((c["value_bins"] if kv else c["key_bins"]) // 2 - 1)
            mx = np.float32((c["max_value"] if kv else c["max_key"])[t])
            sym = _symbols(stream, n, t * C + np.arange(C, dtype=np.int64), bits).astype(np.float32)
            with np.errstate(divide="ignore", invalid="ignore"):
                v = ((sym - center) / center) * mx
            _put(cache, c["blocks_first"], kv, blk, off, _to_out(v, c["out_bf16"]).reshape(H, D))
        return cache
    sink, body, gs = c["sink_tokens"], c["tokens"] - c["sink_tokens"], c["group_size"]
    vg = (C + gs - 1) // gs
    ch = np.arange(C, dtype=np.int64)
    h, d = ch // D, ch % D
    for t, kv, blk, off in _cache_rows(c):
        if t < sink:
            v = _f32((c["value_sink"] if kv else c["key_sink"])[t * C:(t + 1) * C])
        else:
            bt = t - sink
            idx = (h * D + d) * body + bt if kv else (d * H + h) * body + bt
            stream = c["bytestream"][c["value_offset"] if kv else c["key_offset"]:]
            sym = _symbols(stream, c["value_bytes"] if kv else c["key_bytes"], idx, c["bits"])
            m = bt * vg + ch // gs if kv else (bt // gs) * C + ch
            sc = _f32((c["value_scale"] if kv else c["key_scale"])[m]).astype(np.float64)
            ze = _f32((c["value_zero"] if kv else c["key_zero"])[m]).astype(np.float64)
            # s * scale is exact in float64 (8-bit integer times float32); the sum rounds in
            # float64 and again to float32. That double rounding can differ from one fused
            # multiply-add only on rare ties, and none occurs in these cases.
            v = (sym.astype(np.float64) * sc + ze).astype(np.float32)
        _put(cache, c["blocks_first"], kv, blk, off, _to_out(v, c["out_bf16"]).reshape(H, D))
    return cache


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_oracle_matches_numpy_restatement(case):
    want = numpy_restatement(case)
    got = run_oracle(case)
    np.testing.assert_array_equal(got, want)


@pytest.mark.skipif(not VECTORS.exists(), reason="reference quantized-kernel vectors not generated yet")
@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_oracle_matches_reference_kernels(case):
    z = np.load(VECTORS)
    if f"{case['name']}/expected" not in z.files:
        pytest.skip("no reference vectors for this case yet (regenerate with make_ref_quant_vectors.py)")
    for k, v in case.items():
        if isinstance(v, np.ndarray):
            np.testing.assert_array_equal(z[f"{case['name']}/{k}"], v, err_msg=f"seeded input {k} drifted")
    np.testing.assert_array_equal(run_oracle(case), z[f"{case['name']}/expected"])


def test_half_and_bf16_conversions_round_to_nearest_even():
    rng = np.random.default_rng(5)
    u = rng.integers(0, 1 << 32, 20000, dtype=np.uint64).astype(np.uint32)
    edges = np.concatenate([np.arange(0x33000000 - 3, 0x38800000 + 3, 4099, dtype=np.uint32),
                            np.arange(0x477FE000, 0x47800010, 7, dtype=np.uint32)])
    f = np.concatenate([u, edges, edges | 0x80000000]).view(np.float32)
    f = f[~np.isnan(f)]
    L = oracle.lib()
    import ctypes

    L.oracle_float_to_half.restype = ctypes.c_uint16
    L.oracle_float_to_half.argtypes = [ctypes.c_float]
    L.oracle_float_to_bf16.restype = ctypes.c_uint16
    L.oracle_float_to_bf16.argtypes = [ctypes.c_float]
    got_h = np.array([L.oracle_float_to_half(float(x)) for x in f], dtype=np.uint16)
    got_b = np.array([L.oracle_float_to_bf16(float(x)) for x in f], dtype=np.uint16)
    np.testing.assert_array_equal(got_h, _to_out(f, False))
    np.testing.assert_array_equal(got_b, _to_out(f, True))
