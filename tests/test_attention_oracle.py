"""CPU oracle of the fused prefix attention against an independent numpy restatement
(explicit dequantization in float64, exact softmax) and, when committed, against the
reference kernel's outputs (tests/golden/ref_attention_vectors.npz, made on a B200 by
make_ref_attention_vectors.py)."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))

from attention_cases import D, cases, run_oracle, to_float  # noqa: E402

VECTORS = GOLDEN / "ref_attention_vectors.npz"
CASES = cases()


def _symbols(stream: np.ndarray, n: int, bits: int) -> np.ndarray:
    if bits == 3:
        b = np.repeat(stream[: (n + 1) // 2], 2)[:n]
        return ((b >> (4 * (np.arange(n) & 1))) & 7).astype(np.float64)
    idx = np.arange(n, dtype=np.int64) * bits
    byte = idx >> 3
    pad = np.concatenate([stream, np.zeros(2, np.uint8)]).astype(np.uint32)
    w = pad[byte] | (pad[byte + 1] << 8)
    return ((w >> (idx & 7)) & ((1 << bits) - 1)).astype(np.float64)


def dequantized_prefix(c) -> tuple[np.ndarray, np.ndarray]:
    """K, V of the prefix as [prefix, kv_heads, 128] float64."""
    H = c["kv_heads"] if "kv_heads" in c else c["kv_cache"].shape[3]
    C, P, sink = H * D, c["prefix_tokens"], c["sink_tokens"]
    f = lambda a: np.asarray(a, np.float64)  # noqa: E731
    ks = c["bytestream"][c["key_offset"]:c["key_offset"] + c["key_bytes"]]
    vs = c["bytestream"][c["value_offset"]:c["value_offset"] + c["value_bytes"]]
    K = np.zeros((P, C))
    V = np.zeros((P, C))
    if c["codec"] == 0:
        body, gs = P - sink, c["group_size"]
        K[:sink] = f(c["key_sink"]).reshape(sink, C)
        V[:sink] = f(c["value_sink"]).reshape(sink, C)
        sk = _symbols(ks, body * C, c["bits"]).reshape(D, H, body)  # [dim][head][token]
        sv = _symbols(vs, body * C, c["bits"]).reshape(H, D, body)  # [head][dim][token]
        bt = np.arange(body)
        ch = np.arange(C)
        kmeta = (bt[:, None] // gs, ch[None, :])
        k_sym = sk.transpose(2, 1, 0).reshape(body, C)
        K[sink:] = k_sym * f(c["key_scale"])[kmeta] + f(c["key_zero"])[kmeta]
        vmeta = (bt[:, None], ch[None, :] // gs)
        v_sym = sv.transpose(2, 0, 1).reshape(body, C)
        V[sink:] = v_sym * f(c["value_scale"])[vmeta] + f(c["value_zero"])[vmeta]
    else:
        sk = _symbols(ks, P * C, c["bits"]).reshape(D, H, P)
        sv = _symbols(vs, P * C, c["bits"]).reshape(H, P, D)
        K[:] = sk.transpose(2, 1, 0).reshape(P, C) * f(c["key_scale"])[None, :] + f(c["key_zero"])[None, :]
        V[:] = sv.transpose(1, 0, 2).reshape(P, C) * f(c["value_scale"])[:, None] + f(c["value_zero"])[:, None]
    return K.reshape(P, H, D), V.reshape(P, H, D)


def numpy_attention(c) -> np.ndarray:
    cache = to_float(c["kv_cache"], c["cache_bf16"]).astype(np.float64)
    bf = c["blocks_first"]
    nb, bs, H = (cache.shape[0] if bf else cache.shape[1]), cache.shape[2], cache.shape[3]
    S, P = c["sequence_length"], c["prefix_tokens"]
    Kp, Vp = dequantized_prefix(c)
    K = np.zeros((S, H, D))
    V = np.zeros((S, H, D))
    K[:P], V[:P] = Kp, Vp
    for t in range(P, S):
        pb = int(c["block_table"][t // bs])
        if 0 <= pb < nb:
            K[t] = cache[pb, 0, t % bs] if bf else cache[0, pb, t % bs]
            V[t] = cache[pb, 1, t % bs] if bf else cache[1, pb, t % bs]
    q = to_float(c["query"], c["query_bf16"]).astype(np.float64)
    QT, QH = q.shape[:2]
    g = QH // H
    out = np.zeros((QT, QH, D))
    for qt in range(QT):
        end = min(S - 1, c["query_start"] + qt)
        for qh in range(QH):
            s = K[: end + 1, qh // g] @ q[qt, qh] * c["softmax_scale"]
            w = np.exp(s - s.max())
            out[qt, qh] = (w[:, None] * V[: end + 1, qh // g]).sum(0) / w.sum()
    return out


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_oracle_matches_numpy_attention(case):
    got = to_float(run_oracle(case), case["query_bf16"])
    want = numpy_attention(case)
    tol = 1e-2 if case["query_bf16"] else 2e-3
    np.testing.assert_allclose(got, want, atol=tol, rtol=tol)


@pytest.mark.skipif(not VECTORS.exists(), reason="reference attention vectors not generated yet")
@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_oracle_matches_reference_kernel(case):
    z = np.load(VECTORS)
    if f"{case['name']}/expected" not in z.files:
        pytest.skip("no reference vectors for this case yet (regenerate with make_ref_attention_vectors.py)")
    from make_ref_attention_vectors import digest

    for k, v in case.items():
        if isinstance(v, np.ndarray):
            np.testing.assert_array_equal(z[f"{case['name']}/sha256/{k}"], digest(v), err_msg=f"seeded input {k} drifted")
    got = to_float(run_oracle(case), case["query_bf16"])
    ref = to_float(z[f"{case['name']}/expected"], case["query_bf16"])
    # fp32 arithmetic in the same order as the reference kernel: only expf / rounding ties differ
    tol = 1e-2 if case["query_bf16"] else 2e-3
    np.testing.assert_allclose(got, ref, atol=tol, rtol=tol)
