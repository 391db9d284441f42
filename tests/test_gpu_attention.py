"""Fused prefix attention (tcgen05 kernel) against the CPU oracle, the reference kernel's
committed outputs and, where the reference extension is built (oracle/_ref), the reference
kernel itself on the same inputs. Tolerances are the reference test's
(test_origami_fused_attention.py:123): 1.5e-2 for fp16, 3e-2 for bf16, absolute and
relative."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))

from attention_cases import attention_case, cases, run_oracle, to_float  # noqa: E402

pytestmark = pytest.mark.gpu
VECTORS = GOLDEN / "ref_attention_vectors.npz"
CASES = cases()


def _tol(case):
    return 3e-2 if case["query_bf16"] else 1.5e-2


def _t(a: np.ndarray, dev):
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).to(dev)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _args(c, dev):
    qd = torch.bfloat16 if c["query_bf16"] else torch.float16
    cd = torch.bfloat16 if c["cache_bf16"] else torch.float16
    query = _t(c["query"], dev).view(qd)
    return [_t(c["bytestream"], dev), c["key_offset"], c["key_bytes"], c["value_offset"], c["value_bytes"], c["codec"],
            c["bits"], c["group_size"], c["sink_tokens"], _t(c["key_scale"].reshape(-1), dev),
            _t(c["key_zero"].reshape(-1), dev), _t(c["value_scale"].reshape(-1), dev),
            _t(c["value_zero"].reshape(-1), dev), _t(c["key_sink"].reshape(-1), dev),
            _t(c["value_sink"].reshape(-1), dev), query, _t(c["kv_cache"], dev).view(cd), _t(c["block_table"], dev),
            c["prefix_tokens"], c["query_start"], c["sequence_length"], c["softmax_scale"], torch.empty_like(query)]


def run_ours(c, dev, **kw) -> np.ndarray:
    """The case through the drop-in extension op (native_gpu -> liborigami_b200.so)."""
    from origami_b200.lossless import native_gpu

    args = _args(c, dev)
    native_gpu.load_bitpack_cuda_extension().fused_prefix_attention_cuda(*args, **kw)
    return args[-1].view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.fixture(scope="module")
def ref_ext():
    from make_ref_vectors import load_reference_extension

    return load_reference_extension()


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_matches_oracle_and_reference(cuda, case, ref_ext):
    got = to_float(run_ours(case, cuda), case["query_bf16"])
    assert np.isfinite(got).all()
    tol = _tol(case)
    np.testing.assert_allclose(got, to_float(run_oracle(case), case["query_bf16"]), atol=tol, rtol=tol)
    if VECTORS.exists() and f"{case['name']}/expected" in np.load(VECTORS).files:
        ref = to_float(np.load(VECTORS)[f"{case['name']}/expected"], case["query_bf16"])
        np.testing.assert_allclose(got, ref, atol=tol, rtol=tol)
    if ref_ext is not None:
        from make_ref_attention_vectors import run_reference

        np.testing.assert_allclose(got, to_float(run_reference(ref_ext, case), case["query_bf16"]), atol=tol, rtol=tol)


LARGE = [
    # decode over a C2-length prefix: many splits, sink, suffix in the cache
    attention_case("kivi_b2_32k_decode", 501, codec=0, bits=2, prefix=32768, sink=32, group_size=32, kv_heads=8,
                   query_heads=32, query_start=33023, seq_len=33024),
    attention_case("kvquant_b4_8k_q16_bf16", 502, codec=1, bits=4, prefix=8192, kv_heads=8, query_heads=32,
                   query_tokens=16, query_start=8300, query_bf16=True),
    # the bench's ATTN layer shape on the symbol-operand kernel (group 64, staged stream words)
    attention_case("kivi_b2_g64_32k_decode", 503, codec=0, bits=2, prefix=32768, sink=128, group_size=64, kv_heads=8,
                   query_heads=32, query_start=33023, seq_len=33024, query_bf16=True),
]


@pytest.mark.parametrize("case", LARGE, ids=lambda c: c["name"])
def test_long_prefixes_match_reference(cuda, case, ref_ext):
    got = to_float(run_ours(case, cuda), case["query_bf16"])
    tol = _tol(case)
    if ref_ext is not None:
        from make_ref_attention_vectors import run_reference

        want = to_float(run_reference(ref_ext, case), case["query_bf16"])
    else:
        want = to_float(run_oracle(case), case["query_bf16"])
    np.testing.assert_allclose(got, want, atol=tol, rtol=tol)


def test_workspace_is_reused_and_left_zero(cuda):
    from origami_b200 import attention

    c = next(x for x in CASES if x["name"] == "kivi_b2_long_decode")
    need = attention.workspace_bytes(1, 32, 8, c["query_start"], c["sequence_length"], cuda)
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    flags = torch.zeros(1, dtype=torch.int32, device=cuda)
    first = run_ours(c, cuda, workspace=ws, error_flags=flags)
    second = run_ours(c, cuda, workspace=ws, error_flags=flags)
    np.testing.assert_array_equal(first, second)
    assert int(flags.item()) == 0
    counters = ws[: 8 * 4].view(torch.int32)  # one row block per KV head, counters first
    assert int(counters.abs().sum().item()) == 0


def test_reference_error_messages(cuda):
    from origami_b200 import attention

    c = CASES[0]
    args = _args(c, cuda)
    for idx, val, msg in [(5, 2, "codec must be 0 \\(KIVI\\) or 1 \\(KVQuant\\)"),
                          (6, 5, "fused attention supports 2, 3, 4, or 8 bits"),
                          (7, 0, "group_size must be positive"), (18, 0, "prefix_tokens must be positive"),
                          (8, 20, "sink_tokens must be in \\[0, prefix_tokens\\]"),
                          (2, 10 ** 9, "compressed stream ranges exceed bytestream length"),
                          (19, 5, "query must start at or after the compressed prefix"),
                          (20, 10, "query range exceeds sequence length")]:
        bad = list(args)
        bad[idx] = val
        with pytest.raises(RuntimeError, match=msg):
            attention.fused_prefix_attention_cuda(*bad)
    bad = list(args)
    bad[17] = bad[17].to(torch.int64)
    with pytest.raises(RuntimeError, match="block_table must be int32"):
        attention.fused_prefix_attention_cuda(*bad)
    bad = list(args)
    bad[15] = bad[15][:, :, :64].contiguous()
    bad[22] = torch.empty_like(bad[15])
    with pytest.raises(RuntimeError, match="head_dim 128 only"):
        attention.fused_prefix_attention_cuda(*bad)
    bad = list(args)
    bad[9] = bad[9][:3]
    with pytest.raises(RuntimeError, match="KIVI key metadata is too small"):
        attention.fused_prefix_attention_cuda(*bad)
