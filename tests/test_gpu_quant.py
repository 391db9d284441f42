"""Fused CacheGen / KIVI dequantize-to-cache kernels against the CPU oracle, the reference
kernels' golden outputs and, where the reference extension is built (oracle/_ref), the
reference kernels themselves on the same inputs."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))

from quant_cases import cachegen_cache_case, cases, kivi_case, run_oracle  # noqa: E402

from origami_b200.lossless import native_gpu  # noqa: E402

pytestmark = pytest.mark.gpu
VECTORS = GOLDEN / "ref_quant_vectors.npz"
CASES = cases()


def _t(a: np.ndarray, dev) -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).to(dev)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def run_ours(c: dict, dev, error_count=None) -> np.ndarray:
    """The case through the drop-in module (native_gpu -> liborigami_b200.so)."""
    from origami_b200 import quant

    stream = _t(c["bytestream"], dev)
    if c["kind"] == "cg_unpack":
        out = native_gpu.cachegen_unpack_dequantize(
            stream, _t(c["offsets"], dev), _t(c["bits"], dev), _t(c["key_bins"], dev), _t(c["value_bins"], dev),
            _t(c["max_key"], dev), _t(c["max_value"], dev), tokens=c["tokens"], heads=c["heads"],
            head_dim=c["head_dim"])
        return out.cpu().view(torch.int16).numpy().view(np.uint16)
    cache = _t(c["cache"], dev).view(torch.bfloat16 if c["out_bf16"] else torch.float16)
    ids = _t(c["block_ids"], dev)
    if c["kind"] == "cg_cache":
        quant.cachegen_unpack_dequantize_to_kv_cache_cuda(
            stream, c["key_offset"], c["key_bytes"], c["value_offset"], c["value_bytes"], c["key_bits"],
            c["value_bits"], c["key_bins"], c["value_bins"], _t(c["max_key"], dev), _t(c["max_value"], dev), cache,
            ids, c["tokens"], c["heads"], c["head_dim"], error_count=error_count)
    else:
        quant.kivi_dequantize_to_kv_cache_cuda(
            stream, c["key_offset"], c["key_bytes"], c["value_offset"], c["value_bytes"], c["bits"],
            c["group_size"], c["sink_tokens"], _t(c["key_scale"], dev), _t(c["key_zero"], dev),
            _t(c["value_scale"], dev), _t(c["value_zero"], dev), _t(c["key_sink"], dev), _t(c["value_sink"], dev),
            cache, ids, c["tokens"], c["heads"], c["head_dim"], error_count=error_count)
    return cache.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.fixture(scope="module")
def ref_ext():
    from make_ref_vectors import load_reference_extension

    return load_reference_extension()


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_matches_oracle_and_reference(cuda, case, ref_ext):
    got = run_ours(case, cuda)
    np.testing.assert_array_equal(got, run_oracle(case))
    if VECTORS.exists() and f"{case['name']}/expected" in np.load(VECTORS).files:
        np.testing.assert_array_equal(got, np.load(VECTORS)[f"{case['name']}/expected"])
    if ref_ext is not None:
        from make_ref_quant_vectors import run_reference

        np.testing.assert_array_equal(got, run_reference(ref_ext, case))


LARGE = [
    cachegen_cache_case("cg_c2_layer", 401, 32768, 8, 128, 16, 5, 4, 32, 16, np.float16, True, False, spare_blocks=40),
    cachegen_cache_case("cg_c2_layer_fp16_blocks_first", 402, 20000, 8, 128, 16, 4, 4, 16, 16, np.float32, False, True),
    # staged rows: truncated streams (groups reaching the read limit take global loads) and
    # out-of-range block ids, at symbol widths 5 / 3 and 4 / 2
    cachegen_cache_case("cg_staged_truncated", 403, 3001, 4, 64, 16, 5, 3, 32, 8, np.float16, True, False,
                        trunc=(101, 7)),
    cachegen_cache_case("cg_staged_bad_ids", 404, 2050, 2, 128, 16, 4, 2, 16, 4, np.float32, False, True, bad=True),
    kivi_case("kivi_c2_layer_b2", 403, 32768, 128, 8, 128, 16, 2, 64, np.float16, True, False, spare_blocks=40),
    kivi_case("kivi_b4_d64_ragged", 404, 9999, 32, 4, 64, 32, 4, 32, np.float16, False, True),
    kivi_case("kivi_b3_d256", 405, 5000, 0, 2, 256, 16, 3, 128, np.float32, True, False),
    # 2-bit symbols take the table kernel without a transpose: every head_dim, both cache
    # layouts, fp32 metadata, truncated streams (zero-filled staging chunks), bad block ids
    kivi_case("kivi_b2_d256_blocks_first_trunc", 406, 3001, 24, 2, 256, 16, 2, 32, np.float16, False, True,
              trunc=(37, 5)),
    kivi_case("kivi_b2_d64_f32_bad_ids", 407, 7777, 8, 4, 64, 32, 2, 16, np.float32, True, False, bad=True),
    kivi_case("kivi_b2_d128_group8_no_sink", 408, 4100, 0, 3, 128, 16, 2, 8, np.float16, False, False,
              trunc=(0, 19)),
    # block size that is not a power of two (block index by division), and a group size that
    # is not one (the general tile kernel)
    kivi_case("kivi_b2_bs24", 409, 2000, 16, 2, 128, 24, 2, 32, np.float16, True, False),
    kivi_case("kivi_b2_group24", 410, 1500, 8, 2, 64, 16, 2, 24, np.float16, True, False),
]


@pytest.mark.parametrize("case", LARGE, ids=lambda c: c["name"])
def test_full_size_layers_match_oracle(cuda, case, ref_ext):
    got = run_ours(case, cuda)
    np.testing.assert_array_equal(got, run_oracle(case))
    if ref_ext is not None:
        from make_ref_quant_vectors import run_reference

        np.testing.assert_array_equal(got, run_reference(ref_ext, case))


@pytest.mark.parametrize("name", ["cg_bf16_f32max_blocks_first_bad_ids", "kivi_b4_ragged_sink_group",
                                  "kivi_b1_d128_bad_ids"])
def test_bad_block_ids_are_skipped_and_counted(cuda, name, oracle):
    case = next(c for c in CASES if c["name"] == name)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    got = run_ours(case, cuda, error_count=err)
    np.testing.assert_array_equal(got, run_oracle(case))
    bs = case["cache"].shape[2]
    nb = case["cache"].shape[0] if case["blocks_first"] else case["cache"].shape[1]
    ids = case["block_ids"]
    bad_tokens = sum(1 for t in range(case["tokens"]) if not 0 <= ids[t // bs] < nb)
    assert int(err.item()) == 2 * bad_tokens * case["heads"]


def test_reference_error_messages(cuda):
    from origami_b200 import quant

    c = cachegen_cache_case("msg", 9, 20, 2, 16, 16, 4, 4, 16, 16, np.float16, False, False)
    s, mk, mv = _t(c["bytestream"], cuda), _t(c["max_key"], cuda), _t(c["max_value"], cuda)
    cache, ids = _t(c["cache"], cuda).view(torch.float16), _t(c["block_ids"], cuda)
    args = [s, c["key_offset"], c["key_bytes"], c["value_offset"], c["value_bytes"], 4, 4, 16, 16, mk, mv, cache,
            ids, 20, 2, 16]
    for idx, val, msg in [(5, 9, "supports only 1..8 bit symbols"), (7, 1, "bins must be greater than one"),
                          (2, 10 ** 9, "exceed bytestream length"), (13, 10 ** 6, "at least tokens values"),
                          (15, 8, "head shape mismatch")]:
        bad = list(args)
        bad[idx] = val
        with pytest.raises(RuntimeError, match=msg):
            quant.cachegen_unpack_dequantize_to_kv_cache_cuda(*bad)
    with pytest.raises(RuntimeError, match="must be float16 or float32"):
        bad = list(args)
        bad[9], bad[10] = mk.to(torch.float64), mv.to(torch.float64)
        quant.cachegen_unpack_dequantize_to_kv_cache_cuda(*bad)
    with pytest.raises(RuntimeError, match="sink_tokens must be in"):
        z = torch.zeros(4096, dtype=torch.float16, device=cuda)
        quant.kivi_dequantize_to_kv_cache_cuda(s, 0, 1, 0, 1, 2, 64, 21, z, z, z, z, z, z, cache, ids, 20, 2, 16)
