"""The CPU oracle against the reference: pure-Python restatement, known answers, the
reference GPU kernel's own outputs (tests/golden/ref_unpack_vectors.npz, produced on a
B200 by tests/golden/make_ref_vectors.py) and the reference's index_select."""
import json

import numpy as np
import pytest

from conftest import GOLDEN


def _rand_case(rng, layout, shape, specs, bits):
    specs = np.asarray(specs, dtype=np.int64).reshape(-1, 6)
    n = (specs[:, 1] - specs[:, 0]) * (specs[:, 3] - specs[:, 2]) * (specs[:, 5] - specs[:, 4])
    sizes = (n * np.asarray(bits) + 7) // 8
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    flat = rng.integers(0, 256, int(offsets[-1]), dtype=np.uint8)
    return flat, offsets, specs


CASES = [
    (["token", "head", "head_dim"], [5, 2, 8], [[0, 1, 0, 8, 0, 5], [1, 2, 0, 3, 0, 5], [1, 2, 3, 8, 0, 5]], [3, 8, 1]),
    (["head", "head_dim", "token"], [2, 4, 9], [[0, 2, 0, 4, 0, 4], [0, 2, 0, 4, 4, 9]], [5, 7]),
    (["layer", "head", "token", "head_dim"], [1, 3, 6, 4], [[0, 3, 0, 4, 0, 6]], [2]),
    (["head_dim", "layer", "token", "head"], [6, 1, 7, 2], [[0, 2, 0, 6, 0, 7]], [6]),
    (["token", "head", "head_dim"], [3, 2, 5], [[1, 2, 1, 4, 0, 3]], [4]),  # partial coverage
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_unpack_matches_python_restatement(oracle, case):
    layout, shape, specs, bits = CASES[case]
    rng = np.random.default_rng(case)
    flat, offsets, specs = _rand_case(rng, layout, shape, specs, bits)
    got = oracle.unpack_canonical(flat, offsets, bits, specs, shape, layout)
    want = oracle.unpack_canonical_py(flat.tobytes(), offsets, bits, specs, shape, layout)
    np.testing.assert_array_equal(got, want)


def test_pack_known_answer(oracle):
    # symbols 1, 2, 3, 4 at 3 bits, LSB first: 001|010|011|100 -> 0xD1, 0x08
    flat, offsets = oracle.pack_canonical(np.array([1, 2, 3, 4], np.uint8), 3, [[0, 1, 0, 1, 0, 4]], [4, 1, 1],
                                          ["token", "head", "head_dim"])
    assert flat.tolist() == [0xD1, 0x08]
    assert offsets.tolist() == [0, 2]


@pytest.mark.parametrize("bits", [1, 2, 3, 5, 6, 7, 8])
def test_pack_unpack_roundtrip(oracle, bits):
    rng = np.random.default_rng(bits)
    T, H, D = 37, 3, 24
    from origami_b200.lossless.chunking import plan_head_channel_chunks

    specs = [c.layout.spec() for c in plan_head_channel_chunks(layer_index=0, num_heads=H, head_dim=D, token_count=T,
                                                                bytes_per_symbol=1, min_bytes=100, target_bytes=200,
                                                                max_bytes=300)]
    sym = rng.integers(0, 256, T * H * D, dtype=np.uint8)
    flat, offsets = oracle.pack_canonical(sym, bits, specs, [T, H, D], ["token", "head", "head_dim"])
    back = oracle.unpack_canonical(flat, offsets, [bits] * len(specs), specs, [T, H, D], ["token", "head", "head_dim"])
    np.testing.assert_array_equal(back, sym & ((1 << bits) - 1))
    # pad bits of every chunk's last byte are zero
    for k in range(len(specs)):
        n = np.prod(np.diff(np.asarray(specs[k]).reshape(3, 2), axis=1))
        used = int(n) * bits
        if used % 8:
            assert flat[offsets[k + 1] - 1] >> (used % 8) == 0


def test_oracle_matches_reference_kernel_vectors(oracle):
    path = GOLDEN / "ref_unpack_vectors.npz"
    if not path.exists():
        pytest.skip("reference-kernel vectors not generated yet (tests/golden/make_ref_vectors.py on a B200)")
    z = np.load(path)
    index = json.loads(bytes(z["index"]).decode())
    assert len(index) >= 10
    for case in index:
        got = oracle.unpack_canonical(z[case["name"] + "__flat"], case["offsets"], case["bits"], case["specs"],
                                      case["shape"], case["layout"])
        np.testing.assert_array_equal(got, z[case["name"] + "__out"], err_msg=case["name"])


def test_gather_matches_reference_select_blocks(oracle):
    z = np.load(GOLDEN / "select_blocks.npz")
    got = oracle.gather_blocks(z["cache"].view(np.uint16), 0, z["ids"])
    np.testing.assert_array_equal(got, z["selected"].view(np.uint16))
    got = oracle.gather_blocks(z["cache_blocks_first"].view(np.uint16), 1, z["ids"])
    np.testing.assert_array_equal(got, z["selected_blocks_first"].view(np.uint16))


def test_scatter_inverts_gather(oracle):
    rng = np.random.default_rng(3)
    cache = rng.integers(0, 65535, (2, 9, 4, 2, 8), dtype=np.uint16)
    ids = np.array([4, 0, 7])
    value = oracle.gather_blocks(cache, 0, ids)
    fresh = np.zeros_like(cache)
    oracle.scatter_blocks(value, fresh, 0, ids)
    np.testing.assert_array_equal(fresh[:, ids], cache[:, ids])
    assert not fresh[:, [1, 2, 3, 5, 6, 8]].any()
