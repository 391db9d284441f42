"""Plane presets, the split/merge invariant and the C1 CPU lossless round trip."""
import numpy as np
import pytest
import torch

from origami_b200 import BF16_BIT_PLANES, BYTE_PLANES, FP16_BIT_PLANES, LayerFormat, PlaneSpec, plane_spec
from origami_b200.lossless.cpu_qat import CpuLosslessCodec
from origami_b200 import workloads


@pytest.mark.parametrize("spec", [BYTE_PLANES, BF16_BIT_PLANES, FP16_BIT_PLANES])
def test_split_merge_identity_all_patterns(spec):
    x = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    planes = spec.split(x)
    merged = np.zeros_like(x)
    for p, s in zip(planes, spec.shifts):
        assert p.max() < 256
        merged |= p.astype(np.uint16) << s
    np.testing.assert_array_equal(merged, x)


def test_plane_spec_validation():
    with pytest.raises(ValueError):
        PlaneSpec("bad", (8,), (8,))
    with pytest.raises(ValueError):
        PlaneSpec("overlap", (8, 0, 4), (8, 8, 1))
    with pytest.raises(ValueError):
        PlaneSpec("wide", (0, 9), (9, 7))
    assert plane_spec("bit", torch.float16) is FP16_BIT_PLANES
    assert plane_spec("bit", torch.bfloat16) is BF16_BIT_PLANES
    assert plane_spec("byte") is BYTE_PLANES


def test_layer_format_offsets_match_oracle(oracle):
    for planes in (BYTE_PLANES, BF16_BIT_PLANES, FP16_BIT_PLANES):
        for T in (1, 37, 1000, 32768):
            fmt = LayerFormat(T, 8, 128, planes)
            np.testing.assert_array_equal(fmt.offsets, oracle.layer_offsets(fmt.specs, planes.bits))
            assert fmt.num_chunks == 2 * planes.num_planes * fmt.num_specs
            meta = fmt.metadata(torch.bfloat16)
            assert meta["format"] == "origami_planes_v1" and len(meta["components"]) == 2 * planes.num_planes


def _c1_cache():
    cfg = workloads.C1
    T = cfg.tokens[0]
    nb = T // cfg.block_size
    ids = workloads.permuted_block_table(nb, nb + 5, seed=workloads.SEED)
    layers = []
    for layer in range(cfg.layers):
        kv = workloads.kv_values(T, cfg.heads, cfg.head_dim, cfg.dtype, seed=workloads.SEED + 10 * layer)
        cache = torch.zeros((2, nb + 5, cfg.block_size, cfg.heads, cfg.head_dim), dtype=cfg.dtype)
        workloads.scatter_into_cache(cache, kv, ids)
        layers.append(cache)
    return cfg, T, ids, layers


@pytest.mark.parametrize("planes", [BYTE_PLANES, BF16_BIT_PLANES])
def test_c1_cpu_lossless_roundtrip(oracle, planes):
    """Config 1: layout pack -> zlib level 1 -> unpack, byte equality (no GPU)."""
    cfg, T, ids, layers = _c1_cache()
    codec = CpuLosslessCodec("zlib")
    fmt = LayerFormat(T, cfg.heads, cfg.head_dim, planes)
    raw_total = comp_total = 0
    for cache in layers:
        c16 = cache.view(torch.int16).numpy().view(np.uint16)
        packed, offsets = oracle.pack_layer(c16, 0, ids.numpy(), T, planes.shifts, planes.bits, fmt.specs)
        chunks = [torch.from_numpy(packed[a:b].copy()) for a, b in zip(offsets[:-1], offsets[1:])]
        comp = codec.compress_many(chunks)
        back = codec.decompress_many(comp, [c.numel() for c in chunks])
        raw_total += packed.size
        comp_total += sum(c.numel() for c in comp)
        restored_packed = torch.cat(back).numpy()
        fresh = np.zeros_like(c16)
        oracle.restore_layer(restored_packed, planes.shifts, planes.bits, fmt.specs, fresh, 0, ids.numpy(), T)
        np.testing.assert_array_equal(fresh[:, ids.numpy()], c16[:, ids.numpy()])
    assert raw_total == 2 * T * cfg.heads * cfg.head_dim * 2 * cfg.layers
    assert comp_total < raw_total  # the exponent plane compresses


def test_c1_raw_bytes_roundtrip(oracle):
    cfg, T, ids, layers = _c1_cache()
    codec = CpuLosslessCodec("zlib")
    from origami_b200.layer import raw_chunk_bounds

    for cache in layers:
        c16 = cache.view(torch.int16).numpy().view(np.uint16)
        gathered = oracle.gather_blocks(c16, 0, ids.numpy())
        flat = gathered.view(np.uint8).reshape(-1)
        b = raw_chunk_bounds(flat.size)
        chunks = [torch.from_numpy(flat[x:y].copy()) for x, y in zip(b[:-1], b[1:])]
        back = codec.decompress_many(codec.compress_many(chunks), [c.numel() for c in chunks])
        value = torch.cat(back).numpy().view(np.uint16).reshape(gathered.shape)
        fresh = np.zeros_like(c16)
        oracle.scatter_blocks(value, fresh, 0, ids.numpy())
        np.testing.assert_array_equal(fresh, np.where(np.isin(np.arange(c16.shape[1]), ids.numpy())[None, :, None, None, None], c16, 0))
