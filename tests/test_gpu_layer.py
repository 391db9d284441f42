"""Fused layer save / restore on the paged cache against the CPU oracle, plus the
raw-bytes gather / scatter against torch's index_select / index_copy_."""
import numpy as np
import pytest
import torch

from origami_b200 import BF16_BIT_PLANES, BYTE_PLANES, FP16_BIT_PLANES, LayerFormat, PlaneSpec, workloads
from origami_b200.layer import gather_blocks, pack_layer, restore_layer, scatter_blocks

pytestmark = pytest.mark.gpu

ODD_PLANES = PlaneSpec("odd", (12, 4, 0, 9), (4, 5, 4, 3))
GEOMS = [
    # T, block_size, heads, head_dim, chunk target bytes
    (1024, 16, 8, 128, 1 << 20),
    (1000, 16, 8, 128, 1 << 20),
    (37, 16, 2, 64, 1 << 20),
    (333, 32, 4, 256, 1 << 14),
    (4096, 16, 2, 128, 1 << 16),
    (8191, 16, 1, 128, 100_000),
    (70, 16, 3, 8, 1 << 20),
    (1040, 16, 2, 128, 1 << 20),  # aligned runs, partial last tile (TMA path for byte planes)
    (2048, 32, 4, 64, 1 << 20),
    (512, 16, 2, 256, 1 << 20),
    # ragged runs over many tiles per persistent CTA: vectors carried between tiles
    (20000, 16, 8, 128, 1 << 20),
    (30000, 32, 4, 64, 1 << 18),
    (12345, 16, 4, 256, 1 << 20),
    # TMA kernels over odd, 6 and 16 heads, and D = 256 with 8 heads
    (1024, 16, 3, 128, 1 << 20),
    (2048, 16, 6, 64, 1 << 20),
    (512, 16, 16, 128, 1 << 20),
    (256, 16, 8, 256, 1 << 20),
]
PLANES = [BYTE_PLANES, BF16_BIT_PLANES, FP16_BIT_PLANES, ODD_PLANES]


def make_cache(T, bs, H, D, kv_first, seed, dtype=torch.bfloat16, slack=3):
    nb = (T + bs - 1) // bs
    NB = nb + slack
    ids = workloads.permuted_block_table(nb, NB, seed)
    kv = workloads.kv_values(T, H, D, dtype, seed=seed)
    shape = (2, NB, bs, H, D) if kv_first else (NB, 2, bs, H, D)
    g = torch.Generator().manual_seed(seed + 99)
    cache = torch.randint(-32768, 32767, shape, generator=g, dtype=torch.int16).view(dtype)
    workloads.scatter_into_cache(cache, kv, ids, kv_first)
    return cache, ids


def u16(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("kv_first", [True, False])
@pytest.mark.parametrize("planes", PLANES, ids=lambda p: p.name)
@pytest.mark.parametrize("geom", GEOMS, ids=lambda g: "T%d_bs%d_H%d_D%d" % g[:4])
def test_pack_and_restore_match_oracle(oracle, cuda, geom, planes, kv_first):
    T, bs, H, D, tgt = geom
    layout = 0 if kv_first else 1
    cache, ids = make_cache(T, bs, H, D, kv_first, seed=T + H + D)
    fmt = LayerFormat(T, H, D, planes, tgt, tgt, tgt)
    want, offsets = oracle.pack_layer(u16(cache), layout, ids.numpy(), T, planes.shifts, planes.bits, fmt.specs)
    np.testing.assert_array_equal(offsets, fmt.offsets)
    d_cache = cache.to(cuda)
    out = fmt.alloc_packed(cuda)
    out.fill_(0xA5)  # stale bytes must not leak into the result
    got = pack_layer(d_cache, ids, fmt, out=out)
    np.testing.assert_array_equal(got.cpu().numpy(), want)

    # restore into a cache holding different bytes: only the request's token rows change
    dst, _ = make_cache(T, bs, H, D, kv_first, seed=T + H + D + 1)
    expect = u16(dst).copy()
    oracle.restore_layer(want, planes.shifts, planes.bits, fmt.specs, expect, layout, ids.numpy(), T)
    d_dst = dst.to(cuda)
    restore_layer(torch.from_numpy(want).to(cuda), fmt, d_dst, ids.to(cuda))
    np.testing.assert_array_equal(u16(d_dst.cpu()), expect)
    # and the restored tokens are the saved tokens
    back = workloads.tokens_from_cache(d_dst.cpu(), ids, T, kv_first)
    orig = workloads.tokens_from_cache(cache, ids, T, kv_first)
    assert torch.equal(back.view(torch.int16), orig.view(torch.int16))


def test_fp16_cache_roundtrip(cuda):
    T, bs, H, D = 777, 32, 8, 128
    cache, ids = make_cache(T, bs, H, D, True, seed=5, dtype=torch.float16)
    fmt = LayerFormat(T, H, D, FP16_BIT_PLANES)
    d = cache.to(cuda)
    packed = pack_layer(d, ids, fmt)
    fresh = torch.zeros_like(d)
    restore_layer(packed, fmt, fresh, ids)
    t = torch.arange(T)
    blk = ids[t // bs]
    assert torch.equal(fresh.cpu()[:, blk, t % bs].view(torch.int16), cache[:, blk, t % bs].view(torch.int16))


@pytest.mark.parametrize("geom", [(64, 16, 2, 64), (64, 16, 2, 128), (128, 16, 8, 128), (128, 16, 3, 128),
                                  (256, 16, 4, 64)],
                         ids=["h2_d64", "h2_d128", "h8_d128", "h3_d128", "h4_d64"])
def test_bad_block_ids_are_counted_and_skipped(cuda, geom):
    T, bs, H, D = geom
    cache, ids = make_cache(T, bs, H, D, True, seed=11)
    fmt = LayerFormat(T, H, D, BYTE_PLANES)
    d = cache.to(cuda)
    packed = pack_layer(d, ids, fmt)
    bad = ids.clone()
    bad[2] = 10_000
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    fresh = torch.zeros_like(d)
    restore_layer(packed, fmt, fresh, bad, error_count=err)
    assert int(err.item()) == 2 * H * bs  # every (kv, head, token) row of the bad block
    good = [b for b in range(T // bs) if b != 2]
    t = torch.cat([torch.arange(b * bs, (b + 1) * bs) for b in good])
    blk = ids[t // bs]
    assert torch.equal(fresh.cpu()[:, blk, t % bs], cache[:, blk, t % bs])
    err.zero_()
    pack_layer(d, bad, fmt, error_count=err)
    assert int(err.item()) > 0


def test_c2_layer_roundtrip_full_size(cuda):
    """One full C2 layer (32768 tokens, 8 heads): pack -> restore is the identity."""
    cfg = workloads.C2
    T = cfg.tokens[0]
    nb = T // cfg.block_size
    ids = workloads.permuted_block_table(nb, nb, workloads.SEED).to(cuda)
    kv = workloads.kv_values(T, cfg.heads, cfg.head_dim, cfg.dtype, seed=workloads.SEED, v_std=cfg.v_std, device=cuda)
    cache = torch.empty((2, nb, cfg.block_size, cfg.heads, cfg.head_dim), dtype=cfg.dtype, device=cuda)
    workloads.scatter_into_cache(cache, kv, ids)
    for planes in (BYTE_PLANES, BF16_BIT_PLANES):
        fmt = LayerFormat(T, cfg.heads, cfg.head_dim, planes)
        packed = pack_layer(cache, ids, fmt)
        fresh = torch.zeros_like(cache)
        restore_layer(packed, fmt, fresh, ids)
        assert torch.equal(fresh.view(torch.int16), cache.view(torch.int16))
        # plane 0 of K (exponent bits) is the first component; it must be far from uniform
        hi = packed[: int(fmt.offsets[fmt.num_specs])].cpu().numpy()
        assert len(np.unique(hi)) < 200


@pytest.mark.parametrize("kv_first", [True, False])
def test_raw_gather_scatter_match_torch(cuda, kv_first):
    cache, ids = make_cache(500, 16, 4, 64, kv_first, seed=3, slack=9)
    d = cache.to(cuda)
    dim = 1 if kv_first else 0
    got = gather_blocks(d, ids)
    want = torch.index_select(d, dim, ids.to(cuda))
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    fresh = torch.zeros_like(d)
    scatter_blocks(got, fresh, ids)
    expect = torch.zeros_like(d)
    expect.index_copy_(dim, ids.to(cuda), want)
    assert torch.equal(fresh.view(torch.int16), expect.view(torch.int16))


@pytest.mark.parametrize("planes", [BYTE_PLANES, BF16_BIT_PLANES, FP16_BIT_PLANES, ODD_PLANES], ids=lambda p: p.name)
@pytest.mark.parametrize("T, jobs", [(1024, 5), (1000, 3), (256, 131), (3000, 40)])
def test_batched_jobs_match_per_job(oracle, cuda, planes, T, jobs):
    """Batched pack/restore over several layers (own caches, own block tables) gives the
    per-job results and the oracle's bytes; 131 jobs span two persistent launches."""
    from origami_b200.layer import alloc_jobs_packed, job_stride, pack_layers, restore_layers

    bs, H, D = 16, 2, 128
    fmt = LayerFormat(T, H, D, planes, 1 << 16, 1 << 16, 1 << 16)
    caches, ids = [], []
    for j in range(jobs):
        c, i = make_cache(T, bs, H, D, True, seed=1000 + j)
        caches.append(c.to(cuda))
        ids.append(i)
    arena = alloc_jobs_packed(fmt, jobs, cuda)
    arena.fill_(0x5A)
    pack_layers(caches, ids, fmt, arena)
    stride = job_stride(fmt)
    got = arena.cpu().numpy()
    for j in (0, jobs // 2, jobs - 1):
        want, _ = oracle.pack_layer(u16(caches[j].cpu()), 0, ids[j].numpy(), T, planes.shifts, planes.bits, fmt.specs)
        np.testing.assert_array_equal(got[j * stride:j * stride + fmt.packed_bytes], want, err_msg=f"job {j}")
    fresh = [torch.zeros_like(c) for c in caches]
    restore_layers(arena, fmt, fresh, ids)
    t = torch.arange(T)
    for j in range(jobs):
        blk = ids[j][t // bs]
        assert torch.equal(fresh[j].cpu()[:, blk, t % bs].view(torch.int16),
                           caches[j].cpu()[:, blk, t % bs].view(torch.int16)), j


@pytest.mark.parametrize("planes", [BYTE_PLANES, BF16_BIT_PLANES, ODD_PLANES], ids=lambda p: p.name)
@pytest.mark.parametrize("geom", [(1000, 16, 8, 128, 613), (4096, 16, 2, 128, 4000), (333, 32, 4, 256, 33),
                                  (2048, 32, 4, 64, 1500), (30000, 16, 8, 128, 29999)],
                         ids=lambda g: "T%d_bs%d_H%d_D%d_to%d" % g)
def test_prefix_restore_writes_only_the_first_tokens(oracle, cuda, geom, planes):
    """A restore of the first T' < T tokens (the reference narrows a restored layer to
    the request's token count, worker.py:116-130, 1165): rows of those tokens equal a full
    restore's, every other row of the cache keeps its bytes, and only the first
    ceil(T' / block_size) block ids are read."""
    T, bs, H, D, Tp = geom
    cache, ids = make_cache(T, bs, H, D, True, seed=T + 3)
    fmt = LayerFormat(T, H, D, planes)
    want, _ = oracle.pack_layer(u16(cache), 0, ids.numpy(), T, planes.shifts, planes.bits, fmt.specs)
    dst, _ = make_cache(T, bs, H, D, True, seed=T + 4)
    full = u16(dst).copy()
    oracle.restore_layer(want, planes.shifts, planes.bits, fmt.specs, full, 0, ids.numpy(), T)
    expect = u16(dst).copy()
    t = np.arange(Tp)
    blk = ids.numpy()[t // bs]
    expect[:, blk, t % bs] = full[:, blk, t % bs]
    d_dst = dst.to(cuda)
    need = (Tp + bs - 1) // bs
    short_ids = ids[:need].clone()
    restore_layer(torch.from_numpy(want).to(cuda), fmt, d_dst, short_ids.to(cuda), num_tokens=Tp)
    np.testing.assert_array_equal(u16(d_dst.cpu()), expect)


def test_prefix_restore_checks_its_token_count(cuda):
    T, bs, H, D = 256, 16, 2, 128
    cache, ids = make_cache(T, bs, H, D, True, seed=9)
    fmt = LayerFormat(T, H, D, BYTE_PLANES)
    d = cache.to(cuda)
    packed = pack_layer(d, ids, fmt)
    for bad in (0, T + 1):
        with pytest.raises(RuntimeError, match="restore_tokens"):
            restore_layer(packed, fmt, d, ids, num_tokens=bad)


def _request_rows(cache, ids, T):
    """A request's token rows [2, T, H, D] gathered from a paged cache (KV-first)."""
    bs = cache.shape[2]
    t = torch.arange(T, device=cache.device)
    return cache[:, ids[t // bs], t % bs]


def test_c3_layer_in_its_shared_pool_matches_oracle(oracle, cuda):
    """One C3 layer at full size: the 16 ragged requests (T ~ U[4096, 65536]) share one pool
    sized for 120 GB over 32 layers, through interleaved block tables. Requests with the same
    token count are packed in one batched launch, as bench.py does. The oracle checks the
    packed bytes of the shortest and the longest request; restoring every request into a
    fresh pool reproduces each request's rows and writes no other block."""
    from origami_b200.layer import alloc_jobs_packed, job_stride, pack_layers, restore_layers

    cfg = workloads.c3_config()
    tokens, bs, H, D = list(cfg.tokens), cfg.block_size, cfg.heads, cfg.head_dim
    NB = workloads.c3_pool_blocks(cfg)
    tables = [t.to(cuda) for t in workloads.interleaved_block_tables(tokens, bs, NB, workloads.SEED + 5)]
    g = torch.Generator(device=cuda).manual_seed(11)
    pool = torch.randint(-32768, 32767, (2, NB, bs, H, D), generator=g, device=cuda, dtype=torch.int16).view(cfg.dtype)
    for r, T in enumerate(tokens):
        kv = workloads.kv_values(T, H, D, cfg.dtype, seed=workloads.SEED + r, v_std=cfg.v_std, device=cuda)
        workloads.scatter_into_cache(pool, kv, tables[r])
    groups: dict[int, list[int]] = {}
    for r, T in enumerate(tokens):
        groups.setdefault(T, []).append(r)
    packed = {}
    fresh = torch.zeros_like(pool)
    for T, reqs in groups.items():
        fmt = LayerFormat(T, H, D, BYTE_PLANES)
        arena = alloc_jobs_packed(fmt, len(reqs), cuda)
        pack_layers([pool] * len(reqs), [tables[r] for r in reqs], fmt, arena)
        stride = job_stride(fmt)
        for j, r in enumerate(reqs):
            packed[r] = (fmt, arena[j * stride:j * stride + fmt.packed_bytes])
        restore_layers(arena, fmt, [fresh] * len(reqs), [tables[r] for r in reqs])
    for r in (int(np.argmin(tokens)), int(np.argmax(tokens))):
        T = tokens[r]
        fmt, got = packed[r]
        nb = (T + bs - 1) // bs
        compact = pool[:, tables[r][:nb]]  # the request's blocks, in table order
        want, _ = oracle.pack_layer(u16(compact.cpu()), 0, np.arange(nb, dtype=np.int64), T, BYTE_PLANES.shifts,
                                    BYTE_PLANES.bits, fmt.specs)
        np.testing.assert_array_equal(got.cpu().numpy(), want, err_msg=f"request {r} (T={T})")
    used = torch.zeros(NB, dtype=torch.bool, device=cuda)
    for r, T in enumerate(tokens):
        assert torch.equal(_request_rows(fresh, tables[r], T).view(torch.int16),
                           _request_rows(pool, tables[r], T).view(torch.int16)), f"request {r}"
        used[tables[r]] = True
    assert not bool(fresh[:, ~used].view(torch.int16).any())


def test_c5_save_layer_batched_matches_oracle(oracle, cuda):
    """One C5 save layer at full size: 64 requests x 8192 tokens (Qwen2-7B KV: 4 heads,
    D 128, bf16, block 16) packed in one batched launch; the oracle checks jobs 0, 31 and
    63, and restoring every job gives the requests' rows back."""
    from origami_b200.layer import alloc_jobs_packed, job_stride, pack_layers, restore_layers

    cfg = workloads.C5
    R, T, bs, H, D = len(cfg.tokens), cfg.tokens[0], cfg.block_size, cfg.heads, cfg.head_dim
    nb = T // bs
    pool = workloads.permuted_block_table(nb * R, nb * R, workloads.SEED + 4)
    tables = [pool[r * nb:(r + 1) * nb].to(cuda) for r in range(R)]
    cache = torch.empty((2, nb * R, bs, H, D), dtype=cfg.dtype, device=cuda)
    for r in range(R):
        kv = workloads.kv_values(T, H, D, cfg.dtype, seed=workloads.SEED + r, v_std=cfg.v_std, device=cuda)
        workloads.scatter_into_cache(cache, kv, tables[r])
    fmt = LayerFormat(T, H, D, BYTE_PLANES)
    arena = alloc_jobs_packed(fmt, R, cuda)
    pack_layers([cache] * R, tables, fmt, arena)
    stride = job_stride(fmt)
    for r in (0, R // 2 - 1, R - 1):
        compact = cache[:, tables[r]]
        want, _ = oracle.pack_layer(u16(compact.cpu()), 0, np.arange(nb, dtype=np.int64), T, BYTE_PLANES.shifts,
                                    BYTE_PLANES.bits, fmt.specs)
        np.testing.assert_array_equal(arena[r * stride:r * stride + fmt.packed_bytes].cpu().numpy(), want,
                                      err_msg=f"job {r}")
    fresh = torch.zeros_like(cache)
    restore_layers(arena, fmt, [fresh] * R, tables)
    assert torch.equal(fresh.view(torch.int16), cache.view(torch.int16))
