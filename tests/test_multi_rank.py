"""N>1 host logic on CPU: two gloo ranks each save and restore their own KV-head shard
(oracle kernels), the shards never share a chunk, and their union equals the unsharded
restore. The only cross-rank operations are the ones bench.py uses: a barrier and a
max over ranks of a timing."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from origami_b200 import BF16_BIT_PLANES, LayerFormat, workloads
from origami_b200.sharding import head_range, shard_format


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, q):
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(repo), str(repo / "oracle")]
    import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    T, H, D, bs = 300, 4, 32, 16
    nb = (T + bs - 1) // bs
    ids = workloads.permuted_block_table(nb, nb + 2, seed=3)
    kv = workloads.kv_values(T, H, D, torch.bfloat16, seed=3)
    h0, h1 = head_range(rank, world, H)
    cache = torch.zeros((2, nb + 2, bs, h1 - h0, D), dtype=torch.bfloat16)
    workloads.scatter_into_cache(cache, kv[:, :, h0:h1].contiguous(), ids)
    fmt = shard_format(rank, world, T, H, D, BF16_BIT_PLANES, chunk_bytes=2000)
    c16 = cache.view(torch.int16).numpy().view(np.uint16)
    packed, _ = oracle.pack_layer(c16, 0, ids.numpy(), T, fmt.planes.shifts, fmt.planes.bits, fmt.specs)
    fresh = np.zeros_like(c16)
    oracle.restore_layer(packed, fmt.planes.shifts, fmt.planes.bits, fmt.specs, fresh, 0, ids.numpy(), T)
    shard = torch.from_numpy(fresh.view(np.int16).astype(np.int32))  # gloo gathers 32-bit ints
    gathered = [torch.zeros_like(shard) for _ in range(world)]
    dist.all_gather(gathered, shard)  # test-only check of the union; bench.py never moves data
    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.barrier()
    if rank == 0:
        full = torch.cat(gathered, dim=3)
        ref_cache = torch.zeros((2, nb + 2, bs, H, D), dtype=torch.bfloat16)
        workloads.scatter_into_cache(ref_cache, kv, ids)
        q.put((bool(torch.equal(full, ref_cache.view(torch.int16).to(torch.int32))), float(t.item()),
               int(fmt.specs[:, 1].max()), int(packed.size)))
    dist.destroy_process_group()


def test_two_rank_head_sharding():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs)
    equal, tmax, max_head, nbytes = q.get(timeout=10)
    assert equal
    assert tmax == 2.0
    assert max_head == 2  # every chunk of a rank stays inside its 2 heads
    assert nbytes == LayerFormat(300, 2, 32, BF16_BIT_PLANES, 2000, 2000, 2000).packed_bytes


def test_head_range_validation():
    assert head_range(3, 8, 8) == (3, 4)
    assert head_range(1, 2, 8) == (4, 8)
    with pytest.raises(ValueError):
        head_range(0, 3, 8)
    with pytest.raises(ValueError):
        head_range(2, 2, 8)
