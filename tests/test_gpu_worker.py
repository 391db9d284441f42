"""The connector hooks end to end on the GPU: save_kv_layer -> wait_for_save -> store
-> start_load_kv -> wait_for_layer_load, for the plane layouts and the reference's
raw-bytes layout."""
import numpy as np
import pytest
import torch

from origami_b200 import BYTE_PLANES, LayerFormat, workloads
from origami_b200.metadata import OrigamiConnectorMetadata, OrigamiRestoreRequest, OrigamiSaveRequest
from origami_b200.worker import InMemoryStore, OrigamiB200Worker

pytestmark = pytest.mark.gpu


def _caches(cuda, layers, T, bs, H, D, NB, ids, seed, dtype=torch.bfloat16):
    caches, values = {}, {}
    for li in range(layers):
        kv = workloads.kv_values(T, H, D, dtype, seed=seed + li)
        c = torch.zeros((2, NB, bs, H, D), dtype=dtype, device=cuda)
        workloads.scatter_into_cache(c, kv.to(cuda), ids)
        caches[f"model.layers.{li}.self_attn"] = c
        values[f"model.layers.{li}.self_attn"] = kv
    return caches, values


@pytest.mark.parametrize("policy", ["byte", "bit", "raw"])
def test_save_then_restore_through_hooks(cuda, policy):
    T, bs, H, D, layers = 1000, 16, 4, 128, 3
    nb = (T + bs - 1) // bs
    NB = nb + 7
    ids = workloads.permuted_block_table(nb, NB, seed=21)
    caches, values = _caches(cuda, layers, T, bs, H, D, NB, ids, seed=40)
    store = InMemoryStore()
    w = OrigamiB200Worker(layout_policy=policy, chunk_min_bytes=1 << 16, chunk_target_bytes=1 << 16,
                          chunk_max_bytes=1 << 16, store=store, device=cuda)
    w.register_kv_caches(caches)
    ids_t = tuple(int(i) for i in ids)
    w.start_load_kv(OrigamiConnectorMetadata(reqs_to_save={"r0": OrigamiSaveRequest("r0", "key0", (ids_t,), T)}))
    for name, c in caches.items():
        w.save_kv_layer(name, c, None)
    w.wait_for_save()
    payload = store.get("key0")
    assert set(payload.layer_payloads) == set(caches)
    raw = sum(ch.unpacked_bytes for lp in payload.layer_payloads.values() for ch in lp.chunks)
    comp = sum(ch.compressed_bytes for lp in payload.layer_payloads.values() for ch in lp.chunks)
    assert comp < raw
    if policy == "raw":  # the reference's raw-bytes symbols: gathered blocks, in order
        lp = payload.layer_payloads["model.layers.0.self_attn"]
        gathered = torch.index_select(caches["model.layers.0.self_attn"], 1, ids.to(cuda)).cpu()
        assert lp.quant_metadata["byte_count"] == gathered.numel() * 2

    fresh = {n: torch.zeros_like(c) for n, c in caches.items()}
    w2 = OrigamiB200Worker(layout_policy=policy, chunk_min_bytes=1 << 16, chunk_target_bytes=1 << 16,
                           chunk_max_bytes=1 << 16, store=store, device=cuda)
    w2.register_kv_caches(fresh)
    w2.start_load_kv(OrigamiConnectorMetadata(reqs_to_restore={"r1": OrigamiRestoreRequest("r1", "key0", (ids_t,), T)}))
    for name in fresh:
        w2.wait_for_layer_load(name)
    torch.cuda.synchronize()
    _, done = w2.get_finished()
    assert done == {"r1"}
    t = torch.arange(T)
    for name, c in fresh.items():
        got = c.cpu()[:, ids[t // bs], t % bs]
        assert torch.equal(got.view(torch.int16), values[name].view(torch.int16)), name
    w.shutdown()
    w2.shutdown()


def test_missing_artifact_surfaces_in_wait(cuda):
    caches = {"layer.0": torch.zeros((2, 4, 16, 2, 64), dtype=torch.bfloat16, device=cuda)}
    w = OrigamiB200Worker(store=InMemoryStore(), device=cuda)
    w.register_kv_caches(caches)
    w.start_load_kv(OrigamiConnectorMetadata(reqs_to_restore={"r": OrigamiRestoreRequest("r", "nope", ((0, 1),), 20)}))
    with pytest.raises(KeyError):
        w.wait_for_layer_load("layer.0")
    w.shutdown()


@pytest.mark.parametrize("policy", ["byte", "bit", "raw"])
def test_partial_restore_through_hooks(cuda, policy):
    """Save T tokens, restore T' < T through the hooks: the T' token rows come back
    byte-exact and rows past them keep their bytes (whole blocks for the raw layout,
    which restores the blocks the T' tokens need, as the reference does)."""
    T, Tp, bs, H, D, layers = 1000, 613, 16, 4, 128, 2
    nb = (T + bs - 1) // bs
    NB = nb + 7
    ids = workloads.permuted_block_table(nb, NB, seed=23)
    caches, values = _caches(cuda, layers, T, bs, H, D, NB, ids, seed=60)
    store = InMemoryStore()
    kw = dict(layout_policy=policy, chunk_min_bytes=1 << 16, chunk_target_bytes=1 << 16, chunk_max_bytes=1 << 16,
              store=store, device=cuda)
    w = OrigamiB200Worker(**kw)
    w.register_kv_caches(caches)
    ids_t = tuple(int(i) for i in ids)
    w.start_load_kv(OrigamiConnectorMetadata(reqs_to_save={"r0": OrigamiSaveRequest("r0", "k", (ids_t,), T)}))
    for name, c in caches.items():
        w.save_kv_layer(name, c, None)
    w.wait_for_save()

    sentinel = {n: torch.full_like(c, 3.0) for n, c in caches.items()}
    fresh = {n: c.clone() for n, c in sentinel.items()}
    w2 = OrigamiB200Worker(**kw)
    w2.register_kv_caches(fresh)
    w2.start_load_kv(OrigamiConnectorMetadata(reqs_to_restore={"r1": OrigamiRestoreRequest("r1", "k", (ids_t,), Tp)}))
    for name in fresh:
        w2.wait_for_layer_load(name)
    torch.cuda.synchronize()
    upto = (Tp + bs - 1) // bs * bs if policy == "raw" else Tp
    t = torch.arange(upto)
    for name, c in fresh.items():
        got = c.cpu()
        assert torch.equal(got[:, ids[t // bs], t % bs].view(torch.int16), values[name][:, :upto].view(torch.int16))
        untouched = got.clone()
        untouched[:, ids[t // bs], t % bs] = sentinel[name].cpu()[:, ids[t // bs], t % bs]
        assert torch.equal(untouched.view(torch.int16), sentinel[name].cpu().view(torch.int16)), name
    w.shutdown()
    w2.shutdown()


def test_wait_for_layer_load_is_a_stream_wait_once_enqueued(cuda):
    """Once a layer is enqueued, wait_for_layer_load costs the forward thread no host
    wait: it returns while the layer's restore is still running on the GPU and only
    orders the current stream after it."""
    T, bs, H, D, layers = 4096, 16, 8, 128, 3
    nb = T // bs
    ids = workloads.permuted_block_table(nb, nb, seed=5)
    caches, values = _caches(cuda, layers, T, bs, H, D, nb, ids, seed=70)
    store = InMemoryStore()
    kw = dict(layout_policy="byte", store=store, device=cuda, lossless_backend="raw")
    w = OrigamiB200Worker(**kw)
    w.register_kv_caches(caches)
    ids_t = tuple(int(i) for i in ids)
    w.start_load_kv(OrigamiConnectorMetadata(reqs_to_save={"r0": OrigamiSaveRequest("r0", "k", (ids_t,), T)}))
    for name, c in caches.items():
        w.save_kv_layer(name, c, None)
    w.wait_for_save()

    fresh = {n: torch.zeros_like(c) for n, c in caches.items()}
    w2 = OrigamiB200Worker(**kw)
    w2.register_kv_caches(fresh)
    # hold the restore pipeline's streams behind a long device sleep, so that the restore
    # events are certainly still pending when the forward thread asks for the layers
    restore_pipe, _ = w2._pipes(LayerFormat(T, H, D, BYTE_PLANES).packed_bytes)
    with torch.cuda.stream(restore_pipe.copy_stream):
        torch.cuda._sleep(200_000_000)
    w2.start_load_kv(OrigamiConnectorMetadata(reqs_to_restore={"r1": OrigamiRestoreRequest("r1", "k", (ids_t,), T)}))
    futs = [f for fl in w2._pending_layer_futures.values() for f in fl]
    for f in futs:
        f.result(timeout=60)  # every layer decoded and enqueued
    events = [f.result() for f in futs]
    for name in fresh:
        w2.wait_for_layer_load(name)
    assert w2.host_waits == 0
    assert not all(ev.query() for ev in events)  # returned while the restores were still queued
    done = torch.cuda.Event()
    done.record(torch.cuda.current_stream(cuda))
    done.synchronize()  # the current stream was ordered after every layer's restore
    assert all(ev.query() for ev in events)
    t = torch.arange(T)
    for name, c in fresh.items():
        assert torch.equal(c.cpu()[:, ids[t // bs], t % bs].view(torch.int16), values[name].view(torch.int16))
    w.shutdown()
    w2.shutdown()
