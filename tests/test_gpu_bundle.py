"""Save -> bundle_v1 -> restore through the codec handoff, on the GPU: layers packed from
a paged cache, deflated from pinned memory into a bundle by the native codec, then
decoded straight into the restore pipeline's pinned staging and restored into fresh
caches, which must hold the original tokens bit for bit."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from origami_b200 import BF16_BIT_PLANES, BYTE_PLANES, LayerFormat, workloads
from origami_b200.bundle import BundleStore
from origami_b200.layer import pack_layer
from origami_b200.pipeline import RestorePipeline

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("planes", [BYTE_PLANES, BF16_BIT_PLANES], ids=lambda p: p.name)
def test_bundle_roundtrip_through_pinned_staging(cuda, tmp_path, planes):
    T, bs, H, D, L = 3000, 16, 4, 128, 5
    nb = (T + bs - 1) // bs
    NB = nb + 7
    ids = workloads.permuted_block_table(nb, NB, 11)
    caches, fmts, host = [], [], []
    for layer in range(L):
        kv = workloads.kv_values(T, H, D, torch.bfloat16, seed=100 + layer)
        c = torch.zeros((2, NB, bs, H, D), dtype=torch.bfloat16)
        workloads.scatter_into_cache(c, kv, ids)
        caches.append(c.to(cuda))
        fmt = LayerFormat(T, H, D, planes, 1 << 16, 1 << 16, 1 << 16, layer_index=layer)
        fmts.append(fmt)
        h = fmt.alloc_packed("cpu", pin=True)
        h.copy_(pack_layer(caches[-1], ids, fmt))
        host.append(h)
    store = BundleStore(tmp_path)
    store.put_packed_layers(cache_key="req:0", request_id="req", token_count=T, dtype=torch.bfloat16,
                            layers=[(f"layers.{i}.attn", fmts[i], host[i]) for i in range(L)])
    qb = store.open_qat_bundle("req:0")
    pipe = RestorePipeline(cuda, fmts[0].packed_bytes, slots=3)
    fresh = [torch.zeros_like(c) for c in caches]
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    events = [pipe.enqueue_from_bundle(qb, f"layers.{i}.attn", fmts[i], fresh[i], ids.to(cuda), error_count=err)
              for i in range(L)]
    for e in events:
        RestorePipeline.wait_for_layer_load(e)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for i in range(L):
        a = workloads.tokens_from_cache(fresh[i].cpu(), ids, T, True).view(torch.int16)
        b = workloads.tokens_from_cache(caches[i].cpu(), ids, T, True).view(torch.int16)
        assert torch.equal(a, b), i
    # the manifest describes the plane format the worker's restore hook dispatches on
    m = store.read_manifest("req:0")
    assert m["layers"][0]["quant_metadata"]["format"] == "origami_planes_v1"
    assert np.array_equal(np.asarray(m["layers"][2]["quant_metadata"]["chunk_specs"]), fmts[2].specs)
