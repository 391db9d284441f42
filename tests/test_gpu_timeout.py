"""The bounded-wait bail-out of the TMA / bulk-copy layer kernels, on a wait that cannot
complete: an mbarrier that expects bytes no copy delivers (nothing is in flight, so the
run is safe by construction). The kernel must give up, report bit 31 in the error word and
leave the context usable."""
import pytest
import torch

from origami_b200 import BYTE_PLANES, LayerFormat, _lib, workloads
from origami_b200.layer import pack_layer, restore_layer

pytestmark = pytest.mark.gpu

TIMEOUT_FLAG = 0x80000000


def test_wait_that_cannot_complete_reports_the_timeout_flag(cuda):
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream(cuda)
    with torch.cuda.device(cuda):
        rc = _lib.lib().origami_selftest_wait_timeout(err.data_ptr(), 1000, stream.cuda_stream)
    _lib.check(rc, "origami_selftest_wait_timeout")
    torch.cuda.synchronize(cuda)
    word = int(err.item()) & 0xFFFFFFFF
    assert word == TIMEOUT_FLAG  # flagged, and the "phase completed" path was not taken

    # the context is still usable: a layer round trip right after works
    T, bs, H, D = 256, 16, 2, 128
    nb = T // bs
    ids = workloads.permuted_block_table(nb, nb, seed=1)
    cache = torch.randint(-32768, 32767, (2, nb, bs, H, D), dtype=torch.int16).view(torch.bfloat16).to(cuda)
    fmt = LayerFormat(T, H, D, BYTE_PLANES)
    packed = pack_layer(cache, ids, fmt)
    fresh = torch.zeros_like(cache)
    restore_layer(packed, fmt, fresh, ids)
    assert torch.equal(fresh.view(torch.int16), cache.view(torch.int16))


def test_selftest_rejects_bad_arguments(cuda):
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    with pytest.raises(_lib.OrigamiError, match="polls"):
        _lib.check(_lib.lib().origami_selftest_wait_timeout(err.data_ptr(), 0, None), "selftest")
