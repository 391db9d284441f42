"""origami_fused_prefix_attention_noalloc (split workspace in a static device array) against
origami_fused_prefix_attention with a caller-provided workspace: bit-identical outputs on
two calls in a row (the second call reuses the static array the first one left behind),
and a clear error for shapes whose split plan does not fit the array."""
from __future__ import annotations

import ctypes
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))

from attention_cases import attention_case, cases  # noqa: E402

pytestmark = pytest.mark.gpu


def _dev(a: np.ndarray, dev) -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).to(dev)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _inputs(c, dev):
    qd = torch.bfloat16 if c["query_bf16"] else torch.float16
    cd = torch.bfloat16 if c["cache_bf16"] else torch.float16
    t = {k: _dev(c[k].reshape(-1), dev) for k in ("key_scale", "key_zero", "value_scale", "value_zero", "key_sink",
                                                   "value_sink")}
    t["bytestream"] = _dev(c["bytestream"], dev)
    t["query"] = _dev(c["query"], dev).view(qd)
    t["kv_cache"] = _dev(c["kv_cache"], dev).view(cd)
    t["block_table"] = _dev(c["block_table"], dev)
    return t


def _with_workspace(c, t) -> np.ndarray:
    from origami_b200 import attention

    out = torch.empty_like(t["query"])
    attention.fused_prefix_attention_cuda(
        t["bytestream"], c["key_offset"], c["key_bytes"], c["value_offset"], c["value_bytes"], c["codec"], c["bits"],
        c["group_size"], c["sink_tokens"], t["key_scale"], t["key_zero"], t["value_scale"], t["value_zero"],
        t["key_sink"], t["value_sink"], t["query"], t["kv_cache"], t["block_table"], c["prefix_tokens"],
        c["query_start"], c["sequence_length"], c["softmax_scale"], out)
    return out.view(torch.int16).cpu().numpy()


def _noalloc(c, t, flags) -> tuple[int, np.ndarray]:
    from origami_b200 import _lib
    from origami_b200.attention import _QDTYPE, _paged

    out = torch.empty_like(t["query"])
    q, cache = t["query"], t["kv_cache"]
    metas = [t[k] for k in ("key_scale", "key_zero", "value_scale", "value_zero", "key_sink", "value_sink")]
    numel = (ctypes.c_int64 * 6)(*[int(m.numel()) for m in metas])
    paged = _paged(cache)
    rc = _lib.lib().origami_fused_prefix_attention_noalloc(
        t["bytestream"].data_ptr(), t["bytestream"].numel(), c["key_offset"], c["key_bytes"], c["value_offset"],
        c["value_bytes"], c["codec"], c["bits"], c["group_size"], c["sink_tokens"], *[m.data_ptr() for m in metas],
        numel, _lib.ORIGAMI_DTYPE_F16, q.data_ptr(), _QDTYPE[q.dtype], q.shape[0], q.shape[1], q.shape[2],
        ctypes.byref(paged), _QDTYPE[cache.dtype], t["block_table"].data_ptr(), t["block_table"].numel(),
        c["prefix_tokens"], c["query_start"], c["sequence_length"], c["softmax_scale"], out.data_ptr(),
        flags.data_ptr(), torch.cuda.current_stream(q.device).cuda_stream)
    return rc, out.view(torch.int16).cpu().numpy()


@pytest.mark.parametrize("name", ["kivi_b2_long_decode", "kvquant_b4_ragged_gap", "kivi_b4_f16_q128",
                                  "kivi_b3_blocks_first_mixed_bad"])
def test_noalloc_matches_workspace_entry_point_on_two_calls(cuda, name):
    from origami_b200 import _lib, attention

    c = next(x for x in cases() if x["name"] == name)
    t = _inputs(c, cuda)
    want = _with_workspace(c, t)
    flags = torch.zeros(1, dtype=torch.int32, device=cuda)
    for call in range(2):
        rc, got = _noalloc(c, t, flags)
        _lib.check(rc, "origami_fused_prefix_attention_noalloc")
        np.testing.assert_array_equal(got, want, err_msg=f"call {call}")
    assert int(flags.item()) == 0
    kv_heads = int(t["kv_cache"].shape[3])
    if name == "kivi_b2_long_decode":  # this one splits its key range, so the static array is used
        assert attention.workspace_bytes(1, int(t["query"].shape[1]), kv_heads, c["query_start"],
                                         c["sequence_length"], cuda) > 0


def test_noalloc_rejects_plans_larger_than_the_static_array(cuda):
    from origami_b200 import _lib

    c = attention_case("big_plan", 77, codec=1, bits=4, prefix=8192, kv_heads=8, query_heads=32, query_tokens=16,
                       query_start=8300)
    t = _inputs(c, cuda)
    from origami_b200 import attention

    need = attention.workspace_bytes(int(t["query"].shape[0]), int(t["query"].shape[1]), int(t["kv_cache"].shape[3]),
                                     c["query_start"], c["sequence_length"], cuda)
    if need <= 8 << 20:  # the split count follows the SM count; this part splits the range less
        pytest.skip(f"this GPU's plan for the shape needs only {need} bytes")
    flags = torch.zeros(1, dtype=torch.int32, device=cuda)
    rc, _ = _noalloc(c, t, flags)
    assert rc != 0
    msg = _lib.lib().origami_last_error().decode()
    assert "static scratch holds 8388608" in msg and "bytes of split workspace" in msg
