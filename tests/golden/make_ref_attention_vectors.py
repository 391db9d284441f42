"""Known-answer vectors of the reference's fused prefix attention kernel (run on a B200).

    python tests/golden/make_ref_attention_vectors.py [out.npz]

Loads the reference extension compiled from its own sources into oracle/_ref/
(oracle/build_ref.py; csrc/origami/bitpack_layout_cuda.{cpp,cu}) and runs its export
fused_prefix_attention_cuda (bitpack_layout_cuda.cpp:716-890, kernel cu:873-1091) on the
seeded cases of attention_cases.py. The kernel's outputs and a SHA-256 digest of every
seeded input array are stored (the inputs themselves are regenerated from their seeds);
the npz is committed as tests/golden/ref_attention_vectors.npz and pins the CPU oracle and
the origami_b200 kernel to the reference kernel within the reference test's tolerance.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parents[1]))

from attention_cases import cases  # noqa: E402
from make_ref_vectors import load_reference_extension  # noqa: E402


def _t(a, dev):
    import torch

    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).to(dev)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def run_reference(ext, c: dict) -> np.ndarray:
    import torch

    dev = torch.device("cuda", 0)
    qd = torch.bfloat16 if c["query_bf16"] else torch.float16
    cd = torch.bfloat16 if c["cache_bf16"] else torch.float16
    query = _t(c["query"], dev).view(qd)
    cache = _t(c["kv_cache"], dev).view(cd)
    out = torch.empty_like(query)
    ext.fused_prefix_attention_cuda(
        _t(c["bytestream"], dev), c["key_offset"], c["key_bytes"], c["value_offset"], c["value_bytes"], c["codec"],
        c["bits"], c["group_size"], c["sink_tokens"], _t(c["key_scale"].reshape(-1), dev),
        _t(c["key_zero"].reshape(-1), dev), _t(c["value_scale"].reshape(-1), dev),
        _t(c["value_zero"].reshape(-1), dev), _t(c["key_sink"].reshape(-1), dev),
        _t(c["value_sink"].reshape(-1), dev), query, cache, _t(c["block_table"], dev), c["prefix_tokens"],
        c["query_start"], c["sequence_length"], c["softmax_scale"], out)
    torch.cuda.synchronize()
    return out.view(torch.int16).cpu().numpy().view(np.uint16)


def digest(a: np.ndarray) -> np.ndarray:
    """SHA-256 of an array's dtype, shape and bytes, as 32 uint8."""
    h = hashlib.sha256(f"{a.dtype.str}{a.shape}".encode())
    h.update(np.ascontiguousarray(a).tobytes())
    return np.frombuffer(h.digest(), dtype=np.uint8)


def main(path: str) -> None:
    ext = load_reference_extension()
    if ext is None:
        raise SystemExit("reference extension not built (python oracle/build_ref.py)")
    store = {}
    for c in cases():
        out = run_reference(ext, c)
        for k, v in c.items():
            if isinstance(v, np.ndarray):
                store[f"{c['name']}/sha256/{k}"] = digest(v)
        store[f"{c['name']}/expected"] = out
        print(c["name"], out.shape, flush=True)
    np.savez_compressed(path, **store)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(HERE / "ref_attention_vectors.npz"))
