"""Known-answer vectors of the reference's quantized restore kernels (run on a B200).

    python tests/golden/make_ref_quant_vectors.py [out.npz]

Loads the reference extension compiled from its own sources into oracle/_ref/
(oracle/build_ref.py; csrc/origami/bitpack_layout_cuda.{cpp,cu}) and runs its exports
cachegen_unpack_dequantize_to_kv_cache_cuda, cachegen_unpack_dequantize_cuda and
kivi_dequantize_to_kv_cache_cuda (bitpack_layout_cuda.cpp:402-700) on the seeded cases of
quant_cases.py. Inputs and the kernels' outputs are stored; the npz is committed as
tests/golden/ref_quant_vectors.npz and pins the CPU oracle to the reference kernels bit
for bit.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parents[1]))

from make_ref_vectors import load_reference_extension  # noqa: E402
from quant_cases import cases  # noqa: E402


def _t(a, dev):
    import torch

    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).to(dev)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def run_reference(ext, c: dict) -> np.ndarray:
    import torch

    dev = torch.device("cuda", 0)
    stream = _t(c["bytestream"], dev)
    if c["kind"] == "cg_unpack":
        out = ext.cachegen_unpack_dequantize_cuda(stream, _t(c["offsets"], dev), _t(c["bits"], dev),
                                                  _t(c["key_bins"], dev), _t(c["value_bins"], dev),
                                                  _t(c["max_key"], dev), _t(c["max_value"], dev), c["tokens"],
                                                  c["heads"], c["head_dim"])
        torch.cuda.synchronize()
        return out.cpu().view(torch.int16).numpy().view(np.uint16)
    dtype = torch.bfloat16 if c["out_bf16"] else torch.float16
    cache = _t(c["cache"], dev).view(dtype)
    ids = _t(c["block_ids"], dev)
    if c["kind"] == "cg_cache":
        ext.cachegen_unpack_dequantize_to_kv_cache_cuda(
            stream, c["key_offset"], c["key_bytes"], c["value_offset"], c["value_bytes"], c["key_bits"],
            c["value_bits"], c["key_bins"], c["value_bins"], _t(c["max_key"], dev), _t(c["max_value"], dev), cache,
            ids, c["tokens"], c["heads"], c["head_dim"])
    else:
        ext.kivi_dequantize_to_kv_cache_cuda(
            stream, c["key_offset"], c["key_bytes"], c["value_offset"], c["value_bytes"], c["bits"],
            c["group_size"], c["sink_tokens"], _t(c["key_scale"], dev), _t(c["key_zero"], dev),
            _t(c["value_scale"], dev), _t(c["value_zero"], dev), _t(c["key_sink"], dev), _t(c["value_sink"], dev),
            cache, ids, c["tokens"], c["heads"], c["head_dim"])
    torch.cuda.synchronize()
    return cache.view(torch.int16).cpu().numpy().view(np.uint16)


def main(path: str) -> None:
    ext = load_reference_extension()
    if ext is None:
        raise SystemExit("reference extension not built (python oracle/build_ref.py)")
    store = {}
    for c in cases():
        out = run_reference(ext, c)
        for k, v in c.items():
            if isinstance(v, np.ndarray):
                store[f"{c['name']}/{k}"] = v
        store[f"{c['name']}/expected"] = out
        print(c["name"], out.shape)
    np.savez_compressed(path, **store)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(HERE / "ref_quant_vectors.npz"))
