"""Known-answer vectors of the reference's GPU unpack kernel (run on a B200).

    python tests/golden/make_ref_vectors.py [out.npz]

Loads the reference extension compiled from its own sources into oracle/_ref/
(oracle/build_ref.py; csrc/origami/bitpack_layout_cuda.{cpp,cu}), feeds it seeded packed
chunk streams over a set of layouts, bit widths and chunk specs (token sub-ranges,
partial coverage, multi-head chunks, the raw [1, 1, N] layout) and stores inputs and
the kernel's outputs. The npz is committed as tests/golden/ref_unpack_vectors.npz and
pins the CPU oracle to the reference kernel bit for bit.
"""
from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
REF_SO = REPO / "oracle" / "_ref" / "origami_ref_bitpack.so"


def load_reference_extension():
    import torch  # noqa: F401  (provides the ATen symbols the extension links against)

    if not REF_SO.exists():
        return None
    spec = importlib.util.spec_from_file_location("origami_ref_bitpack", str(REF_SO))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def axis_positions(layout):
    return [layout.index("token"), layout.index("head"), layout.index("head_dim"),
            layout.index("layer") if "layer" in layout else -1]


def planner_specs(H, D, T, target):
    sys.path.insert(0, str(REPO))
    from origami_b200.lossless.chunking import plan_head_channel_chunks

    return [c.layout.spec() for c in plan_head_channel_chunks(
        layer_index=0, num_heads=H, head_dim=D, token_count=T, bytes_per_symbol=1, min_bytes=target,
        target_bytes=target, max_bytes=target)]


def cases():
    rng = np.random.default_rng(7)
    out = []
    s = planner_specs(3, 16, 37, 200)
    out.append(("planner_thd", ["token", "head", "head_dim"], [37, 3, 16], s,
                [int(b) for b in rng.integers(1, 9, len(s))]))
    out.append(("token_subranges", ["head", "head_dim", "token"], [2, 8, 50],
                [[0, 2, 0, 8, 0, 25], [0, 2, 0, 8, 25, 50]], [3, 5]))
    out.append(("partial_layer4", ["layer", "head", "head_dim", "token"], [1, 4, 24, 33],
                [[0, 1, 0, 24, 0, 33], [2, 4, 4, 20, 3, 30]], [6, 2]))
    out.append(("raw_bytes", ["token", "head", "head_dim"], [1, 1, 5000],
                [[0, 1, 0, 1024, 0, 1], [0, 1, 1024, 2048, 0, 1], [0, 1, 2048, 3072, 0, 1],
                 [0, 1, 3072, 4096, 0, 1], [0, 1, 4096, 5000, 0, 1]], [8, 8, 8, 8, 8]))
    s = planner_specs(3, 40, 21, 300)
    out.append(("htd_bits7", ["head", "token", "head_dim"], [3, 21, 40], s, [7] * len(s)))
    for b in (8, 7, 1, 6, 2):
        s = planner_specs(8, 128, 64, 16 << 10)
        out.append((f"plane_component_b{b}", ["token", "head", "head_dim"], [64, 8, 128], s, [b] * len(s)))
    s = planner_specs(2, 64, 203, 4000)
    out.append(("ragged_tokens", ["token", "head", "head_dim"], [203, 2, 64], s,
                [int(b) for b in rng.integers(1, 9, len(s))]))
    return out


def main(path: str) -> None:
    import torch

    ext = load_reference_extension()
    if ext is None:
        raise SystemExit(f"reference extension not built at {REF_SO}")
    rng = np.random.default_rng(11)
    arrays = {}
    index = []
    for name, layout, shape, specs, bits in cases():
        specs_np = np.asarray(specs, dtype=np.int64).reshape(-1, 6)
        n = (specs_np[:, 1] - specs_np[:, 0]) * (specs_np[:, 3] - specs_np[:, 2]) * (specs_np[:, 5] - specs_np[:, 4])
        sizes = (n * np.asarray(bits) + 7) // 8
        offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
        flat = rng.integers(0, 256, int(offsets[-1]), dtype=np.uint8)
        dev = torch.device("cuda")
        out = ext.unpack_canonical_storage_chunks_cuda(
            torch.from_numpy(flat).to(dev), torch.from_numpy(offsets).to(dev),
            torch.tensor(bits, dtype=torch.int64, device=dev), torch.tensor(shape, dtype=torch.int64),
            torch.tensor(axis_positions(layout), dtype=torch.int64),
            int(shape[layout.index("token")]), int(shape[layout.index("head")]), int(shape[layout.index("head_dim")]),
            torch.from_numpy(specs_np).to(dev))
        torch.cuda.synchronize()
        arrays[f"{name}__flat"] = flat
        arrays[f"{name}__out"] = out.cpu().numpy()
        index.append({"name": name, "layout": layout, "shape": shape, "specs": specs_np.tolist(),
                      "bits": [int(b) for b in bits], "offsets": offsets.tolist()})
    arrays["index"] = np.frombuffer(json.dumps(index).encode(), dtype=np.uint8)
    np.savez_compressed(path, **arrays)
    print("wrote", path, len(index), "cases")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(REPO / "tests" / "golden" / "ref_unpack_vectors.npz"))
