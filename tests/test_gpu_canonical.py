"""GPU canonical pack / unpack (drop-in for the reference ops) against the CPU oracle
and against the reference's own CUDA kernel (oracle/_ref, built from its sources)."""
import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN, REPO
from origami_b200 import _lib
from origami_b200.lossless import native_cpu, native_gpu
from origami_b200.lossless.chunking import plan_head_channel_chunks

pytestmark = pytest.mark.gpu


def planner(H, D, T, target):
    return [c.layout.spec() for c in plan_head_channel_chunks(layer_index=0, num_heads=H, head_dim=D, token_count=T,
                                                               bytes_per_symbol=1, min_bytes=target,
                                                               target_bytes=target, max_bytes=target)]


def cases():
    rng = np.random.default_rng(5)
    out = []
    # tile path: head_dim innermost, full-token specs
    for (T, H, D, tgt) in [(37, 3, 16, 200), (1000, 2, 64, 5000), (4096, 4, 128, 1 << 17), (203, 2, 64, 4000),
                           (5, 1, 8, 16), (129, 8, 128, 1 << 20), (3000, 1, 256, 1 << 14)]:
        s = planner(H, D, T, tgt)
        out.append((["token", "head", "head_dim"], [T, H, D], s, [int(b) for b in rng.integers(1, 9, len(s))]))
        out.append((["head", "token", "head_dim"], [H, T, D], s, [8] * len(s)))
        out.append((["layer", "token", "head", "head_dim"], [1, T, H, D], s, [7] * len(s)))
    # linear path: token innermost, token sub-ranges, partial coverage, raw [1,1,N]
    out.append((["head", "head_dim", "token"], [2, 8, 50], [[0, 2, 0, 8, 0, 25], [0, 2, 0, 8, 25, 50]], [3, 5]))
    out.append((["layer", "head", "head_dim", "token"], [1, 4, 24, 33], [[0, 1, 0, 24, 0, 33], [2, 4, 4, 20, 3, 30]],
                [6, 2]))
    out.append((["token", "head", "head_dim"], [1, 1, 5_000_003],
                [[0, 1, a, min(a + (1 << 20), 5_000_003), 0, 1] for a in range(0, 5_000_003, 1 << 20)], [8] * 5))
    out.append((["token", "head_dim", "head"], [40, 12, 3], planner(3, 12, 40, 100), [4] * len(planner(3, 12, 40, 100))))
    out.append((["token", "head", "head_dim"], [64, 2, 16], [[1, 2, 0, 16, 0, 64]], [8]))  # head 0 uncovered
    return out


CASES = cases()


@pytest.mark.parametrize("i", range(len(CASES)))
def test_unpack_matches_oracle(oracle, cuda, i):
    layout, shape, specs, bits = CASES[i]
    rng = np.random.default_rng(100 + i)
    specs_np = np.asarray(specs, dtype=np.int64).reshape(-1, 6)
    n = (specs_np[:, 1] - specs_np[:, 0]) * (specs_np[:, 3] - specs_np[:, 2]) * (specs_np[:, 5] - specs_np[:, 4])
    sizes = (n * np.asarray(bits) + 7) // 8
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    flat = rng.integers(0, 256, int(offsets[-1]), dtype=np.uint8)
    want = oracle.unpack_canonical(flat, offsets, bits, specs_np, shape, layout)
    chunks = [torch.from_numpy(flat[a:b].copy()).to(cuda) for a, b in zip(offsets[:-1], offsets[1:])]
    got = native_gpu.unpack_canonical_storage_chunks(chunks, bits, shape, layout, specs_np, device=cuda)
    np.testing.assert_array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("i", range(len(CASES)))
def test_pack_matches_oracle(oracle, cuda, i):
    layout, shape, specs, bits = CASES[i]
    rng = np.random.default_rng(200 + i)
    sym = rng.integers(0, 256, int(np.prod(shape)), dtype=np.uint8)
    want, offsets = oracle.pack_canonical(sym, bits, specs, shape, layout)
    got = native_gpu.pack_canonical_storage_chunks(torch.from_numpy(sym).to(cuda), bits, shape, layout, specs)
    assert len(got) == len(specs)
    np.testing.assert_array_equal(torch.cat(got).cpu().numpy(), want)


def test_pack_overwrites_stale_output(oracle, cuda):
    """Masked word merges must clear stale bits of a reused output buffer."""
    T, H, D = 203, 2, 64
    specs = np.asarray(planner(H, D, T, 4000), dtype=np.int64)
    bits = [5] * len(specs)
    rng = np.random.default_rng(9)
    sym = rng.integers(0, 256, T * H * D, dtype=np.uint8)
    want, offsets = oracle.pack_canonical(sym, bits, specs, [T, H, D], ["token", "head", "head_dim"])
    L = _lib.lib()
    d_sym = torch.from_numpy(sym).to(cuda)
    out = torch.full(((int(offsets[-1]) + 15) // 16 * 16,), 0xFF, dtype=torch.uint8, device=cuda)
    bits_np = np.asarray(bits, dtype=np.int64)
    shape = np.asarray([T, H, D], dtype=np.int64)
    axes = np.asarray([0, 1, 2, -1], dtype=np.int64)
    d_off, d_bits, d_specs = (native_gpu.upload_i64(a, cuda) for a in (offsets, bits_np, specs))
    rc = L.origami_pack_canonical_storage_chunks(
        d_sym.data_ptr(), d_sym.numel(), d_off.data_ptr(), d_bits.data_ptr(), d_specs.data_ptr(), offsets.ctypes.data,
        bits_np.ctypes.data, specs.ctypes.data, len(specs), shape.ctypes.data, 3, axes.ctypes.data, T, H, D,
        out.data_ptr(), int(offsets[-1]), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "pack")
    got = out.cpu().numpy()
    np.testing.assert_array_equal(got[: int(offsets[-1])], want)
    assert (got[int(offsets[-1]):] == 0xFF).all()  # bytes past the chunks untouched


def test_drop_in_cpu_entry_points(oracle, cuda):
    """native_cpu.pack/unpack (stubs in the reference) return host tensors here."""
    T, H, D = 100, 4, 32
    specs = planner(H, D, T, 3000)
    sym = torch.randint(0, 256, (T * H * D,), dtype=torch.uint8)
    chunks = native_cpu.pack_head_channel_chunks(sym, 6, T, H, D, specs)
    assert all(c.device.type == "cpu" for c in chunks)
    want, offsets = oracle.pack_canonical(sym.numpy(), 6, specs, [T, H, D], ["token", "head", "head_dim"])
    np.testing.assert_array_equal(torch.cat(chunks).numpy(), want)
    back = native_cpu.unpack_head_channel_chunks(chunks, 6, T, H, D, specs)
    assert back.device.type == "cpu"
    np.testing.assert_array_equal(back.numpy(), sym.numpy() & 63)


def test_extension_surface_matches_reference_signature(oracle, cuda):
    ext = native_gpu.load_bitpack_cuda_extension()
    T, H, D = 40, 2, 16
    specs = np.asarray(planner(H, D, T, 300), dtype=np.int64)
    bits = np.full(len(specs), 7, dtype=np.int64)
    n = (specs[:, 1] - specs[:, 0]) * (specs[:, 3] - specs[:, 2]) * (specs[:, 5] - specs[:, 4])
    offsets = np.concatenate([[0], np.cumsum((n * 7 + 7) // 8)]).astype(np.int64)
    flat = np.random.default_rng(1).integers(0, 256, int(offsets[-1]), dtype=np.uint8)
    out = ext.unpack_canonical_storage_chunks_cuda(
        torch.from_numpy(flat).to(cuda), torch.from_numpy(offsets).to(cuda), torch.from_numpy(bits).to(cuda),
        torch.tensor([T, H, D]), torch.tensor([0, 1, 2, -1]), T, H, D, torch.from_numpy(specs).to(cuda))
    want = oracle.unpack_canonical(flat, offsets, bits, specs, [T, H, D], ["token", "head", "head_dim"])
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    with pytest.raises(_lib.OrigamiError, match="byte size mismatch"):
        bad = offsets.copy()
        bad[-1] += 1
        ext.unpack_canonical_storage_chunks_cuda(
            torch.from_numpy(flat).to(cuda), torch.from_numpy(bad).to(cuda), torch.from_numpy(bits).to(cuda),
            torch.tensor([T, H, D]), torch.tensor([0, 1, 2, -1]), T, H, D, torch.from_numpy(specs).to(cuda))


def _reference_extension():
    import importlib.util

    so = REPO / "oracle" / "_ref" / "origami_ref_bitpack.so"
    if not so.exists():
        pytest.skip("reference extension not built (oracle/build_ref.py)")
    spec = importlib.util.spec_from_file_location("origami_ref_bitpack", str(so))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("i", range(len(CASES)))
def test_reference_kernel_unpacks_our_pack(oracle, cuda, i):
    """Pack with origami_b200, unpack with the reference's own kernel: symbols return."""
    ref = _reference_extension()
    layout, shape, specs, bits = CASES[i]
    if int(np.prod(shape)) > 2_000_000:
        pytest.skip("reference kernel case kept small")
    rng = np.random.default_rng(300 + i)
    sym = rng.integers(0, 256, int(np.prod(shape)), dtype=np.uint8)
    chunks = native_gpu.pack_canonical_storage_chunks(torch.from_numpy(sym).to(cuda), bits, shape, layout, specs)
    flat = torch.cat(chunks)
    sizes = [c.numel() for c in chunks]
    offsets = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]), dtype=torch.int64, device=cuda)
    axes = native_cpu.axis_positions(layout)
    lay = native_cpu.normalize_symbol_layout(layout)
    out = ref.unpack_canonical_storage_chunks_cuda(
        flat, offsets, torch.tensor(bits, dtype=torch.int64, device=cuda), torch.tensor(shape, dtype=torch.int64),
        torch.tensor(axes, dtype=torch.int64), shape[lay.index("token")], shape[lay.index("head")],
        shape[lay.index("head_dim")], torch.tensor(specs, dtype=torch.int64, device=cuda))
    ours = native_gpu.unpack_canonical_storage_chunks(chunks, bits, shape, layout, specs, device=cuda)
    np.testing.assert_array_equal(out.cpu().numpy(), ours.cpu().numpy())
    want = oracle.unpack_canonical(torch.cat(chunks).cpu().numpy(), offsets.cpu().numpy(), bits, specs, shape, layout)
    np.testing.assert_array_equal(out.cpu().numpy(), want)


def test_matches_committed_reference_vectors(cuda):
    path = GOLDEN / "ref_unpack_vectors.npz"
    if not path.exists():
        pytest.skip("reference-kernel vectors not generated yet")
    z = np.load(path)
    for case in json.loads(bytes(z["index"]).decode()):
        flat = z[case["name"] + "__flat"]
        offs = case["offsets"]
        chunks = [torch.from_numpy(flat[a:b].copy()).to(cuda) for a, b in zip(offs[:-1], offs[1:])]
        got = native_gpu.unpack_canonical_storage_chunks(chunks, case["bits"], case["shape"], case["layout"],
                                                         case["specs"], device=cuda)
        np.testing.assert_array_equal(got.cpu().numpy(), z[case["name"] + "__out"], err_msg=case["name"])
