"""Host lossless codec at the boundary of the GPU path.

Mirrors the reference's CpuLosslessCodec (lossless/cpu_qat.py:12-134) for the software
backends: raw DEFLATE at zlib level 1 with wbits=-15, or the identity ``raw`` backend.
The Intel QAT backend is hardware this build does not target; requesting it raises
unless ``allow_zlib_fallback`` is set, as in the reference. The codec stays on the
host: the GPU path ends at the packed chunks.
"""
from __future__ import annotations

import zlib
from concurrent.futures import ThreadPoolExecutor

import torch


class CpuLosslessCodec:
    def __init__(self, backend: str = "zlib", allow_zlib_fallback: bool = False, *, threads: int = 0,
                 **_qat_tuning):
        self.backend = backend
        self.allow_zlib_fallback = allow_zlib_fallback
        self.qat_codec = "qat_codec"
        if backend == "qat":
            if not allow_zlib_fallback:
                raise RuntimeError(
                    "Origami QAT backend is not available. Set origami_lossless_cpu_backend='zlib' for tests or "
                    "enable origami_allow_zlib_fallback for development.")
            self.backend = "zlib"
        elif backend not in {"zlib", "raw"}:
            raise ValueError(f"Unsupported Origami CPU lossless backend {backend!r}")
        self._pool = ThreadPoolExecutor(max_workers=threads) if threads > 1 else None

    @staticmethod
    def _cpu_u8(data: torch.Tensor) -> torch.Tensor:
        return data.detach().cpu().to(torch.uint8).reshape(-1).contiguous()

    @staticmethod
    def _zlib_compress(data: torch.Tensor) -> torch.Tensor:
        flat = CpuLosslessCodec._cpu_u8(data)
        c = zlib.compressobj(level=1, wbits=-15, strategy=zlib.Z_DEFAULT_STRATEGY)
        enc = c.compress(flat.numpy().tobytes()) + c.flush()
        return torch.frombuffer(bytearray(enc), dtype=torch.uint8).clone()

    @staticmethod
    def _zlib_decompress(data: torch.Tensor, output_bytes: int) -> torch.Tensor:
        flat = CpuLosslessCodec._cpu_u8(data)
        dec = zlib.decompress(flat.numpy().tobytes(), wbits=-15)
        if len(dec) != int(output_bytes):
            raise RuntimeError(f"Origami CPU lossless decoded {len(dec)} bytes, expected {int(output_bytes)}")
        return torch.frombuffer(bytearray(dec), dtype=torch.uint8).clone()

    def _map(self, fn, *iters):
        if self._pool is not None:
            return list(self._pool.map(fn, *iters))
        return [fn(*a) for a in zip(*iters)]

    def compress_many(self, chunks) -> list[torch.Tensor]:
        if self.backend == "raw":
            return [self._cpu_u8(c) for c in chunks]
        return self._map(self._zlib_compress, list(chunks))

    def decompress_many(self, chunks, output_bytes) -> list[torch.Tensor]:
        if len(chunks) != len(output_bytes):
            raise ValueError("chunks and output_bytes must have the same length")
        if self.backend == "raw":
            out = []
            for c, n in zip(chunks, output_bytes):
                flat = self._cpu_u8(c)
                if int(flat.numel()) != int(n):
                    raise RuntimeError(f"Origami raw backend received {int(flat.numel())} bytes, expected {int(n)}")
                out.append(flat)
            return out
        return self._map(self._zlib_decompress, list(chunks), [int(n) for n in output_bytes])

    def compress(self, data: torch.Tensor) -> torch.Tensor:
        return self.compress_many([data])[0]

    def decompress(self, data: torch.Tensor, *, output_bytes: int) -> torch.Tensor:
        return self.decompress_many([data], [int(output_bytes)])[0]
