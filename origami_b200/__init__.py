"""origami_b200: B200-native (sm_100a) KV layout hot path of Origami.

Save side: paged bf16/fp16 KV blocks -> byte/bit planes -> canonical chunks for the
host lossless codec. Restore side: the inverse, scattered straight into the paged
cache. Kernels live in liborigami_b200.so (C ABI: include/origami_b200.h).
"""
from origami_b200.planes import (BF16_BIT_PLANES, BYTE_PLANES, FP16_BIT_PLANES, LayerFormat, PlaneSpec,
                                 plane_spec)

__all__ = ["BYTE_PLANES", "BF16_BIT_PLANES", "FP16_BIT_PLANES", "LayerFormat", "PlaneSpec", "plane_spec"]
__version__ = "0.1.0"
