// Chunk-order ("linear") canonical pack/unpack for any source layout and any spec,
// including token sub-ranges and layouts whose innermost axis is not head_dim.
//
// Each thread owns 16 consecutive symbols of one chunk (16*bits bits = 2*bits whole
// bytes, so threads never share a packed byte). The symbol order and bit placement are
// those of the reference kernel (csrc/origami/bitpack_layout_cuda.cu:70-128); the tile
// kernels are the fast path, this one covers every remaining case.
#pragma once

#include "common.cuh"

namespace origami {

struct CanonStrides {
  int64_t st, sh, sc;  // element (= byte) strides of the token, head and head_dim axes
};

__device__ __forceinline__ uint32_t read_symbol(const uint8_t* src, int64_t src_bytes,
                                                int64_t symbol_index, int bits) {
  if (bits == 8) return src[symbol_index];
  const int64_t bit_pos = symbol_index * bits;
  const int64_t byte_idx = bit_pos >> 3;
  const int shift = static_cast<int>(bit_pos & 7);
  uint32_t packed = 0;
  if (byte_idx < src_bytes) packed = src[byte_idx];
  if (byte_idx + 1 < src_bytes) packed |= static_cast<uint32_t>(src[byte_idx + 1]) << 8;
  return (packed >> shift) & ((1u << bits) - 1u);
}

__global__ void __launch_bounds__(kThreads)
    canon_unpack_linear(const uint8_t* __restrict__ packed, const int64_t* __restrict__ offsets,
                        const int64_t* __restrict__ chunk_bits, const int64_t* __restrict__ specs,
                        CanonStrides ls, uint8_t* __restrict__ out) {
  const int64_t k = blockIdx.y;
  const int64_t* sp = specs + 6 * k;
  const int64_t h0 = sp[0], c0 = sp[2], t0 = sp[4];
  const int64_t C = sp[3] - sp[2];
  const int64_t TS = sp[5] - sp[4];
  const int64_t n = (sp[1] - sp[0]) * C * TS;
  const int bits = static_cast<int>(chunk_bits[k]);
  const int64_t base = offsets[k];
  const int64_t cbytes = offsets[k + 1] - base;
  const uint8_t* src = packed + base;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x * 16;
  for (int64_t L0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 16; L0 < n; L0 += step) {
    const int cnt = static_cast<int>(min64(16, n - L0));
    int64_t hh = L0 / (C * TS);
    const int64_t rem = L0 - hh * C * TS;
    int64_t cc = rem / TS;
    int64_t tt = rem - cc * TS;
    const int64_t first = (t0 + tt) * ls.st + (h0 + hh) * ls.sh + (c0 + cc) * ls.sc;
    // 16 contiguous destination bytes: along tokens (token stride 1) or along channels
    // (one token per run, head_dim stride 1).
    const bool contiguous = bits == 8 && cnt == 16 &&
                            ((ls.st == 1 && tt + 16 <= TS) || (TS == 1 && ls.sc == 1 && cc + 16 <= C));
    if (contiguous) {
      const uint8_t* s = src + L0;
      uint8_t* d = out + first;
      if (((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d)) & 15) == 0) {
        *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(s);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) d[i] = s[i];
      }
      continue;
    }
    for (int i = 0; i < cnt; ++i) {
      out[(t0 + tt) * ls.st + (h0 + hh) * ls.sh + (c0 + cc) * ls.sc] =
          static_cast<uint8_t>(read_symbol(src, cbytes, L0 + i, bits));
      if (++tt == TS) {
        tt = 0;
        if (++cc == C) {
          cc = 0;
          ++hh;
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads)
    canon_pack_linear(const uint8_t* __restrict__ symbols, const int64_t* __restrict__ offsets,
                      const int64_t* __restrict__ chunk_bits, const int64_t* __restrict__ specs,
                      CanonStrides ls, uint8_t* __restrict__ packed) {
  const int64_t k = blockIdx.y;
  const int64_t* sp = specs + 6 * k;
  const int64_t h0 = sp[0], c0 = sp[2], t0 = sp[4];
  const int64_t C = sp[3] - sp[2];
  const int64_t TS = sp[5] - sp[4];
  const int64_t n = (sp[1] - sp[0]) * C * TS;
  const int bits = static_cast<int>(chunk_bits[k]);
  const uint32_t mask = (1u << bits) - 1u;
  uint8_t* dst = packed + offsets[k];
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x * 16;
  for (int64_t L0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 16; L0 < n; L0 += step) {
    const int cnt = static_cast<int>(min64(16, n - L0));
    int64_t hh = L0 / (C * TS);
    const int64_t rem = L0 - hh * C * TS;
    int64_t cc = rem / TS;
    int64_t tt = rem - cc * TS;
    uint64_t acc[2] = {0u, 0u};
    for (int i = 0; i < cnt; ++i) {
      const uint64_t s =
          symbols[(t0 + tt) * ls.st + (h0 + hh) * ls.sh + (c0 + cc) * ls.sc] & mask;
      const int pos = i * bits;  // < 128
      acc[pos >> 6] |= s << (pos & 63);
      if ((pos & 63) + bits > 64) acc[1] |= s >> (64 - (pos & 63));
      if (++tt == TS) {
        tt = 0;
        if (++cc == C) {
          cc = 0;
          ++hh;
        }
      }
    }
    const int64_t b0 = (L0 * bits) >> 3;  // L0 is a multiple of 16: byte aligned
    const int nbytes = static_cast<int>((((L0 + cnt) * bits + 7) >> 3) - b0);
    uint8_t* d = dst + b0;
    if (nbytes == 16 && (reinterpret_cast<uintptr_t>(d) & 15) == 0) {
      *reinterpret_cast<uint4*>(d) =
          make_uint4(static_cast<uint32_t>(acc[0]), static_cast<uint32_t>(acc[0] >> 32),
                     static_cast<uint32_t>(acc[1]), static_cast<uint32_t>(acc[1] >> 32));
    } else {
      for (int j = 0; j < nbytes; ++j) d[j] = static_cast<uint8_t>(acc[j >> 3] >> (8 * (j & 7)));
    }
  }
}

// ---------------------------------------------------------------------------------------
// Raw block gather / scatter (index_select / index_copy_ along the block dimension).
// A slab is the contiguous run of one block: bs*H*D elements per (kv, block) for the
// KV-first layout, 2*bs*H*D per block for the blocks-first layout.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads)
    gather_slabs(const uint8_t* __restrict__ cache, int64_t slab_bytes, int64_t slabs_per_block_id,
                 int64_t num_cache_blocks, const int64_t* __restrict__ ids, int64_t nb,
                 uint8_t* __restrict__ out, uint32_t* err) {
  const int64_t vec = slab_bytes >> 4;
  for (int64_t q = blockIdx.x; q < slabs_per_block_id * nb; q += gridDim.x) {
    const int64_t kv = q / nb;
    const int64_t j = q - kv * nb;
    const int64_t blk = ids[j];
    uint4* d = reinterpret_cast<uint4*>(out + q * slab_bytes);
    if (blk < 0 || blk >= num_cache_blocks) {
      if (threadIdx.x == 0 && err) atomicAdd(err, 1u);
      for (int64_t v = threadIdx.x; v < vec; v += kThreads) d[v] = make_uint4(0u, 0u, 0u, 0u);
      continue;
    }
    const uint4* s = reinterpret_cast<const uint4*>(cache + (kv * num_cache_blocks + blk) * slab_bytes);
    for (int64_t v = threadIdx.x; v < vec; v += kThreads) st_global_cs16(d + v, __ldg(s + v));
  }
}

__global__ void __launch_bounds__(kThreads)
    scatter_slabs(const uint8_t* __restrict__ in, int64_t slab_bytes, int64_t slabs_per_block_id,
                  int64_t num_cache_blocks, const int64_t* __restrict__ ids, int64_t nb,
                  uint8_t* __restrict__ cache, uint32_t* err) {
  const int64_t vec = slab_bytes >> 4;
  for (int64_t q = blockIdx.x; q < slabs_per_block_id * nb; q += gridDim.x) {
    const int64_t kv = q / nb;
    const int64_t j = q - kv * nb;
    const int64_t blk = ids[j];
    if (blk < 0 || blk >= num_cache_blocks) {
      if (threadIdx.x == 0 && err) atomicAdd(err, 1u);
      continue;
    }
    const uint4* s = reinterpret_cast<const uint4*>(in + q * slab_bytes);
    uint4* d = reinterpret_cast<uint4*>(cache + (kv * num_cache_blocks + blk) * slab_bytes);
    for (int64_t v = threadIdx.x; v < vec; v += kThreads) st_global_cs16(d + v, __ldg(s + v));
  }
}

}  // namespace origami
