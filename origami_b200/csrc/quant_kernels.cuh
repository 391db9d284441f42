// Fused dequantize-to-paged-cache kernels for the reference's lossy restore paths:
//
//  cachegen_to_cache  <- cachegen_unpack_dequantize_to_kv_cache_kernel
//                        (csrc/origami/bitpack_layout_cuda.cu:348-423)
//  cachegen_unpack    <- cachegen_unpack_dequantize_kernel (bitpack_layout_cuda.cu:141-185)
//  kivi_to_cache      <- kivi_dequantize_to_kv_cache_kernel (bitpack_layout_cuda.cu:577-683)
//  kivi_to_cache_elem    (same op, one element per thread, for shapes the tile kernel
//                        does not cover)
//
// Arithmetic is the reference's, step for step, so the results are bit-identical:
//  CacheGen: value = ((float(s) - c) / c) * max[token], c = float(bins / 2 - 1); the
//            quotient depends on s only, so it is tabulated once per CTA (one IEEE
//            division per symbol value) and every element costs one multiply.
//  KIVI:     value = fma(float(s), scale, zero) (the reference's s * scale + zero, which
//            nvcc contracts to one fused multiply-add), sink tokens copied from the sink
//            tensors; out-of-range block ids are skipped (and counted).
//  Symbols are dense LSB-first at `bits` per symbol; bytes at or past a stream's length
//  read as zero (unpack_symbol_direct, bitpack_layout_cuda.cu:295-312), except that
//  8-bit symbols, which the reference reads unchecked, run on to the bytestream's end
//  (the host passes that limit).
//
// Layout work differs from the reference: CacheGen streams are token-major, so a warp
// decodes one (kv, token) row of the paged cache with 16-byte stores; KIVI streams are
// channel-major (value: head > head_dim > token, key: head_dim > head > token), so a
// CTA stages TT-token runs of every channel of one head, transposes 8x8 symbol blocks in
// registers and writes whole cache rows.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace origami {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ uint32_t out_bits(float v);
template <>
__device__ __forceinline__ uint32_t out_bits<__half>(float v) {
  return __half_as_ushort(__float2half_rn(v));
}
template <>
__device__ __forceinline__ uint32_t out_bits<__nv_bfloat16>(float v) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// Two elements rounded to nearest-even in one paired conversion (lo in bits 0-15): the
// same bits as two out_bits calls.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  const __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// One symbol with the reference's bounds rule.
__device__ __forceinline__ uint32_t symbol_at(const uint8_t* s, int64_t nbytes, int64_t index, int bits) {
  if (bits == 8) return index < nbytes ? s[index] : 0u;
  const int64_t bit = index * bits;
  const int64_t byte = bit >> 3;
  uint32_t w = byte < nbytes ? s[byte] : 0u;
  if (byte + 1 < nbytes) w |= static_cast<uint32_t>(s[byte + 1]) << 8;
  return (w >> (bit & 7)) & ((1u << bits) - 1u);
}

// The 64 bits holding symbols 8k .. 8k+7 of a stream (they start on a byte boundary: byte
// k * bits), as two aligned 8-byte loads; bytes at or past nbytes read as zero.
__device__ __forceinline__ uint64_t symbols8_raw(const uint8_t* s, int64_t nbytes, int64_t k, int bits) {
  const int64_t byte = k * bits;
  if (byte + bits <= nbytes) {
    const uintptr_t addr = reinterpret_cast<uintptr_t>(s + byte);
    const uint64_t* p = reinterpret_cast<const uint64_t*>(addr & ~static_cast<uintptr_t>(7));
    const int sh = static_cast<int>(addr & 7) * 8;
    uint64_t v = __ldg(p) >> sh;
    if (sh + 8 * bits > 64) v |= __ldg(p + 1) << (64 - sh);
    return v;
  }
  uint64_t v = 0;
  for (int j = 0; j < bits; ++j)
    if (byte + j < nbytes) v |= static_cast<uint64_t>(s[byte + j]) << (8 * j);
  return v;
}

// Eight b-bit symbols of a 64-bit field (symbol k at bits [k*b, (k+1)*b)) -> eight
// dequantized elements q[s] * m, packed as 16 bytes. Symbols 0..3 come from the low word,
// 4..7 from the field shifted by 4*b; each is one shift and one mask from its table index.
template <typename OUT>
__device__ __forceinline__ uint4 dequant8(const float* q, float m, uint64_t field, int bits) {
  const uint32_t mask = (1u << bits) - 1u;
  const uint32_t w[2] = {static_cast<uint32_t>(field), static_cast<uint32_t>(field >> (4 * bits))};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t x = w[j >> 1];
    const int k = 2 * (j & 1);
    const uint32_t e0 = out_bits<OUT>(q[(x >> (k * bits)) & mask] * m);
    const uint32_t e1 = out_bits<OUT>(q[(x >> ((k + 1) * bits)) & mask] * m);
    o[j] = __byte_perm(e0, e1, 0x5410);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// ---------------------------------------------------------------------------------------
// CacheGen -> paged cache
// ---------------------------------------------------------------------------------------
struct CgArgs {
  const uint8_t* stream[2];  // key, value
  int64_t stream_bytes[2];
  int32_t bits[2];
  int64_t bins[2];
  const void* maxv[2];  // [tokens] per stream (float or half)
  uint8_t* cache;
  const int64_t* ids;
  int64_t kv_stride, block_stride, token_stride;  // elements
  int64_t num_blocks, block_size, tokens;
  int32_t heads;
  int32_t C;     // heads * head_dim
  int32_t nvec;  // C / 8 (vector path) or C (scalar path)
  uint32_t* err;
};

__device__ __forceinline__ void cg_table(float (*table)[256], const int64_t* bins) {
  for (int i = threadIdx.x; i < 512; i += blockDim.x) {
    const int kv = i >> 8;
    const float center = static_cast<float>(bins[kv] / 2 - 1);
    table[kv][i & 255] = (static_cast<float>(i & 255) - center) / center;
  }
  __syncthreads();
}

// Eight b-bit symbols of a 64-bit field -> eight output elements looked up by warp shuffle:
// lane l holds `lut`, the finished 16-bit element for symbol value l (b <= 5). All 32 lanes
// must execute it.
__device__ __forceinline__ uint4 lookup8_shfl(uint32_t lut, uint64_t field, int bits) {
  const uint32_t mask = (1u << bits) - 1u;
  const uint32_t w[2] = {static_cast<uint32_t>(field), static_cast<uint32_t>(field >> (4 * bits))};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t x = w[j >> 1];
    const int k = 2 * (j & 1);
    const uint32_t e0 = __shfl_sync(0xFFFFFFFFu, lut, static_cast<int>((x >> (k * bits)) & mask));
    const uint32_t e1 = __shfl_sync(0xFFFFFFFFu, lut, static_cast<int>((x >> ((k + 1) * bits)) & mask));
    o[j] = __byte_perm(e0, e1, 0x5410);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// One (kv, token) row of BITS-bit symbols (BITS <= 5) by shuffle lookups: lane l's vectors
// v = l, l + 32, ... of eight symbols each, one 16-byte store per vector. The constant
// width turns every field shift and mask into an immediate.
template <int BITS, typename OUT>
__device__ __forceinline__ void cg_row_shfl(const uint8_t* s, int64_t nb, int64_t k0, int nvec, uint32_t lut, OUT* dst,
                                            int lane) {
  for (int v0 = 0; v0 < nvec; v0 += 32) {
    const int v = v0 + lane;
    const uint64_t field = v < nvec ? symbols8_raw(s, nb, k0 + v, BITS) : 0;
    const uint4 out = lookup8_shfl(lut, field, BITS);
    if (v < nvec) st_global_cs16(dst + 8 * v, out);
  }
}

// A warp per (kv, token) row; VEC: eight symbols -> one 16-byte store per lane step.
// Symbols of up to 5 bits (every CacheGen bins setting of the reference,
// cachegen_adapter.py:49-57) are dequantized by shuffle: each lane computes the finished
// element for one symbol value, ((v - c) / c) * max then the output rounding, exactly as the
// reference does per element, and the other lanes fetch it. Wider symbols go through the
// shared-memory quotient table, a multiply and a conversion per element.
// Launched with programmatic dependent launch (the kernel after it may be scheduled early;
// this one waits for the kernel before it ahead of any global access).
__device__ __forceinline__ void dependent_launch_entry() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
}

template <typename MAXT, typename OUT, bool VEC>
__global__ void __launch_bounds__(kThreads) cachegen_to_cache(const __grid_constant__ CgArgs a) {
  __shared__ float table[2][256];
  dependent_launch_entry();
  cg_table(table, a.bins);
  const int lane = threadIdx.x & 31;
  const int64_t rows = 2 * a.tokens;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
  for (int64_t row = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); row < rows; row += warps) {
    const int kv = row >= a.tokens ? 1 : 0;
    const int64_t t = row - kv * a.tokens;
    const int64_t bi = static_cast<int32_t>(t) / static_cast<int32_t>(a.block_size);
    const uint8_t* s = a.stream[kv];
    const int64_t nb = a.stream_bytes[kv];
    const int bits = a.bits[kv];
    const float m = to_f32(static_cast<const MAXT*>(a.maxv[kv])[t]);
    const int64_t blk = a.ids[bi];
    if (blk < 0 || blk >= a.num_blocks) {  // counted per (kv, token, head) row
      if (lane == 0 && a.err) atomicAdd(a.err, static_cast<uint32_t>(a.heads));
      continue;
    }
    OUT* dst = reinterpret_cast<OUT*>(a.cache) + kv * a.kv_stride + blk * a.block_stride +
               (t - bi * a.block_size) * a.token_stride;
    if constexpr (VEC) {
      if (bits <= 5) {
        const uint32_t lut = out_bits<OUT>(table[kv][lane] * m);
        const int64_t k0 = t * a.nvec;
        switch (bits) {  // warp-uniform
          case 5: cg_row_shfl<5, OUT>(s, nb, k0, a.nvec, lut, dst, lane); break;
          case 4: cg_row_shfl<4, OUT>(s, nb, k0, a.nvec, lut, dst, lane); break;
          case 3: cg_row_shfl<3, OUT>(s, nb, k0, a.nvec, lut, dst, lane); break;
          case 2: cg_row_shfl<2, OUT>(s, nb, k0, a.nvec, lut, dst, lane); break;
          default: cg_row_shfl<1, OUT>(s, nb, k0, a.nvec, lut, dst, lane); break;
        }
      } else {
        for (int v = lane; v < a.nvec; v += 32)
          st_global_cs16(dst + 8 * v, dequant8<OUT>(table[kv], m, symbols8_raw(s, nb, t * a.nvec + v, bits), bits));
      }
    } else {
      for (int c = lane; c < a.C; c += 32) {
        const uint32_t sym = symbol_at(s, nb, t * a.C + c, bits);
        reinterpret_cast<uint16_t*>(dst)[c] = static_cast<uint16_t>(out_bits<OUT>(table[kv][sym] * m));
      }
    }
  }
}

// Staged CacheGen -> paged cache (VEC rows, symbols of at most 5 bits on both streams).
//
// Rows are taken in groups of kCgGroupRows consecutive tokens of one stream. A group's
// symbol bytes are contiguous, so one thread brings them into shared memory with one bulk
// copy (from the 16-byte line holding the first byte; two stages, bounded mbarrier waits),
// and the group's max values and block ids are fetched into registers one group ahead. A
// warp decodes kCgRowsPerWarp rows from shared memory: lane l's fields of vectors l + 32 i
// (one routine per symbol width), the shuffle lookup of cachegen_to_cache (each lane
// computes the finished element for one symbol value), one 16-byte store per vector. A
// group whose bytes reach the stream's read limit or the end of the bytestream is decoded
// from global memory, with the reference's bounds rule, instead. 32-row groups and 4 CTAs
// an SM (64 registers) measured fastest (8- and 16-row groups pay the group barriers and
// fetches too often; 64-row stages leave 2 CTAs an SM).
constexpr int kCgRowsPerWarp = 4;
constexpr int kCgGroupRows = kCgRowsPerWarp * (kThreads / 32);

struct CgStageGeo {
  // per stage: kCgGroupRows rows of the wider stream + one line + 8 bytes of read slack
  __host__ __device__ static int bytes_for(int64_t row_bytes) {
    return static_cast<int>(((kCgGroupRows * row_bytes + 16 + 8) + 127) / 128 * 128);
  }
};

// The 8 * BITS bits of a vector's symbols from byte p of a staged row (BITS <= 5, so they
// lie in the two aligned 32-bit words from p & ~3; the stage has 8 bytes of read slack).
template <int BITS>
__device__ __forceinline__ uint64_t field_from_smem(const uint8_t* p) {
  static_assert(BITS <= 5, "a field of at most 40 bits");
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~static_cast<uintptr_t>(3));
  const int sh = static_cast<int>(a & 3) * 8;
  const uint32_t w0 = w[0], w1 = w[1];
  return (static_cast<uint64_t>(w1 >> sh) << 32) | __funnelshift_r(w0, w1, sh);
}

// Eight BITS-bit symbols -> eight output elements by warp shuffle within segments of
// 2^BITS lanes: lane l holds the finished element for symbol value l mod 2^BITS, and the
// shuffle takes its source lane modulo the segment width, so a symbol's field needs a shift
// but no mask. All 32 lanes must execute it.
template <int BITS>
__device__ __forceinline__ uint4 lookup8_seg(uint32_t lut, uint64_t field) {
  constexpr int W = 1 << BITS;
  const uint32_t w[2] = {static_cast<uint32_t>(field), static_cast<uint32_t>(field >> (4 * BITS))};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t x = w[j >> 1];
    const int k = 2 * (j & 1);
    const uint32_t e0 = __shfl_sync(0xFFFFFFFFu, lut, static_cast<int>(x >> (k * BITS)), W);
    const uint32_t e1 = __shfl_sync(0xFFFFFFFFu, lut, static_cast<int>(x >> ((k + 1) * BITS)), W);
    o[j] = __byte_perm(e0, e1, 0x5410);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// One row of BITS-bit symbols: lane l's vectors l, l + 32, ... from the staged row (STAGED)
// or, for a group that reaches the stream's read limit, from global memory with the
// reference's bounds rule.
template <int BITS, bool STAGED, typename OUT>
__device__ __forceinline__ void cg_row_seg(const uint8_t* row, const uint8_t* gs, int64_t nb, int64_t k0, int nvec,
                                           uint32_t lut, OUT* dst, int lane) {
  for (int v0 = 0; v0 < nvec; v0 += 32) {
    const int v = v0 + lane;
    uint64_t field = 0;
    if (v < nvec) field = STAGED ? field_from_smem<BITS>(row + v * BITS) : symbols8_raw(gs, nb, k0 + v, BITS);
    const uint4 out = lookup8_seg<BITS>(lut, field);
    if (v < nvec) st_global_cs16(dst + 8 * v, out);
  }
}

template <typename MAXT, typename OUT>
__global__ void __launch_bounds__(kThreads, 4) cachegen_staged(const __grid_constant__ CgArgs a, int stage_bytes,
                                                          const uint8_t* buf_end) {
  __shared__ float table[2][256];
  __shared__ float gmax[2][kCgGroupRows];
  __shared__ int64_t gblk[2][kCgGroupRows];
  __shared__ __align__(8) uint64_t bars[2];
  extern __shared__ __align__(128) uint8_t cg_stage[];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t gpk = (a.tokens + kCgGroupRows - 1) / kCgGroupRows;  // groups per stream
  const int64_t groups = 2 * gpk;
  const int64_t step = gridDim.x;
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  dependent_launch_entry();
  cg_table(table, a.bins);  // (ends with a barrier: the mbarriers are initialised for all)
  int64_t g = blockIdx.x;
  if (g >= groups) return;

  // Issue group gg into stage s: thread 0 starts the bulk copy (or arrives without bytes
  // when the group takes the global path); threads below kCgGroupRows fetch their row's
  // max and block id into registers. Returns the group's byte offset into the stage (-1:
  // global path).
  float pm = 0.f;
  int64_t pb = 0;
  auto issue = [&](int64_t gg, int s) -> int {
    const int kv = gg >= gpk ? 1 : 0;
    const int64_t r0 = (gg - kv * gpk) * kCgGroupRows;
    const int64_t r1 = min64(r0 + kCgGroupRows, a.tokens);
    const int64_t rb = static_cast<int64_t>(a.nvec) * a.bits[kv];  // bytes of a row
    const uintptr_t first = reinterpret_cast<uintptr_t>(a.stream[kv]) + static_cast<uintptr_t>(r0 * rb);
    const uintptr_t end = reinterpret_cast<uintptr_t>(a.stream[kv]) + static_cast<uintptr_t>(r1 * rb);
    const uintptr_t lo = first & ~static_cast<uintptr_t>(15);
    const uintptr_t hi = (end + 15) & ~static_cast<uintptr_t>(15);
    const bool fast = r1 * rb <= a.stream_bytes[kv] && hi <= reinterpret_cast<uintptr_t>(buf_end);
    if (tid == 0) {
      if (fast) {
        mbar_expect_tx(&bars[s], static_cast<uint32_t>(hi - lo));
        bulk_load(cg_stage + s * stage_bytes, reinterpret_cast<const void*>(lo), static_cast<uint32_t>(hi - lo),
                  &bars[s]);
      } else {
        mbar_arrive(&bars[s]);
      }
    }
    if (tid < kCgGroupRows) {
      const int64_t t = r0 + tid;
      if (t < a.tokens) {
        pm = to_f32(static_cast<const MAXT*>(a.maxv[kv])[t]);
        pb = a.ids[static_cast<int32_t>(t) / static_cast<int32_t>(a.block_size)];
      }
    }
    return fast ? static_cast<int>(first - lo) : -1;
  };

  int off_cur = issue(g, 0);
  if (tid < kCgGroupRows) {
    gmax[0][tid] = pm;
    gblk[0][tid] = pb;
  }
  uint32_t phases = 0;
  for (int j = 0;; ++j, g += step) {
    const int s = j & 1;
    const bool has_next = g + step < groups;
    __syncthreads();  // stage s ^ 1 and its max / block ids are free; stage s's are written
    const int off_next = has_next ? issue(g + step, s ^ 1) : -1;
    if (stage_wait_or_bail(&bars[s], (phases >> s) & 1u, &bars[s ^ 1], (phases >> (s ^ 1)) & 1u, has_next, a.err))
      return;
    phases ^= 1u << s;

    const int kv = g >= gpk ? 1 : 0;
#pragma unroll 1
    for (int k = 0; k < kCgRowsPerWarp; ++k) {
      const int rr = warp + k * (kThreads / 32);  // row of the group
      const int64_t t = (g - kv * gpk) * kCgGroupRows + rr;
      if (t >= a.tokens) break;
      const int bits = a.bits[kv];
      const int64_t blk = gblk[s][rr];
      if (blk < 0 || blk >= a.num_blocks) {  // counted per (kv, token, head) row
        if (lane == 0 && a.err) atomicAdd(a.err, static_cast<uint32_t>(a.heads));
      } else {
        const int64_t bi = static_cast<int32_t>(t) / static_cast<int32_t>(a.block_size);
        OUT* dst = reinterpret_cast<OUT*>(a.cache) + kv * a.kv_stride + blk * a.block_stride +
                   (t - bi * a.block_size) * a.token_stride;
        // lane l: the element for symbol value l mod 2^bits (segmented shuffles)
        const uint32_t lut = out_bits<OUT>(table[kv][lane & ((1 << bits) - 1)] * gmax[s][rr]);
        const uint8_t* row = off_cur >= 0 ? cg_stage + s * stage_bytes + off_cur + rr * a.nvec * bits : nullptr;
        const uint8_t* gs = a.stream[kv];
        const int64_t nb = a.stream_bytes[kv];
        const int64_t k0 = t * a.nvec;
#define ORIGAMI_CG_ROW(ST)                                                          \
  switch (bits) { /* warp-uniform */                                                \
    case 5: cg_row_seg<5, ST, OUT>(row, gs, nb, k0, a.nvec, lut, dst, lane); break;   \
    case 4: cg_row_seg<4, ST, OUT>(row, gs, nb, k0, a.nvec, lut, dst, lane); break;   \
    case 3: cg_row_seg<3, ST, OUT>(row, gs, nb, k0, a.nvec, lut, dst, lane); break;   \
    case 2: cg_row_seg<2, ST, OUT>(row, gs, nb, k0, a.nvec, lut, dst, lane); break;   \
    default: cg_row_seg<1, ST, OUT>(row, gs, nb, k0, a.nvec, lut, dst, lane); break;  \
  }
        if (row) {
          ORIGAMI_CG_ROW(true)
        } else {
          ORIGAMI_CG_ROW(false)
        }
#undef ORIGAMI_CG_ROW
      }
    }
    if (!has_next) break;
    if (tid < kCgGroupRows) {
      gmax[s ^ 1][tid] = pm;
      gblk[s ^ 1][tid] = pb;
    }
    off_cur = off_next;
  }
}

// ---------------------------------------------------------------------------------------
// CacheGen -> [layers, 2, heads, tokens, head_dim] fp16 (no cache)
// ---------------------------------------------------------------------------------------
struct CgUnpackArgs {
  const uint8_t* bytestream;
  int64_t bytestream_bytes;
  const int64_t* offsets;  // [2 * layers + 1], device
  const int64_t* bits;     // [2 * layers], device
  const int64_t* key_bins;
  const int64_t* value_bins;
  const void* max_key;  // [layers * tokens]
  const void* max_value;
  __half* out;
  int64_t layers, tokens, heads, head_dim;
};

// grid.y = stream (kv * layers + layer); a warp per (token, head) row of that stream.
template <typename MAXT, bool VEC>
__global__ void __launch_bounds__(kThreads) cachegen_unpack(const __grid_constant__ CgUnpackArgs a) {
  __shared__ float table[256];
  const int64_t sidx = blockIdx.y;
  const int kv = sidx >= a.layers ? 1 : 0;
  const int64_t layer = sidx - kv * a.layers;
  {
    const int64_t bins = kv ? a.value_bins[layer] : a.key_bins[layer];
    const float center = static_cast<float>(bins / 2 - 1);
    for (int i = threadIdx.x; i < 256; i += blockDim.x) table[i] = (static_cast<float>(i) - center) / center;
    __syncthreads();
  }
  const uint8_t* s = a.bytestream + a.offsets[sidx];
  const int bits = static_cast<int>(a.bits[sidx]);
  // 8-bit symbols are read up to the bytestream end, as the reference's unchecked
  // src[index] does (bitpack_layout_cuda.cu:74-76); narrower ones up to the stream length
  const int64_t nb = bits == 8 ? a.bytestream_bytes - a.offsets[sidx] : a.offsets[sidx + 1] - a.offsets[sidx];
  const MAXT* mx = static_cast<const MAXT*>(kv ? a.max_value : a.max_key) + layer * a.tokens;
  const int lane = threadIdx.x & 31;
  const int64_t C = a.heads * a.head_dim;
  const int64_t rows = a.tokens * a.heads;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
  for (int64_t row = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); row < rows; row += warps) {
    const int64_t t = row / a.heads;
    const int64_t h = row - t * a.heads;
    const float m = to_f32(mx[t]);
    __half* dst = a.out + (((layer * 2 + kv) * a.heads + h) * a.tokens + t) * a.head_dim;
    if constexpr (VEC) {
      const int64_t k0 = (t * C + h * a.head_dim) >> 3;
      const int nvec = static_cast<int>(a.head_dim / 8);
      if (bits <= 5) {
        const uint32_t lut = out_bits<__half>(table[lane] * m);
        for (int v0 = 0; v0 < nvec; v0 += 32) {
          const int v = v0 + lane;
          const uint64_t field = v < nvec ? symbols8_raw(s, nb, k0 + v, bits) : 0;
          const uint4 out = lookup8_shfl(lut, field, bits);
          if (v < nvec) st_global_cs16(dst + 8 * v, out);
        }
      } else {
        for (int v = lane; v < nvec; v += 32)
          st_global_cs16(dst + 8 * v, dequant8<__half>(table, m, symbols8_raw(s, nb, k0 + v, bits), bits));
      }
    } else {
      for (int64_t d = lane; d < a.head_dim; d += 32) {
        const uint32_t sym = symbol_at(s, nb, t * C + h * a.head_dim + d, bits);
        reinterpret_cast<uint16_t*>(dst)[d] = static_cast<uint16_t>(out_bits<__half>(table[sym] * m));
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// KIVI -> paged cache
// ---------------------------------------------------------------------------------------
struct KiviArgs {
  const uint8_t* stream[2];  // key, value
  int64_t stream_bytes[2];
  const void* scale[2];  // key: [key_groups, C]; value: [body_tokens, value_groups]
  const void* zero[2];
  const void* sink[2];  // [sink_tokens, C]
  uint8_t* cache;
  const int64_t* ids;
  int64_t kv_stride, block_stride, token_stride, head_stride;  // elements
  int64_t num_blocks, block_size, tokens, num_ids;
  int64_t sink_tokens, body_tokens, group_size, value_groups;
  int32_t bits, H, D;
  int32_t group_shift, block_shift;  // log2 of group_size / block_size; -1: not a power of two
  int32_t tiles_per_head, num_tiles;
  uint32_t* err;
};

// Dequantized element (kv, token t, channel ch = h * D + d) for a body token; symbol s.
template <typename META>
__device__ __forceinline__ float kivi_body(const KiviArgs& a, int kv, int64_t bt, int64_t ch, uint32_t s) {
  int64_t idx;
  if (kv) idx = bt * a.value_groups + ch / a.group_size;
  else idx = (bt / a.group_size) * (static_cast<int64_t>(a.H) * a.D) + ch;
  return __fmaf_rn(static_cast<float>(s), to_f32(static_cast<const META*>(a.scale[kv])[idx]),
                   to_f32(static_cast<const META*>(a.zero[kv])[idx]));
}

template <typename META>
__device__ __forceinline__ float kivi_sink(const KiviArgs& a, int kv, int64_t t, int64_t ch) {
  return to_f32(static_cast<const META*>(a.sink[kv])[t * (static_cast<int64_t>(a.H) * a.D) + ch]);
}

// Stream index of (kv, head h, channel d, body token bt).
__device__ __forceinline__ int64_t kivi_index(const KiviArgs& a, int kv, int64_t h, int64_t d, int64_t bt) {
  const int64_t chan = kv ? h * a.D + d : d * a.H + h;
  return chan * a.body_tokens + bt;
}

// One element per thread (any head_dim, sink count and group size).
template <typename META, typename OUT>
__global__ void __launch_bounds__(kThreads) kivi_to_cache_elem(const __grid_constant__ KiviArgs a) {
  const int64_t C = static_cast<int64_t>(a.H) * a.D;
  const int64_t total = 2 * a.tokens * C;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int kv = i >= a.tokens * C ? 1 : 0;
    const int64_t r = i - kv * a.tokens * C;
    const int64_t t = r / C;
    const int64_t ch = r - t * C;
    const int64_t bi = t / a.block_size;
    const int64_t blk = a.ids[bi];
    if (blk < 0 || blk >= a.num_blocks) {  // counted per (kv, token, head) row
      if (ch % a.D == 0 && a.err) atomicAdd(a.err, 1u);
      continue;
    }
    float v;
    if (t < a.sink_tokens) {
      v = kivi_sink<META>(a, kv, t, ch);
    } else {
      const int64_t bt = t - a.sink_tokens;
      const int64_t h = ch / a.D;
      const uint32_t s = symbol_at(a.stream[kv], a.stream_bytes[kv], kivi_index(a, kv, h, ch - h * a.D, bt), a.bits);
      v = kivi_body<META>(a, kv, bt, ch, s);
    }
    reinterpret_cast<uint16_t*>(a.cache)[kv * a.kv_stride + blk * a.block_stride +
                                          (t - bi * a.block_size) * a.token_stride + ch] =
        static_cast<uint16_t>(out_bits<OUT>(v));
  }
}

// Tile kernel: CTA = (kv, head, TT tokens) x all D channels, 256 threads as A token octets
// x O channel octets (O = D / 8 divides 256, TT = 8 * A). Needs sink_tokens % 8 == 0 so a
// token octet is all sink or all body. UNI (group_size % 8 == 0): the value group of a
// channel octet and the key group of a token octet are single groups.
// Eight META values as one 16-byte-aligned vector access.
// The four finished elements fma(s, scale, zero) for s = 0..3 as a table of two words
// (entry s in bytes 2s, 2s + 1), so that symbols of at most 2 bits dequantize with one
// byte permute instead of an int -> float and a float -> 16-bit conversion each.
template <typename OUT>
__device__ __forceinline__ uint2 lut4(float scale, float zero) {
  return make_uint2(pack2<OUT>(__fmaf_rn(0.f, scale, zero), __fmaf_rn(1.f, scale, zero)),
                    pack2<OUT>(__fmaf_rn(2.f, scale, zero), __fmaf_rn(3.f, scale, zero)));
}
// Two elements from one table: `pair` holds symbol s0 in byte 0 and s1 in byte 1.
__device__ __forceinline__ uint32_t lut4_pair(uint2 t, uint32_t pair) {
  return __byte_perm(t.x, t.y, 0x1010u + 0x22u * pair);
}
// One element (low 16 bits) from a table.
__device__ __forceinline__ uint32_t lut4_one(uint2 t, uint32_t s) { return __byte_perm(t.x, t.y, 0x10u + 0x22u * s); }

template <typename META>
struct alignas(16) VecOf {
  META v[8];
};

// Shared memory: [runs: D rows x rs][bit0: D x int32][rowoff: TT x int64][token rows]
// [scale, zero: kMetaSlots x max(TT, D) META each]. The staged-run row holds up to TT
// bytes (8-bit symbols) plus word slack; its stride is not a multiple of 128 bytes at
// eight rows, so the two channel octets of a warp read different banks.
constexpr int kMetaSlots = 4;

template <int D, typename META>
struct KiviGeo {
  static constexpr int O = D / 8;
  static constexpr int A = kThreads / O;
  static constexpr int TT = 8 * A;
  static constexpr int rs = TT + 24;
  static constexpr int runs_bytes = D * rs;
  static constexpr int rows_off = runs_bytes + D * 4 + TT * 8;
  static constexpr int rows_bytes = TT * D * 2;
  static constexpr int meta_off = rows_off + rows_bytes;
  static constexpr int meta_elems = kMetaSlots * (TT > D ? TT : D);
  static constexpr int smem_bytes = meta_off + 2 * meta_elems * static_cast<int>(sizeof(META));
};

template <typename META, typename OUT, int D, bool UNI>
__global__ void __launch_bounds__(kThreads) kivi_to_cache(const __grid_constant__ KiviArgs a) {
  using G = KiviGeo<D, META>;
  extern __shared__ __align__(16) uint8_t kivi_smem[];
  uint8_t* runs = kivi_smem;
  int32_t* bit0 = reinterpret_cast<int32_t*>(kivi_smem + G::runs_bytes);
  int64_t* rowoff = reinterpret_cast<int64_t*>(kivi_smem + G::runs_bytes + D * 4);
  uint8_t* rows_sm = kivi_smem + G::rows_off;
  META* msc = reinterpret_cast<META*>(kivi_smem + G::meta_off);
  META* mze = msc + G::meta_elems;
  const int tid = threadIdx.x;
  const int bits = a.bits;
  const int64_t C = static_cast<int64_t>(a.H) * D;
  dependent_launch_entry();

  for (int tile = blockIdx.x; tile < a.num_tiles; tile += gridDim.x) {
    const int tt = tile % a.tiles_per_head;
    const int rest = tile / a.tiles_per_head;
    const int h = rest % a.H;
    const int kv = rest / a.H;
    const int64_t t0 = static_cast<int64_t>(tt) * G::TT;
    const int64_t tb0 = max64(t0, a.sink_tokens);
    const int64_t tb1 = min64(t0 + G::TT, a.tokens);
    const int nbody = static_cast<int>(max64(tb1 - tb0, 0));

    // row offsets through the block table
    for (int r = tid; r < G::TT; r += kThreads) {
      const int64_t t = t0 + r;
      int64_t off = -1;
      if (t < a.tokens) {
        const int64_t bi = static_cast<uint32_t>(t) / static_cast<uint32_t>(a.block_size);  // both below 2^31
        const int64_t blk = a.ids[bi];
        if (blk < 0 || blk >= a.num_blocks) {
          if (a.err) atomicAdd(a.err, 1u);
        } else {
          off = kv * a.kv_stride + blk * a.block_stride + (t - bi * a.block_size) * a.token_stride +
                static_cast<int64_t>(h) * a.head_stride;
        }
      }
      rowoff[r] = off;
    }
    // stage the body run of every channel; bytes at or past the stream end read as zero
    if (nbody > 0) {
      // 4-byte words from the aligned word holding the run's first byte
      const uint8_t* s = a.stream[kv];
      const uintptr_t end = reinterpret_cast<uintptr_t>(s) + static_cast<uintptr_t>(a.stream_bytes[kv]);
      const int words = ((nbody * bits + 7) >> 3) / 4 + 2;
      // word i = d * words + w of the staged runs, walked without division: consecutive
      // dims' runs are dstep bits apart (key runs: H * body symbols; value runs: body)
      const int64_t dstep = static_cast<int64_t>(kv ? 1 : a.H) * a.body_tokens * bits;
      const int qd = kThreads / words, rw = kThreads % words;
      int d = tid / words, w = tid - (tid / words) * words;
      int64_t bitpos = kivi_index(a, kv, h, d, tb0 - a.sink_tokens) * bits;
      for (int i = tid; i < D * words; i += kThreads) {
        const uintptr_t first = reinterpret_cast<uintptr_t>(s) + static_cast<uintptr_t>(bitpos >> 3);
        const uintptr_t wa = (first & ~static_cast<uintptr_t>(3)) + 4u * static_cast<uintptr_t>(w);
        uint32_t v = 0;
        if (wa < end) {
          v = __ldg(reinterpret_cast<const uint32_t*>(wa));
          if (wa + 4 > end) v &= (1u << (8 * static_cast<int>(end - wa))) - 1u;
        }
        reinterpret_cast<uint32_t*>(runs + d * G::rs)[w] = v;
        if (w == 0) bit0[d] = static_cast<int32_t>((first & 3u) * 8u + static_cast<uintptr_t>(bitpos & 7));
        w += rw;
        d += qd;
        bitpos += qd * dstep;
        if (w >= words) {
          w -= words;
          d += 1;
          bitpos += dstep;
        }
      }
    }
    // UNI: this tile's scale / zero, coalesced into shared memory when they fit in
    // kMetaSlots value groups (one token's slots per row) or key groups (one group's D
    // channels per row); otherwise phase B reads them from global memory.
    bool staged = false;
    int mbase = 0;  // first staged value group / key group
    if constexpr (UNI) {
      if (nbody > 0) {
        const META* sc = static_cast<const META*>(a.scale[kv]);
        const META* ze = static_cast<const META*>(a.zero[kv]);
        if (kv) {
          // (channel and token counts are below 2^31, checked on the host: 32-bit divisions)
          mbase = h * D / static_cast<int>(a.group_size);
          const int ng = static_cast<int>((h * D + D - 1) / static_cast<int>(a.group_size) - mbase + 1);
          if (ng <= kMetaSlots) {
            staged = true;
            // [group][token]: a thread's eight tokens of one group are one vector
            for (int i = tid; i < nbody * ng; i += kThreads) {
              const int r = i / ng;
              const int g = i - r * ng;
              const int64_t idx = (tb0 - a.sink_tokens + r) * a.value_groups + mbase + g;
              msc[g * G::TT + r] = sc[idx];
              mze[g * G::TT + r] = ze[idx];
            }
          }
        } else {
          mbase = static_cast<int>(tb0 - a.sink_tokens) / static_cast<int>(a.group_size);
          const int nkg = static_cast<int>(tb1 - 1 - a.sink_tokens) / static_cast<int>(a.group_size) - mbase + 1;
          if (nkg <= kMetaSlots) {
            staged = true;
            for (int i = tid; i < nkg * D; i += kThreads) {
              const int r = i / D;
              const int d = i - r * D;
              const int64_t idx = (mbase + r) * C + static_cast<int64_t>(h) * D + d;
              msc[r * D + d] = sc[idx];
              mze[r * D + d] = ze[idx];
            }
          }
        }
      }
    }
    __syncthreads();

    const int ao = tid % G::A;
    const int o = tid / G::A;
    const int64_t tq = t0 + 8 * ao;  // first token of this thread's octet
    uint32_t outw[8][4];
    if (tq < a.tokens) {
      if (tq < a.sink_tokens) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int64_t t = min64(tq + i, a.tokens - 1);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int64_t ch = static_cast<int64_t>(h) * D + 8 * o + 2 * j;
            outw[i][j] = out_bits<OUT>(kivi_sink<META>(a, kv, t, ch)) |
                         (out_bits<OUT>(kivi_sink<META>(a, kv, t, ch + 1)) << 16);
          }
        }
      } else {
        // 8 tokens x 8 channels of symbols: windows per channel, 8x8 byte transpose
        uint32_t lo[8], hi[8];
        const int k0 = static_cast<int>(tq - tb0);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int d = 8 * o + j;
          uint32_t v0, v1;
          window64(runs + d * G::rs, bit0[d] + k0 * bits, v0, v1);
          spread8_rt(v0, v1, bits, lo[j], hi[j]);
        }
        transpose8x8(lo, hi);  // lo[i] / hi[i]: channels 0..3 / 4..7 of token i
        const int64_t bq = tq - a.sink_tokens;
        const int64_t ch0 = static_cast<int64_t>(h) * D + 8 * o;
        if constexpr (UNI) {
          const META* sc = static_cast<const META*>(a.scale[kv]);
          const META* ze = static_cast<const META*>(a.zero[kv]);
          if (kv) {
            const int g = static_cast<int>(ch0) / static_cast<int>(a.group_size);
            META vs[8], vz[8];
            if (staged) {  // tokens k0 .. k0 + 7 of group g (k0 % 8 == 0): one vector each
              const int base = (g - mbase) * G::TT + k0;
              *reinterpret_cast<VecOf<META>*>(vs) = *reinterpret_cast<const VecOf<META>*>(msc + base);
              *reinterpret_cast<VecOf<META>*>(vz) = *reinterpret_cast<const VecOf<META>*>(mze + base);
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int64_t idx = min64(bq + i, a.body_tokens - 1) * a.value_groups + g;
                vs[i] = sc[idx];
                vz[i] = ze[idx];
              }
            }
            if (bits <= 2) {
              // one (scale, zero) per token row: a table per row, two channels per permute
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const uint2 t = lut4<OUT>(to_f32(vs[i]), to_f32(vz[i]));
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint32_t w = j < 2 ? lo[i] : hi[i];
                  outw[i][j] = lut4_pair(t, (w >> ((j & 1) * 16)) & 0x0303u);
                }
              }
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float fs = to_f32(vs[i]);
                const float fz = to_f32(vz[i]);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint32_t w = j < 2 ? lo[i] : hi[i];
                  const int sh = (j & 1) * 16;
                  outw[i][j] = out_bits<OUT>(__fmaf_rn(static_cast<float>((w >> sh) & 0xFF), fs, fz)) |
                               (out_bits<OUT>(__fmaf_rn(static_cast<float>((w >> (sh + 8)) & 0xFF), fs, fz)) << 16);
                }
              }
            }
          } else {
            float fs[8], fz[8];
            if (staged) {
              const int base = (static_cast<int>(bq) / static_cast<int>(a.group_size) - mbase) * D + 8 * o;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                fs[j] = to_f32(msc[base + j]);
                fz[j] = to_f32(mze[base + j]);
              }
            } else {
              const int64_t base = (bq / a.group_size) * C + ch0;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                fs[j] = to_f32(sc[base + j]);
                fz[j] = to_f32(ze[base + j]);
              }
            }
            if (bits <= 2) {
              // one (scale, zero) per channel: a table per channel, one permute per element
              uint2 t[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) t[j] = lut4<OUT>(fs[j], fz[j]);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint32_t w = (j < 2 ? lo[i] : hi[i]) >> ((j & 1) * 16);
                  outw[i][j] = __byte_perm(lut4_one(t[2 * j], w & 0x03u), lut4_one(t[2 * j + 1], (w >> 8) & 0x03u),
                                           0x5410);
                }
              }
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint32_t w = j < 2 ? lo[i] : hi[i];
                  const int sh = (j & 1) * 16;
                  const int c = 2 * j;
                  outw[i][j] =
                      out_bits<OUT>(__fmaf_rn(static_cast<float>((w >> sh) & 0xFF), fs[c], fz[c])) |
                      (out_bits<OUT>(__fmaf_rn(static_cast<float>((w >> (sh + 8)) & 0xFF), fs[c + 1], fz[c + 1]))
                       << 16);
                }
              }
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int64_t bt = min64(bq + i, a.body_tokens - 1);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t w = j < 2 ? lo[i] : hi[i];
              const int sh = (j & 1) * 16;
              const int64_t ch = ch0 + 2 * j;
              outw[i][j] = out_bits<OUT>(kivi_body<META>(a, kv, bt, ch, (w >> sh) & 0xFF)) |
                           (out_bits<OUT>(kivi_body<META>(a, kv, bt, ch + 1, (w >> (sh + 8)) & 0xFF)) << 16);
            }
          }
        }
      }
      const int phys = (o + ao) & (G::O - 1);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        *reinterpret_cast<uint4*>(rows_sm + (8 * ao + i) * (D * 2) + phys * 16) =
            make_uint4(outw[i][0], outw[i][1], outw[i][2], outw[i][3]);
    }
    __syncthreads();
    const int oc = tid % G::O;
    for (int r = tid / G::O; r < G::TT; r += kThreads / G::O) {
      const int64_t off = rowoff[r];
      if (off < 0) continue;
      st_global_cs16(reinterpret_cast<uint16_t*>(a.cache) + off + 8 * oc,
                     *reinterpret_cast<const uint4*>(rows_sm + r * (D * 2) + ((oc + (r >> 3)) & (G::O - 1)) * 16));
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------
// 2-bit KIVI (the reference's default width) -> paged cache
//
// Same tiles and thread mapping as kivi_to_cache (CTA = (kv, head, TT tokens) x D
// channels, a thread = 8 tokens x 8 channels), without a transpose: a thread's channel
// runs are read as 16-bit fields (8 tokens x 2 bits), two channels are interleaved into one
// word by a byte permute, and each output word (two channels of one token) is a byte
// permute of a 4-entry table fma(s, scale, zero), s = 0..3, whose selector is built for two
// tokens at once by one multiply-add. Runs are staged by 16-byte cp.async chunks; finished
// token rows leave shared memory as whole-row bulk copies (one per row, issued by the
// thread that owns the row), drained only before the next tile's rows are written.
//
// Tiles run head-fastest (tile = h + H * (tt + tiles_per_head * kv)): the CTAs in flight
// write all heads of the same token rows (whole cache rows, DRAM-page friendly) and read
// consecutive stretches of every channel run. Group and block sizes are powers of two
// (shifts); token counts are below 2^31.
// ---------------------------------------------------------------------------------------
template <int D, typename META>
struct Kivi2Geo {
  static constexpr int O = D / 8;
  static constexpr int A = kThreads / O;
  static constexpr int TT = 8 * A;  // at most kThreads: thread r owns token row r
  // a run of TT symbols is TT / 4 bytes, staged from the 16-byte chunk holding its first
  // byte, with one chunk of slack for the 64-bit window at its end
  static constexpr int chunks = (TT / 4 + 16) / 16 + 1;
  static constexpr int rs = 16 * chunks;
  static constexpr int row_bytes = D * 2;
  // token rows with 16 bytes of padding after every 8 rows: the 8 rows a thread writes
  // land in different banks for the threads of a quarter warp, and every row stays
  // 16-byte aligned for its bulk copy
  static constexpr int rows_bytes = TT * row_bytes + (TT / 8) * 16;
  static constexpr int runs_off = rows_bytes;
  static constexpr int bit0_off = runs_off + D * rs;
  static constexpr int lut_off = bit0_off + D * 4;
  // finished 4-entry tables fma(s, scale, zero), s = 0..3, of up to kSlots groups: values
  // as [group slot][token % 8][token / 8] (the threads of a token octet read consecutive
  // entries), keys as [group slot][channel]
  static constexpr int kSlots = 3;
  static constexpr int lut_entries = kSlots * (TT > D ? TT : D);
  static constexpr int smem_bytes = lut_off + lut_entries * 8;
  // 5 CTAs an SM where their shared memory fits (1 KB reserved per CTA of 228 KB), else 4
  static constexpr int min_ctas = 5 * (smem_bytes + 1024) <= 228 * 1024 ? 5 : 4;
  static_assert(TT <= kThreads, "one token row per thread");
};

// Permute selectors of tokens k (bits 0-15) and k + 4 (bits 16-31) from a word holding
// channel A's and channel B's symbols as bytes [A 0-3, B 0-3, A 4-7, B 4-7]: byte j of the
// masked word is a symbol s, and 0x22 * s + 0x10 is the selector nibble pair (2s, 2s + 1).
__device__ __forceinline__ uint32_t kivi2_selectors(uint32_t w2, int k) {
  return ((w2 >> (2 * k)) & 0x03030303u) * 0x22u + 0x10101010u;
}

template <typename META, typename OUT, int D>
__global__ void __launch_bounds__(kThreads, Kivi2Geo<D, META>::min_ctas) kivi2_to_cache(const __grid_constant__ KiviArgs a) {
  using G = Kivi2Geo<D, META>;
  extern __shared__ __align__(128) uint8_t kivi2_smem[];
  uint8_t* rows_sm = kivi2_smem;
  uint8_t* runs = kivi2_smem + G::runs_off;
  int32_t* bit0 = reinterpret_cast<int32_t*>(kivi2_smem + G::bit0_off);
  uint2* lut = reinterpret_cast<uint2*>(kivi2_smem + G::lut_off);
  const int tid = threadIdx.x;
  const int64_t C = static_cast<int64_t>(a.H) * D;
  const int ao = tid % G::A;
  const int o = tid / G::A;
  const int gs = a.group_shift;
  const int sink = static_cast<int>(a.sink_tokens);
  const int tokens = static_cast<int>(a.tokens);
  dependent_launch_entry();

  // tile = h + H * r, r = tt + tiles_per_head * kv; advanced by gridDim.x without divisions
  const int tph = a.tiles_per_head;
  const int step_h = static_cast<int>(gridDim.x) % a.H;
  const int step_r = static_cast<int>(gridDim.x) / a.H;
  int h = static_cast<int>(blockIdx.x) % a.H;
  int r = static_cast<int>(blockIdx.x) / a.H;
  for (int tile = blockIdx.x; tile < a.num_tiles; tile += gridDim.x) {
    const int kv = r >= tph ? 1 : 0;
    const int t0 = (r - kv * tph) * G::TT;
    const int tb0 = max(t0, sink);
    const int tb1 = min(t0 + G::TT, tokens);
    const int nbody = max(tb1 - tb0, 0);

    // this thread's cache row: token t0 + tid, through the block table (-1: not written)
    int64_t off = -1;
    if (tid < G::TT) {
      const int t = t0 + tid;
      if (t < tokens) {
        const int bi = a.block_shift >= 0 ? t >> a.block_shift : t / static_cast<int>(a.block_size);
        const int64_t blk = a.ids[bi];
        if (blk < 0 || blk >= a.num_blocks) {
          if (a.err) atomicAdd(a.err, 1u);
        } else {
          off = kv * a.kv_stride + blk * a.block_stride +
                static_cast<int64_t>(t - bi * static_cast<int>(a.block_size)) * a.token_stride +
                static_cast<int64_t>(h) * a.head_stride;
        }
      }
    }
    // stage the body run of every channel as 16-byte chunks from the chunk holding its
    // first byte (aligned in absolute address, so a chunk that starts before the stream
    // shares a 16-byte line with the run's first byte; bytes at or past the stream end read
    // as zero through the cp.async source size)
    if (nbody > 0) {
      const uintptr_t sbase = reinterpret_cast<uintptr_t>(a.stream[kv]);
      const uintptr_t end = sbase + static_cast<uintptr_t>(a.stream_bytes[kv]);
      const int64_t dstep = static_cast<int64_t>(kv ? 1 : a.H) * a.body_tokens * 2;  // bits between dims' runs
      const int64_t bit_d0 = kivi_index(a, kv, h, 0, tb0 - sink) * 2;
#pragma unroll
      for (int i = tid; i < D * G::chunks; i += kThreads) {
        const int d = i / G::chunks;
        const int c = i % G::chunks;
        const int64_t bitpos = bit_d0 + d * dstep;
        const uintptr_t first = sbase + static_cast<uintptr_t>(bitpos >> 3);
        const uintptr_t line = first & ~static_cast<uintptr_t>(15);
        const uintptr_t chunk = line + 16u * static_cast<uintptr_t>(c);
        const uint32_t nbytes = chunk + 16 <= end ? 16u : (chunk < end ? static_cast<uint32_t>(end - chunk) : 0u);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(runs + d * G::rs + 16 * c)),
                     "l"(nbytes ? chunk : line), "r"(nbytes)
                     : "memory");
        if (c == 0) bit0[d] = static_cast<int32_t>((first & 15u) * 8u + static_cast<uintptr_t>(bitpos & 7));
      }
      asm volatile("cp.async.commit_group;\n" ::: "memory");
    }
    // this tile's tables in shared memory when they fit in kSlots value groups or key
    // groups (each thread loads one (scale, zero) pair and writes its finished table);
    // otherwise the dequantization builds them from global memory
    bool staged = false;
    int mbase = 0;  // first staged value group / key group
    if (nbody > 0) {
      const META* sc = static_cast<const META*>(a.scale[kv]);
      const META* ze = static_cast<const META*>(a.zero[kv]);
      if (kv) {
        mbase = (h * D) >> gs;
        const int ng = ((h * D + D - 1) >> gs) - mbase + 1;
        if (ng <= G::kSlots) {
          staged = true;
          for (int e = tid; e < ng * G::TT; e += kThreads) {
            const int g = e / G::TT;
            const int rr = e % G::TT;
            if (rr < nbody) {
              const int64_t idx = static_cast<int64_t>(tb0 - sink + rr) * a.value_groups + mbase + g;
              lut[(g * 8 + (rr & 7)) * G::A + (rr >> 3)] = lut4<OUT>(to_f32(sc[idx]), to_f32(ze[idx]));
            }
          }
        }
      } else {
        mbase = (tb0 - sink) >> gs;
        const int nkg = ((tb1 - 1 - sink) >> gs) - mbase + 1;
        if (nkg <= G::kSlots) {
          staged = true;
          for (int e = tid; e < nkg * D; e += kThreads) {
            const int64_t idx = static_cast<int64_t>(mbase + e / D) * C + h * D + (e % D);
            lut[e] = lut4<OUT>(to_f32(sc[idx]), to_f32(ze[idx]));
          }
        }
      }
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    }
    // the previous tile's rows have been read out of shared memory by their bulk copies
    if (tid < G::TT) asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
    __syncthreads();

    const int tq = t0 + 8 * ao;  // first token of this thread's octet
    if (tq < tokens) {
      uint32_t outw[8][4];
      const int ch0 = h * D + 8 * o;
      if (tq < sink) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int t = min(tq + i, tokens - 1);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            outw[i][j] = pack2<OUT>(kivi_sink<META>(a, kv, t, ch0 + 2 * j), kivi_sink<META>(a, kv, t, ch0 + 2 * j + 1));
        }
      } else {
        // w2[c]: channels 8o + 2c (A) and 8o + 2c + 1 (B) as bytes [A 0-3, B 0-3, A 4-7, B 4-7]
        // of tokens tq .. tq + 7, 2 bits each
        const int k0 = tq - tb0;
        uint32_t w2[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t f[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int d = 8 * o + 2 * c + e;
            const int pos = bit0[d] + 2 * k0;
            const uint32_t* row = reinterpret_cast<const uint32_t*>(runs + d * G::rs);
            f[e] = __funnelshift_r(row[pos >> 5], row[(pos >> 5) + 1], pos & 31);
          }
          w2[c] = __byte_perm(f[0], f[1], 0x5140u);
        }
        const int bq = tq - sink;
        const META* sc = static_cast<const META*>(a.scale[kv]);
        const META* ze = static_cast<const META*>(a.zero[kv]);
        if (kv) {
          // values: one (scale, zero) per token and channel group, one table per token
          const int g = ch0 >> gs;
          // body token k0 + i of group g (k0 % 8 == 0): octet k0 / 8, entry i
          const uint2* lp = lut + ((g - mbase) * 8) * G::A + (k0 >> 3);
          auto table = [&](int i) -> uint2 {
            if (staged) return lp[i * G::A];
            const int64_t idx =
                static_cast<int64_t>(min(bq + i, static_cast<int>(a.body_tokens) - 1)) * a.value_groups + g;
            return lut4<OUT>(to_f32(sc[idx]), to_f32(ze[idx]));
          };
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint2 tl = table(k);
            const uint2 th = table(k + 4);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t y = kivi2_selectors(w2[c], k);
              outw[k][c] = __byte_perm(tl.x, tl.y, y);
              outw[k + 4][c] = __byte_perm(th.x, th.y, y >> 16);
            }
          }
        } else {
          // keys: one (scale, zero) per channel and token group, one table per channel;
          // channel A's table gives the low half of a word, channel B's the high half
          uint2 t[8];
          if (staged) {
            const uint4* lp = reinterpret_cast<const uint4*>(lut + ((bq >> gs) - mbase) * D + 8 * o);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 v = lp[q];
              t[2 * q] = make_uint2(v.x, v.y);
              t[2 * q + 1] = make_uint2(v.z, v.w);
            }
          } else {
            const int64_t base = static_cast<int64_t>(bq >> gs) * C + ch0;
#pragma unroll
            for (int j = 0; j < 8; ++j) t[j] = lut4<OUT>(to_f32(sc[base + j]), to_f32(ze[base + j]));
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t y = kivi2_selectors(w2[c], k);
              const uint32_t yh = y >> 16;
              outw[k][c] = __byte_perm(__byte_perm(t[2 * c].x, t[2 * c].y, y),
                                       __byte_perm(t[2 * c + 1].x, t[2 * c + 1].y, y), 0x7610u);
              outw[k + 4][c] = __byte_perm(__byte_perm(t[2 * c].x, t[2 * c].y, yh),
                                           __byte_perm(t[2 * c + 1].x, t[2 * c + 1].y, yh), 0x7610u);
            }
          }
        }
      }
      uint8_t* dst = rows_sm + 8 * ao * G::row_bytes + 16 * (ao + o);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        *reinterpret_cast<uint4*>(dst + i * G::row_bytes) = make_uint4(outw[i][0], outw[i][1], outw[i][2], outw[i][3]);
    }
    // rows written by the generic proxy, read by the bulk copies
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    __syncthreads();
    if (tid < G::TT) {
      if (off >= 0)
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(a.cache + 2 * off),
                     "r"(smem_u32(rows_sm + tid * G::row_bytes + 16 * (tid >> 3))), "r"(G::row_bytes)
                     : "memory");
      asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
    }
    h += step_h;
    r += step_r;
    if (h >= a.H) {
      h -= a.H;
      ++r;
    }
  }
  // the last rows are in global memory before the CTA leaves
  if (tid < G::TT) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
}
}  // namespace origami
