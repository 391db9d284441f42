// Fused attention over a quantized prefix and a paged suffix (drop-in for the reference's
// origami_fused_prefix_attention_kernel, bitpack_layout_cuda.cu:873-1091).
//
// Semantics kept from the reference: query token q (of query_tokens, at absolute position
// query_start + q) attends to keys [0, min(sequence_length - 1, query_start + q)]; keys
// below prefix_tokens are dequantized from the KIVI (codec 0) or KVQuant (codec 1) symbol
// streams, the others are read from the paged cache through block_table (int32); an
// out-of-range block id reads as zero K and V (the key still takes part in the softmax
// with score 0). head_dim is 128; query head qh uses KV head qh / (query_heads / kv_heads).
//
// Design. One CTA (256 threads) owns one KV head, NQ query rows (row = query token x query
// head of the GQA group, heads fastest) and one contiguous range of 128-key tiles. The
// contraction runs on the tensor cores with the keys on the MMA's M dimension, so that a
// decode step's handful of query rows fills N (N >= 8) instead of wasting M:
//   S^T [128 keys x NQ] = K_tile [128 x 128 dims] . Q^T                 (tcgen05, TMEM)
//   O^T [128 dims x NQ] += V^T_tile [128 dims x 128 keys] . P^T           (tcgen05, TMEM)
// All 256 threads dequantize the K and V^T tiles (fp32 fma(s, scale, zero) as the
// reference, rounded to the query type) into shared memory in the canonical K-major
// SWIZZLE_NONE layout of the MMA; warps 0-3 (one TMEM lane = one key each) run the online
// softmax and write P; warps 4-7 (one TMEM lane = one dim each) rescale O. Long prefixes
// are split over CTAs; each split leaves (O, max, sum) in the caller's workspace and the
// last split of a row block to finish merges them (self-resetting arrival counter).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "common.cuh"

namespace origami {

namespace attn {

constexpr int kD = 128;            // head_dim
constexpr int kKT = 128;           // keys per tile
constexpr int kThreadsA = 256;
constexpr int kLBO = 144;          // bytes between adjacent 8-element K chunks of a core-matrix row group
constexpr int kSBO = 16 * kLBO + 16;  // bytes between 8-row groups of a [rows x 128] operand tile
constexpr int kTileBytes = 16 * kSBO;  // a [128 x 128] 16-bit operand tile
constexpr uint32_t kOCol = 64;     // TMEM column of O^T (S^T starts at column 0)
constexpr uint32_t kTmemCols = 128;

// Byte offset of element (row r, k) in a canonical [rows x 128] operand tile: 8 x 16-byte
// core matrices, K chunks kLBO apart, row groups kSBO apart. The 16-byte paddings (kLBO =
// 36 words, kSBO = 580 words, both 4 mod 32) make the 16-byte dequant stores of 8 threads
// that are 8 chunks or 8 row groups apart hit 8 different bank quads.
__device__ __forceinline__ uint32_t tile_off(int r, int k) {
  return static_cast<uint32_t>((r >> 3) * kSBO + (k >> 3) * kLBO + (r & 7) * 16 + (k & 7) * 2);
}

// Shared-memory matrix descriptor (tcgen05): start address, LBO, SBO in 16-byte units,
// descriptor version 1, base offset 0, SWIZZLE_NONE.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (static_cast<uint64_t>(addr >> 4) & 0x3FFFull) | (static_cast<uint64_t>(kLBO >> 4) << 16) |
         (static_cast<uint64_t>(kSBO >> 4) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::f16: fp32 accumulator, A and B of the query type (both
// F16 or both BF16), both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t instr_desc(bool bf16, int n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(128 >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  const uint32_t z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(z)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_ld8(uint32_t addr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st8(uint32_t addr, const float (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(addr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
               "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
               "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// 16-bit element conversions (QT = __half or __nv_bfloat16).
template <typename QT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float bits_to_float(uint16_t b, bool bf16) {
  return bf16 ? __uint_as_float(static_cast<uint32_t>(b) << 16) : __half2float(__ushort_as_half(b));
}
template <typename QT>
__device__ __forceinline__ uint16_t from_float(float v);
template <>
__device__ __forceinline__ uint16_t from_float<__half>(float v) {
  return __half_as_ushort(__float2half_rn(v));
}
template <>
__device__ __forceinline__ uint16_t from_float<__nv_bfloat16>(float v) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}
template <typename QT>
__host__ __device__ constexpr bool is_bf16() {
  return std::is_same<QT, __nv_bfloat16>::value;
}

// 8 x 8 transpose of 16-bit elements held as 8 rows of 4 words (element c of row r in
// word c / 2, half c % 2).
__device__ __forceinline__ void transpose8x8_u16(uint32_t (&m)[8][4]) {
#pragma unroll
  for (int r = 0; r < 8; r += 2) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t a = m[r][w], b = m[r + 1][w];
      m[r][w] = __byte_perm(a, b, 0x5410);
      m[r + 1][w] = __byte_perm(a, b, 0x7632);
    }
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    if ((r & 2) == 0) {
#pragma unroll
      for (int w = 0; w < 4; w += 2) {
        const uint32_t t = m[r][w + 1];
        m[r][w + 1] = m[r + 2][w];
        m[r + 2][w] = t;
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      const uint32_t t = m[r][w + 2];
      m[r][w + 2] = m[r + 4][w];
      m[r + 4][w] = t;
    }
  }
}

}  // namespace attn

struct AttnArgs {
  const uint8_t* stream[2];      // key / value symbol streams (bytestream + offset)
  const uint8_t* bytes_end;      // end of the bytestream: no load reaches past its 4-byte word
  const uint8_t* stream_end[2];  // ends of the key / value streams (stream + key_bytes / value_bytes)
  int32_t slot_bits, sym_mask;   // bits per symbol slot (4 for nibble-packed 3-bit) and value mask
  int64_t group_size, sink, prefix, body;  // body = tokens held in the symbol streams
  const __half* scale[2];        // KIVI: key [ceil(body/gs), C], value [body, ceil(C/gs)]; KVQuant: key [C], value [prefix]
  const __half* zero[2];
  const __half* sink_kv[2];      // KIVI sink tokens [sink, C]
  const uint16_t* query;         // [q_tokens, q_heads, 128]
  uint16_t* output;
  const uint16_t* cache;         // paged cache, elements of the cache type
  int64_t kv_stride, block_stride, token_stride;  // elements
  int64_t num_blocks, block_size;
  const int32_t* block_table;
  int64_t q_start, seq_len;
  int32_t q_tokens, q_heads, kv_heads, group, rows, row_blocks, splits;
  int32_t cache_bf16, cache_vec;  // cache element type; 16-byte aligned cache rows
  int32_t meta_vec;               // scale / zero tensors 16-byte aligned (8-channel vector loads)
  int32_t sym_len;                // bits per symbol value (3 for nibble-packed 3-bit)
  float scale_log2;               // softmax_scale * log2(e)
  float* ws_o;                    // [kv_heads * row_blocks * splits * NQ * 128] partial O
  float* ws_ml;                   // [kv_heads * row_blocks * splits * NQ * 2] partial max / sum
  uint32_t* counters;             // [kv_heads * row_blocks], zero between calls
  uint32_t* err;
};

namespace attn {

// 64 bits of a symbol stream from bit position `bit` (bytes past the bytestream read as 0).
__device__ __forceinline__ uint64_t bits64(const AttnArgs& a, const uint8_t* s, int64_t bit) {
  const uint8_t* p = s + (bit >> 3);
  const uintptr_t pa = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(pa & ~static_cast<uintptr_t>(3));
  const int sh = static_cast<int>((pa & 3) * 8 + (bit & 7));
  const uintptr_t end = (reinterpret_cast<uintptr_t>(a.bytes_end) + 3) & ~static_cast<uintptr_t>(3);
  uint32_t w0, w1, w2;
  if (reinterpret_cast<uintptr_t>(w + 3) <= end) {
    w0 = __ldg(w);
    w1 = __ldg(w + 1);
    w2 = __ldg(w + 2);
  } else {
    uint32_t v[3] = {0u, 0u, 0u};
    const uint8_t* b = reinterpret_cast<const uint8_t*>(w);
    for (int i = 0; i < 12; ++i)
      if (b + i < a.bytes_end) v[i >> 2] |= static_cast<uint32_t>(__ldg(b + i)) << ((i & 3) * 8);
    w0 = v[0];
    w1 = v[1];
    w2 = v[2];
  }
  const uint64_t lo = (static_cast<uint64_t>(w1) << 32) | w0;
  return sh == 0 ? lo : (lo >> sh) | (static_cast<uint64_t>(w2) << (64 - sh));
}

__device__ __forceinline__ float h2f(const __half* p, int64_t i) { return __half2float(__ldg(p + i)); }

// 32 or 64 stream bits from bit position `bit` as two words (bytes past the bytestream
// read as 0); `narrow` (8 symbols of at most 4 bits) loads two aligned words instead of three.
struct Win {
  uint32_t lo, hi;
};
__device__ __forceinline__ Win window(const AttnArgs& a, const uint8_t* s, int64_t bit, bool narrow) {
  const uintptr_t pa = reinterpret_cast<uintptr_t>(s + (bit >> 3));
  const uint32_t* w = reinterpret_cast<const uint32_t*>(pa & ~static_cast<uintptr_t>(3));
  const uint32_t sh = static_cast<uint32_t>((pa & 3) * 8 + (bit & 7));
  const uintptr_t end = (reinterpret_cast<uintptr_t>(a.bytes_end) + 3) & ~static_cast<uintptr_t>(3);
  uint32_t w0, w1, w2 = 0u;
  if (reinterpret_cast<uintptr_t>(w + 3) <= end) {
    w0 = __ldg(w);
    w1 = __ldg(w + 1);
    if (!narrow) w2 = __ldg(w + 2);
  } else {
    uint32_t v[3] = {0u, 0u, 0u};
    const uint8_t* b = reinterpret_cast<const uint8_t*>(w);
    for (int i = 0; i < 12; ++i)
      if (b + i < a.bytes_end) v[i >> 2] |= static_cast<uint32_t>(__ldg(b + i)) << ((i & 3) * 8);
    w0 = v[0];
    w1 = v[1];
    w2 = v[2];
  }
  Win r;
  r.lo = __funnelshift_r(w0, w1, sh);
  r.hi = narrow ? 0u : __funnelshift_r(w1, w2, sh);
  return r;
}

// The same without the end check, for windows known to end inside the bytestream.
__device__ __forceinline__ Win window_in(const uint8_t* s, int64_t bit, bool narrow) {
  const uintptr_t pa = reinterpret_cast<uintptr_t>(s + (bit >> 3));
  const uint32_t* w = reinterpret_cast<const uint32_t*>(pa & ~static_cast<uintptr_t>(3));
  const uint32_t sh = static_cast<uint32_t>((pa & 3) * 8 + (bit & 7));
  const uint32_t w0 = __ldg(w), w1 = __ldg(w + 1), w2 = narrow ? 0u : __ldg(w + 2);
  Win r;
  r.lo = __funnelshift_r(w0, w1, sh);
  r.hi = narrow ? 0u : __funnelshift_r(w1, w2, sh);
  return r;
}
// Whether the 12 bytes a window at `bit` may touch lie inside the bytestream's last word.
__device__ __forceinline__ bool window_inside(const AttnArgs& a, const uint8_t* s, int64_t bit) {
  const uintptr_t pa = reinterpret_cast<uintptr_t>(s + (bit >> 3)) & ~static_cast<uintptr_t>(3);
  return pa + 12 <= ((reinterpret_cast<uintptr_t>(a.bytes_end) + 3) & ~static_cast<uintptr_t>(3));
}

// 8 windows at bit positions base + j * step (increasing), all loads issued before any use.
__device__ __forceinline__ void windows8(const AttnArgs& a, const uint8_t* s, int64_t base, int64_t step, bool narrow,
                                         Win (&w)[8]) {
  if (window_inside(a, s, base + 7 * step)) {
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = window_in(s, base + j * step, narrow);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = window(a, s, base + j * step, narrow);
  }
}

// The symbol at bit `pos` of a window as an exact float: bfe, then 2^23 + s - 2^23 (no
// int -> float conversion instruction; exact for every symbol value).
__device__ __forceinline__ float sym_at(const Win& w, uint32_t pos, uint32_t len) {
  const uint32_t word = pos < 32 ? w.lo : w.hi;
  uint32_t v;
  asm("bfe.u32 %0, %1, %2, %3;" : "=r"(v) : "r"(word), "r"(pos & 31u), "r"(len));
  return __uint_as_float(0x4B000000u | v) - 8388608.f;
}

// 8 consecutive fp16 values p[i .. i+7] as floats (one 16-byte load when `vec`).
__device__ __forceinline__ void h2f8(const __half* p, int64_t i, bool vec, float (&o)[8]) {
  if (vec) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p + i));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
      o[2 * k] = f.x;
      o[2 * k + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = h2f(p, i + k);
  }
}

// Symbol `idx` of stream kv.
__device__ __forceinline__ uint32_t symbol(const AttnArgs& a, int kv, int64_t idx) {
  return static_cast<uint32_t>(bits64(a, a.stream[kv], idx * a.slot_bits)) & static_cast<uint32_t>(a.sym_mask);
}

// One element (kv, key, channel ch = h * 128 + d) as the reference reads it, in fp32;
// nullopt-free: keys past `kmax` and invalid blocks read as 0.
template <int CODEC>
__device__ float element(const AttnArgs& a, int kv, int64_t key, int h, int d, int64_t kmax) {
  if (key > kmax) return 0.f;
  const int64_t C = static_cast<int64_t>(a.kv_heads) * kD;
  const int64_t ch = static_cast<int64_t>(h) * kD + d;
  if (key < a.prefix) {
    if (CODEC == 0) {
      if (key < a.sink) return h2f(a.sink_kv[kv], key * C + ch);
      const int64_t bt = key - a.sink;
      if (kv == 0) {
        const uint32_t s = symbol(a, 0, (static_cast<int64_t>(d) * a.kv_heads + h) * a.body + bt);
        const int64_t m = (bt / a.group_size) * C + ch;
        return __fmaf_rn(static_cast<float>(s), h2f(a.scale[0], m), h2f(a.zero[0], m));
      }
      const uint32_t s = symbol(a, 1, ch * a.body + bt);
      const int64_t vg = (C + a.group_size - 1) / a.group_size;
      const int64_t m = bt * vg + ch / a.group_size;
      return __fmaf_rn(static_cast<float>(s), h2f(a.scale[1], m), h2f(a.zero[1], m));
    }
    if (kv == 0) {
      const uint32_t s = symbol(a, 0, (static_cast<int64_t>(d) * a.kv_heads + h) * a.prefix + key);
      return __fmaf_rn(static_cast<float>(s), h2f(a.scale[0], ch), h2f(a.zero[0], ch));
    }
    const uint32_t s = symbol(a, 1, (static_cast<int64_t>(h) * a.prefix + key) * kD + d);
    return __fmaf_rn(static_cast<float>(s), h2f(a.scale[1], key), h2f(a.zero[1], key));
  }
  const int64_t pb = __ldg(a.block_table + key / a.block_size);
  if (pb < 0 || pb >= a.num_blocks) return 0.f;
  const int64_t e = kv * a.kv_stride + pb * a.block_stride + (key % a.block_size) * a.token_stride + ch;
  return bits_to_float(__ldg(a.cache + e), a.cache_bf16 != 0);
}

// 8 cache elements (dims 8*dq .. 8*dq + 7) of one key as 4 words of the query type.
template <typename QT>
__device__ __forceinline__ void cache_row8(const AttnArgs& a, int kv, int64_t key, int h, int dq, uint32_t (&w)[4]) {
  const int64_t pb = __ldg(a.block_table + key / a.block_size);
  if (pb < 0 || pb >= a.num_blocks) {
    w[0] = w[1] = w[2] = w[3] = 0u;
    return;
  }
  const int64_t e = kv * a.kv_stride + pb * a.block_stride + (key % a.block_size) * a.token_stride +
                    static_cast<int64_t>(h) * kD + 8 * dq;
  if (a.cache_vec) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(a.cache + e));
    w[0] = v.x;
    w[1] = v.y;
    w[2] = v.z;
    w[3] = v.w;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w[i] = static_cast<uint32_t>(__ldg(a.cache + e + 2 * i)) | (static_cast<uint32_t>(__ldg(a.cache + e + 2 * i + 1)) << 16);
  }
  if (a.cache_bf16 != static_cast<int32_t>(is_bf16<QT>())) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w[i] = pack2<QT>(bits_to_float(static_cast<uint16_t>(w[i] & 0xFFFF), a.cache_bf16 != 0),
                       bits_to_float(static_cast<uint16_t>(w[i] >> 16), a.cache_bf16 != 0));
  }
}

// 8 sink elements (dims 8*dq .. 8*dq + 7) of sink token `key` as 4 words of the query type.
template <typename QT>
__device__ __forceinline__ void sink_row8(const AttnArgs& a, int kv, int64_t key, int h, int dq, uint32_t (&w)[4]) {
  const int64_t C = static_cast<int64_t>(a.kv_heads) * kD;
  float f[8];
  h2f8(a.sink_kv[kv], key * C + static_cast<int64_t>(h) * kD + 8 * dq, a.meta_vec != 0, f);
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = pack2<QT>(f[2 * i], f[2 * i + 1]);
}

}  // namespace attn

namespace attn {

// An 8 x 8 block element by element (sink tokens, octets that straddle the sink, prefix or
// kmax boundaries): rows are keys (K) or dims (V^T). Rarely taken, so kept out of line
// and not unrolled to keep the hot loop's code small.
template <typename QT, int CODEC>
__device__ __noinline__ void block_by_element(const AttnArgs& a, int kv, int h, int64_t kb, int dq, int64_t kmax,
                                              uint8_t* dst) {
  for (int r = 0; r < 8; ++r) {
    uint32_t w4[4];
    for (int w = 0; w < 4; ++w) {
      const float lo = kv == 0 ? element<CODEC>(a, 0, kb + r, h, 8 * dq + 2 * w, kmax)
                               : element<CODEC>(a, 1, kb + 2 * w, h, 8 * dq + r, kmax);
      const float hi = kv == 0 ? element<CODEC>(a, 0, kb + r, h, 8 * dq + 2 * w + 1, kmax)
                               : element<CODEC>(a, 1, kb + 2 * w + 1, h, 8 * dq + r, kmax);
      w4[w] = pack2<QT>(lo, hi);
    }
    *reinterpret_cast<uint4*>(dst + r * 16) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
  }
}

// Per-thread constants of the dequant blocks (one CTA = one KV head h; the thread's K
// block has dims 8*k_dq.., its V^T block dims 8*v_dq..).
struct BlockCtx {
  int64_t k_row0, k_row;  // K stream bit of (dim 8*k_dq, token 0); bits between consecutive dims
  int64_t v_row0, v_row;  // V stream: KIVI (dim 8*v_dq, token 0) / dims; KVQuant (token 0, dim 8*v_dq) / tokens
  int64_t v_cg0, v_cg7;   // KIVI value channel groups of dims 8*v_dq and 8*v_dq + 7
  float ksc[8], kze[8];   // KVQuant per-channel key scale / zero of the K block's dims
};

template <int CODEC>
__device__ __forceinline__ void block_ctx(const AttnArgs& a, int h, int k_dq, int v_dq, BlockCtx& c) {
  const int64_t slot = a.slot_bits;
  const int64_t run = CODEC == 0 ? a.body : a.prefix;  // tokens per K (and KIVI V) dim run
  c.k_row0 = (static_cast<int64_t>(8 * k_dq) * a.kv_heads + h) * run * slot;
  c.k_row = static_cast<int64_t>(a.kv_heads) * run * slot;
  if (CODEC == 0) {
    c.v_row0 = (static_cast<int64_t>(h) * kD + 8 * v_dq) * a.body * slot;
    c.v_row = a.body * slot;
    const int64_t ch0 = static_cast<int64_t>(h) * kD + 8 * v_dq;
    c.v_cg0 = ch0 / a.group_size;
    c.v_cg7 = (ch0 + 7) / a.group_size;
  } else {
    c.v_row0 = (static_cast<int64_t>(h) * a.prefix * kD + 8 * v_dq) * slot;
    c.v_row = kD * slot;
    c.v_cg0 = c.v_cg7 = 0;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    c.ksc[j] = 0.f;
    c.kze[j] = 0.f;
  }
  if (CODEC == 1) {
    const int64_t ch0 = static_cast<int64_t>(h) * kD + 8 * k_dq;
    h2f8(a.scale[0], ch0, a.meta_vec != 0, c.ksc);
    h2f8(a.zero[0], ch0, a.meta_vec != 0, c.kze);
  }
}

// K block: keys kb .. kb+7 (rows) x dims 8*dq .. 8*dq+7, into the K tile at row group ko.
template <typename QT, int CODEC>
__device__ __forceinline__ void k_block(const AttnArgs& a, const BlockCtx& c, int h, int64_t kb, int dq, int ko,
                                        int64_t kmax, uint8_t* tile) {
  uint32_t m[8][4];
  const int64_t C = static_cast<int64_t>(a.kv_heads) * kD;
  const int64_t ch0 = static_cast<int64_t>(h) * kD + 8 * dq;
  const bool in_kmax = kb + 7 <= kmax;
  if (in_kmax && kb + 7 < a.prefix && (CODEC == 1 || kb >= a.sink)) {
    // each dim's run holds the 8 keys consecutively
    const int64_t bt0 = CODEC == 0 ? kb - a.sink : kb;
    const bool narrow = a.slot_bits <= 4;
    const uint32_t slot = static_cast<uint32_t>(a.slot_bits), len = static_cast<uint32_t>(a.sym_len);
    Win win[8];
    windows8(a, a.stream[0], c.k_row0 + bt0 * a.slot_bits, c.k_row, narrow, win);
    float sc[8], ze[8];
    int64_t g = 0, r = 0;
    if (CODEC == 0) {
      g = bt0 / a.group_size;
      r = bt0 - g * a.group_size;
      h2f8(a.scale[0], g * C + ch0, a.meta_vec != 0, sc);
      h2f8(a.zero[0], g * C + ch0, a.meta_vec != 0, ze);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (CODEC == 0 && i > 0) {
        // a group of at least 8 tokens changes at most once inside 8 keys
        const int64_t gi = a.group_size >= 8 ? g + (r + i == a.group_size ? 1 : 0) : (bt0 + i) / a.group_size;
        if (gi != g) {
          g = gi;
          if (a.group_size >= 8) r -= a.group_size;
          h2f8(a.scale[0], g * C + ch0, a.meta_vec != 0, sc);
          h2f8(a.zero[0], g * C + ch0, a.meta_vec != 0, ze);
        }
      }
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float sy = sym_at(win[j], i * slot, len);
        v[j] = CODEC == 0 ? __fmaf_rn(sy, sc[j], ze[j]) : __fmaf_rn(sy, c.ksc[j], c.kze[j]);
      }
#pragma unroll
      for (int w = 0; w < 4; ++w) m[i][w] = pack2<QT>(v[2 * w], v[2 * w + 1]);
    }
  } else if (in_kmax && kb >= a.prefix) {
#pragma unroll
    for (int i = 0; i < 8; ++i) cache_row8<QT>(a, 0, kb + i, h, dq, m[i]);
  } else if (CODEC == 0 && in_kmax && kb + 7 < a.sink) {
#pragma unroll
    for (int i = 0; i < 8; ++i) sink_row8<QT>(a, 0, kb + i, h, dq, m[i]);
  } else {
    block_by_element<QT, CODEC>(a, 0, h, kb, dq, kmax, tile + ko * kSBO + dq * kLBO);
    return;
  }
  uint8_t* dst = tile + ko * kSBO + dq * kLBO;
#pragma unroll
  for (int i = 0; i < 8; ++i) *reinterpret_cast<uint4*>(dst + i * 16) = make_uint4(m[i][0], m[i][1], m[i][2], m[i][3]);
}

// V^T block: dims 8*dq .. 8*dq+7 (rows) x keys kb .. kb+7, into the V^T tile at row group dq.
template <typename QT, int CODEC>
__device__ __forceinline__ void v_block(const AttnArgs& a, const BlockCtx& c, int h, int64_t kb, int dq, int ko,
                                        int64_t kmax, uint8_t* tile) {
  uint32_t m[8][4];
  const int64_t C = static_cast<int64_t>(a.kv_heads) * kD;
  const int64_t ch0 = static_cast<int64_t>(h) * kD + 8 * dq;
  const bool in_kmax = kb + 7 <= kmax;
  if (in_kmax && kb + 7 < a.prefix && (CODEC == 1 || kb >= a.sink)) {
    const bool narrow = a.slot_bits <= 4;
    const uint32_t slot = static_cast<uint32_t>(a.slot_bits), len = static_cast<uint32_t>(a.sym_len);
    if (CODEC == 0) {
      // dim j's run holds the 8 keys consecutively; scale / zero by (key, channel group)
      const int64_t bt0 = kb - a.sink;
      const int64_t vg = (C + a.group_size - 1) / a.group_size;
      const bool one_group = c.v_cg0 == c.v_cg7;
      Win wins[8];
      windows8(a, a.stream[1], c.v_row0 + bt0 * a.slot_bits, c.v_row, narrow, wins);
      float sc[8], ze[8];
      if (one_group) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          sc[i] = h2f(a.scale[1], (bt0 + i) * vg + c.v_cg0);
          ze[i] = h2f(a.zero[1], (bt0 + i) * vg + c.v_cg0);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const Win& win = wins[j];
        float v[8];
        if (one_group) {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = __fmaf_rn(sym_at(win, i * slot, len), sc[i], ze[i]);
        } else {
          const int64_t cg = (ch0 + j) / a.group_size;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            v[i] = __fmaf_rn(sym_at(win, i * slot, len), h2f(a.scale[1], (bt0 + i) * vg + cg),
                             h2f(a.zero[1], (bt0 + i) * vg + cg));
        }
#pragma unroll
        for (int w = 0; w < 4; ++w) m[j][w] = pack2<QT>(v[2 * w], v[2 * w + 1]);
      }
    } else {
      // key i's run holds the 8 dims consecutively; one scale / zero per key. Rows are
      // built per key, then transposed to rows per dim.
      Win wins[8];
      windows8(a, a.stream[1], c.v_row0 + kb * c.v_row, c.v_row, narrow, wins);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const Win& win = wins[i];
        const float sc = h2f(a.scale[1], kb + i), ze = h2f(a.zero[1], kb + i);
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __fmaf_rn(sym_at(win, j * slot, len), sc, ze);
#pragma unroll
        for (int w = 0; w < 4; ++w) m[i][w] = pack2<QT>(v[2 * w], v[2 * w + 1]);
      }
      transpose8x8_u16(m);
    }
  } else if (in_kmax && kb >= a.prefix) {
#pragma unroll
    for (int i = 0; i < 8; ++i) cache_row8<QT>(a, 1, kb + i, h, dq, m[i]);
    transpose8x8_u16(m);
  } else if (CODEC == 0 && in_kmax && kb + 7 < a.sink) {
#pragma unroll
    for (int i = 0; i < 8; ++i) sink_row8<QT>(a, 1, kb + i, h, dq, m[i]);
    transpose8x8_u16(m);
  } else {
    block_by_element<QT, CODEC>(a, 1, h, kb, dq, kmax, tile + dq * kSBO + ko * kLBO);
    return;
  }
  uint8_t* dst = tile + dq * kSBO + ko * kLBO;
#pragma unroll
  for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(dst + j * 16) = make_uint4(m[j][0], m[j][1], m[j][2], m[j][3]);
}

// Reduce 8 values over the 32 lanes of a warp with 9 shuffles; lane l ends with the
// result for value index ((l >> 4) & 1) * 4 + ((l >> 3) & 1) * 2 + ((l >> 2) & 1).
template <bool MAX>
__device__ __forceinline__ float warp_reduce8(const float (&v)[8], int lane) {
  auto op = [](float x, float y) { return MAX ? fmaxf(x, y) : x + y; };
  float a4[4], a2[2];
  const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float send = b4 ? v[k] : v[k + 4];
    const float keep = b4 ? v[k + 4] : v[k];
    a4[k] = op(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float send = b3 ? a4[k] : a4[k + 2];
    const float keep = b3 ? a4[k + 2] : a4[k];
    a2[k] = op(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
  const float send = b2 ? a2[0] : a2[1];
  float r = op(b2 ? a2[1] : a2[0], __shfl_xor_sync(0xffffffffu, send, 4));
  r = op(r, __shfl_xor_sync(0xffffffffu, r, 2));
  r = op(r, __shfl_xor_sync(0xffffffffu, r, 1));
  return r;
}

__device__ __forceinline__ void named_sync_softmax() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }

}  // namespace attn

// Merge of the splits of one row block by the CTA that finished last. The first round of
// partial-O loads goes out before the weights: one warp per row turns the splits' (max,
// sum) into weights exp2(max_s - max) / sum in `stage` (splits * NQ floats of free shared
// memory); each thread then accumulates NQ / 8 float4 of O over the splits, 16 float4
// loads in flight.
template <typename QT, int NQ>
__device__ __forceinline__ void split_merge(const AttnArgs& a, int h, int rb, int row0, float* stage) {
  using namespace attn;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __threadfence();
  const int64_t blk0 = (static_cast<int64_t>(h) * a.row_blocks + rb) * a.splits;
  constexpr int kPer = NQ * kD / 4 / kThreadsA;  // float4 of O per thread
  constexpr int kU = kPer >= 16 ? 1 : 16 / kPer;  // splits per round
  constexpr int kSplit4 = NQ * kD / 4;            // float4 per split
  const float4* o = reinterpret_cast<const float4*>(a.ws_o + blk0 * NQ * kD);
  float4 v[kPer][kU];
#pragma unroll
  for (int k = 0; k < kPer; ++k)
#pragma unroll
    for (int u = 0; u < kU; ++u)
      v[k][u] = u < a.splits ? __ldcg(o + static_cast<int64_t>(u) * kSplit4 + tid + k * kThreadsA)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
  float* w_sm = stage;  // [splits][NQ]
  for (int n = warp; n < NQ; n += kThreadsA / 32) {
    // (max, sum) of splits lane + 32 i, loaded once (splits <= 4096 / NQ <= 512)
    constexpr int kMl = (4096 / NQ + 31) / 32;
    float2 ml[kMl];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMl; ++i) {
      const int s2 = lane + 32 * i;
      ml[i] = s2 < a.splits ? __ldcg(reinterpret_cast<const float2*>(a.ws_ml) + (blk0 + s2) * NQ + n)
                            : make_float2(-INFINITY, 0.f);
      mx = fmaxf(mx, ml[i].x);
    }
#pragma unroll
    for (int x = 16; x > 0; x >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, x));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kMl; ++i) {
      const int s2 = lane + 32 * i;
      if (s2 < a.splits) {
        const float w = ml[i].x == -INFINITY ? 0.f : exp2f(ml[i].x - mx);
        sum += w * ml[i].y;
        w_sm[s2 * NQ + n] = w;
      }
    }
#pragma unroll
    for (int x = 16; x > 0; x >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, x);
    const float inv = 1.f / sum;
    __syncwarp();
    for (int s2 = lane; s2 < a.splits; s2 += 32) w_sm[s2 * NQ + n] *= inv;
  }
  __syncthreads();
  auto fma4 = [](float4& c, const float4& x, float w) {
    c.x = __fmaf_rn(x.x, w, c.x);
    c.y = __fmaf_rn(x.y, w, c.y);
    c.z = __fmaf_rn(x.z, w, c.z);
    c.w = __fmaf_rn(x.w, w, c.w);
  };
  float4 acc[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s2 = 0; s2 < a.splits; s2 += kU) {
    if (s2 > 0) {
#pragma unroll
      for (int k = 0; k < kPer; ++k)
#pragma unroll
        for (int u = 0; u < kU; ++u)
          v[k][u] = s2 + u < a.splits ? __ldcg(o + static_cast<int64_t>(s2 + u) * kSplit4 + tid + k * kThreadsA)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k)
#pragma unroll
      for (int u = 0; u < kU; ++u)
        if (s2 + u < a.splits) fma4(acc[k], v[k][u], w_sm[(s2 + u) * NQ + (tid + k * kThreadsA) / (kD / 4)]);
  }
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int f = tid + k * kThreadsA;
    const int row = row0 + f / (kD / 4), d = (f % (kD / 4)) * 4;
    if (row >= a.rows) continue;
    const int64_t q = row / a.group;
    const int64_t qh = static_cast<int64_t>(h) * a.group + row % a.group;
    uint16_t* out = a.output + (q * a.q_heads + qh) * kD + d;
    out[0] = from_float<QT>(acc[k].x);
    out[1] = from_float<QT>(acc[k].y);
    out[2] = from_float<QT>(acc[k].z);
    out[3] = from_float<QT>(acc[k].w);
  }
}

template <int NQ>
struct AttnSmem {
  static constexpr int q_bytes = (NQ / 8) * attn::kSBO;  // Q rows and P rows, [NQ x 128] each
  static constexpr int scalars = 4 * NQ + 4 * NQ;        // red[4][NQ], m_run, l_run, alpha, m_new
  static constexpr int bytes = 2 * attn::kTileBytes + 2 * q_bytes + scalars * 4 + NQ * 8 + 16 + 16 + 128;
};

// grid = kv_heads * row_blocks * splits CTAs of 256 threads.
template <typename QT, int CODEC, int NQ>
__global__ void __launch_bounds__(attn::kThreadsA, 2) prefix_attention(const __grid_constant__ AttnArgs a) {
  using namespace attn;
  static_assert(NQ % 8 == 0 && NQ >= 8 && NQ <= 64, "NQ rows per CTA");
  extern __shared__ __align__(128) uint8_t attn_smem[];
  uint8_t* sm = attn_smem + ((128 - (smem_u32(attn_smem) & 127)) & 127);
  uint8_t* kt_sm = sm;                                   // K tile  [128 keys x 128 dims]
  uint8_t* vt_sm = kt_sm + kTileBytes;                   // V^T tile [128 dims x 128 keys]
  uint8_t* q_sm = vt_sm + kTileBytes;                    // Q rows  [NQ x 128 dims]
  uint8_t* p_sm = q_sm + AttnSmem<NQ>::q_bytes;          // P rows  [NQ x 128 keys]
  float* red = reinterpret_cast<float*>(p_sm + AttnSmem<NQ>::q_bytes);  // [4][NQ]
  float* m_run = red + 4 * NQ;
  float* l_run = m_run + NQ;
  float* alpha = l_run + NQ;
  float* m_new = alpha + NQ;
  int64_t* cend = reinterpret_cast<int64_t*>(m_new + NQ);  // causal end of each row, -1 = no row
  uint64_t* bars = reinterpret_cast<uint64_t*>(cend + NQ);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
  uint32_t* last_flag = tslot + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sp = static_cast<int>(blockIdx.x % a.splits);
  const int rest = static_cast<int>(blockIdx.x / a.splits);
  const int rb = rest % a.row_blocks;
  const int h = rest / a.row_blocks;
  const int row0 = rb * NQ;
  const int last_row = min(a.rows, row0 + NQ) - 1;
  const int64_t kmax = min(a.seq_len - 1, a.q_start + last_row / a.group);
  const int nkt = static_cast<int>(kmax / kKT) + 1;
  const int t_begin = static_cast<int>(static_cast<int64_t>(sp) * nkt / a.splits);
  const int t_end = static_cast<int>(static_cast<int64_t>(sp + 1) * nkt / a.splits);
  constexpr bool kBf16 = is_bf16<QT>();
  constexpr uint32_t idesc = instr_desc(kBf16, NQ);

  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tslot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  // Q rows of this block (zero for rows past the end)
  for (int e = tid; e < NQ * 16; e += kThreadsA) {
    const int n = e >> 4, c = e & 15;
    const int row = row0 + n;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (row < a.rows) {
      const int64_t q = row / a.group;
      const int64_t qh = static_cast<int64_t>(h) * a.group + row % a.group;
      const uint16_t* src = a.query + (q * a.q_heads + qh) * kD + 8 * c;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        w[i] = static_cast<uint32_t>(src[2 * i]) | (static_cast<uint32_t>(src[2 * i + 1]) << 16);
    }
    *reinterpret_cast<uint4*>(q_sm + (n >> 3) * kSBO + c * kLBO + (n & 7) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (tid < NQ) {
    const int row = row0 + tid;
    m_run[tid] = -INFINITY;
    l_run[tid] = 0.f;
    cend[tid] = row < a.rows ? min(a.seq_len - 1, a.q_start + row / a.group) : -1;
  }
  // key octet fastest in both blocks: 16 lanes read one dim's run contiguously
  const int k_ko = tid & 15, k_dq = tid >> 4;
  const int v_ko = tid & 15, v_dq = tid >> 4;
  BlockCtx bctx;
  block_ctx<CODEC>(a, h, k_dq, v_dq, bctx);
  proxy_fence();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
  uint32_t ph1 = 0u, ph2 = 0u;
  bool failed = false;

  for (int kt = t_begin; kt < t_end; ++kt) {
    const int j = kt - t_begin;
    const int64_t k0 = static_cast<int64_t>(kt) * kKT;
    // K tile: its previous reader (MMA 1 of the previous tile) has completed.
    k_block<QT, CODEC>(a, bctx, h, k0 + 8 * k_ko, k_dq, k_ko, kmax, kt_sm);
    if (j > 0) {  // V^T tile and P: wait for MMA 2 of the previous tile
      const bool ok = mbar_wait_bounded(&bars[1], ph2);
      ph2 ^= 1u;
      if (__syncthreads_or(!ok)) {
        failed = true;
        break;
      }
    }
    v_block<QT, CODEC>(a, bctx, h, k0 + 8 * v_ko, v_dq, v_ko, kmax, vt_sm);
    proxy_fence();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int s = 0; s < kD / 16; ++s)
        mma_f16(tmem, smem_desc(smem_u32(kt_sm) + 2 * s * kLBO), smem_desc(smem_u32(q_sm) + 2 * s * kLBO), idesc,
                s > 0 ? 1u : 0u);
      mma_commit(&bars[0]);
    }
    {
      const bool ok = mbar_wait_bounded(&bars[0], ph1);
      ph1 ^= 1u;
      if (__syncthreads_or(!ok)) {
        failed = true;
        break;
      }
    }
    tc_fence_after();

    if (warp < 4) {
      // Online softmax: this thread is key k0 + tid; column n of S^T is row n's score.
      const int64_t key = k0 + tid;
#pragma unroll
      for (int c = 0; c < NQ; c += 8) {
        float s[8];
        tmem_ld8(tmem + lane_base + c, s);
#pragma unroll
        for (int n = 0; n < 8; ++n) s[n] = key <= cend[c + n] ? s[n] * a.scale_log2 : -INFINITY;
        const float r = warp_reduce8<true>(s, lane);
        if ((lane & 3) == 0) red[warp * NQ + c + ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1)] = r;
      }
      named_sync_softmax();
      if (tid < NQ) {
        const float tmax = fmaxf(fmaxf(red[tid], red[NQ + tid]), fmaxf(red[2 * NQ + tid], red[3 * NQ + tid]));
        const float mo = m_run[tid];
        const float mn = fmaxf(mo, tmax);
        alpha[tid] = mn == -INFINITY ? 1.f : exp2f(mo - mn);
        m_new[tid] = mn;
      }
      named_sync_softmax();
#pragma unroll
      for (int c = 0; c < NQ; c += 8) {
        float s[8], p[8];
        tmem_ld8(tmem + lane_base + c, s);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const float x = key <= cend[c + n] ? s[n] * a.scale_log2 : -INFINITY;
          p[n] = x == -INFINITY ? 0.f : exp2f(x - m_new[c + n]);
          *reinterpret_cast<uint16_t*>(p_sm + tile_off(c + n, tid)) = from_float<QT>(p[n]);
        }
        const float r = warp_reduce8<false>(p, lane);
        if ((lane & 3) == 0) red[warp * NQ + c + ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1)] = r;
      }
      named_sync_softmax();
      if (tid < NQ) {
        l_run[tid] = l_run[tid] * alpha[tid] + (red[tid] + red[NQ + tid]) + (red[2 * NQ + tid] + red[3 * NQ + tid]);
        m_run[tid] = m_new[tid];
      }
    }
    const bool rescale = __syncthreads_or(tid < NQ && alpha[tid] != 1.f) && j > 0;
    if (warp >= 4 && rescale) {
#pragma unroll
      for (int c = 0; c < NQ; c += 8) {
        float o[8];
        tmem_ld8(tmem + lane_base + kOCol + c, o);
#pragma unroll
        for (int n = 0; n < 8; ++n) o[n] *= alpha[c + n];
        tmem_st8(tmem + lane_base + kOCol + c, o);
      }
      tmem_st_wait();
    }
    proxy_fence();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int s = 0; s < kKT / 16; ++s)
        mma_f16(tmem + kOCol, smem_desc(smem_u32(vt_sm) + 2 * s * kLBO), smem_desc(smem_u32(p_sm) + 2 * s * kLBO),
                idesc, (j > 0 || s > 0) ? 1u : 0u);
      mma_commit(&bars[1]);
    }
  }
  const bool any_tiles = t_end > t_begin;
  if (!failed && any_tiles) {
    const bool ok = mbar_wait_bounded(&bars[1], ph2);
    ph2 ^= 1u;
    failed = __syncthreads_or(!ok);
  }
  if (failed) {
    if (tid == 0 && a.err) atomicOr(a.err, kWaitTimeoutFlag);
    // give the copies in flight one more bounded wait before the columns are released
    mbar_wait_bounded(&bars[0], ph1 ^ 1u);
    mbar_wait_bounded(&bars[1], ph2 ^ 1u);
  } else {
    tc_fence_after();
    if (a.splits == 1) {
      if (warp >= 4) {
        const int d = (warp - 4) * 32 + lane;
#pragma unroll
        for (int c = 0; c < NQ; c += 8) {
          float o[8];
          tmem_ld8(tmem + lane_base + kOCol + c, o);
#pragma unroll
          for (int n = 0; n < 8; ++n) {
            const int row = row0 + c + n;
            if (row < a.rows) {
              const int64_t q = row / a.group;
              const int64_t qh = static_cast<int64_t>(h) * a.group + row % a.group;
              a.output[(q * a.q_heads + qh) * kD + d] = from_float<QT>(o[n] / l_run[c + n]);
            }
          }
        }
      }
    } else {
      const int64_t blk = (static_cast<int64_t>(h) * a.row_blocks + rb) * a.splits + sp;
      if (warp >= 4) {
        const int d = (warp - 4) * 32 + lane;
#pragma unroll
        for (int c = 0; c < NQ; c += 8) {
          float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if (any_tiles) tmem_ld8(tmem + lane_base + kOCol + c, o);
#pragma unroll
          for (int n = 0; n < 8; ++n) a.ws_o[(blk * NQ + c + n) * kD + d] = o[n];
        }
      }
      if (tid < NQ) {
        a.ws_ml[(blk * NQ + tid) * 2] = m_run[tid];
        a.ws_ml[(blk * NQ + tid) * 2 + 1] = l_run[tid];
      }
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        const uint32_t prev = atomicInc(&a.counters[static_cast<int64_t>(h) * a.row_blocks + rb],
                                        static_cast<uint32_t>(a.splits - 1));
        *last_flag = prev == static_cast<uint32_t>(a.splits - 1) ? 1u : 0u;
      }
      __syncthreads();
      if (*last_flag) {
        split_merge<QT, NQ>(a, h, rb, row0, reinterpret_cast<float*>(kt_sm));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols));
  }
}

}  // namespace origami
