// Device helpers shared by the origami_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace origami {

constexpr int kThreads = 256;

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// Tokens per tile for head_dim D: (TT/8) * (D/8) <= 256 work items of 8x8 elements.
__host__ __device__ constexpr int tile_tokens_for(int D) { return 8 * (2048 / D); }

// Shared-memory row stride of one (plane, channel) run of TT symbols at `bits` bits:
// 16-byte rounded; restore rows get 32 spare bytes for unaligned run starts.
__host__ __device__ constexpr int run_stride(int TT, int bits, bool restore) {
  return ((((TT * bits + 7) / 8) + 15) & ~15) + (restore ? 32 : 0);
}

// ---------------------------------------------------------------------------
// Asynchronous global -> shared copies (bypass registers, complete at wait).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src)
               : "memory");
}

__device__ __forceinline__ void cp_async8(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src)
               : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

// ---------------------------------------------------------------------------
// mbarriers and bulk (TMA) copies. Waits are bounded: a kernel whose wait runs out
// flags kWaitTimeoutFlag in its error word instead of spinning forever.
// ---------------------------------------------------------------------------
constexpr uint32_t kWaitTimeoutFlag = 0x80000000u;

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Polls of a bounded mbarrier wait: far beyond any copy's latency, short enough that a
// wait that cannot complete returns an error status in well under a minute.
constexpr uint32_t kWaitPolls = 1u << 22;

// Bounded wait for phase `parity` of an mbarrier; false when the bound ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t polls = kWaitPolls) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < polls; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// Wait for a stage's copies, agreed by the whole CTA (every thread must call it). When any
// thread's bounded wait runs out, the CTA sets kWaitTimeoutFlag in *err, waits once more
// (bounded) for the copies it still has in flight on this stage and, when other_live, on
// the other stage, and the caller returns: true means "leave the kernel". A copy that has
// not landed after that second bound means the memory system itself is stuck; the CTA
// still leaves (the flag already marks the launch's output as void) rather than wait for
// ever. A CTA never waits on another CTA or kernel here, only on its own copies.
__device__ __forceinline__ bool stage_wait_or_bail(uint64_t* bar, uint32_t parity, uint64_t* other,
                                                   uint32_t other_parity, bool other_live, uint32_t* err,
                                                   uint32_t polls = kWaitPolls) {
  const bool ok = mbar_wait_bounded(bar, parity, polls);
  if (!__syncthreads_or(!ok)) return false;
  if (threadIdx.x == 0 && err) atomicOr(err, kWaitTimeoutFlag);
  mbar_wait_bounded(bar, parity, polls);
  if (other_live) mbar_wait_bounded(other, other_parity, polls);
  return true;
}

__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

// 1-D bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16),
// completing `bytes` transactions on the mbarrier.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_u32(smem_dst)),
               "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Streaming 16-byte global store (data is not re-read by this kernel).
__device__ __forceinline__ void st_global_cs16(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};\n" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void st_global_cs8(void* p, uint2 v) {
  asm volatile("st.global.cs.v2.u32 [%0], {%1, %2};\n" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}

// ---------------------------------------------------------------------------
// Byte permutes and transposes.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  return __byte_perm(a, b, sel);
}

// Transpose a 4x4 byte matrix held as 4 words (word r = row r, byte c = column c).
__device__ __forceinline__ void transpose4x4(uint32_t& a0, uint32_t& a1, uint32_t& a2,
                                             uint32_t& a3) {
  const uint32_t t0 = prmt(a0, a1, 0x5140);
  const uint32_t t1 = prmt(a0, a1, 0x7362);
  const uint32_t t2 = prmt(a2, a3, 0x5140);
  const uint32_t t3 = prmt(a2, a3, 0x7362);
  a0 = prmt(t0, t2, 0x5410);
  a1 = prmt(t0, t2, 0x7632);
  a2 = prmt(t1, t3, 0x5410);
  a3 = prmt(t1, t3, 0x7632);
}

// Transpose an 8x8 byte matrix: row r is (lo[r] = bytes 0..3, hi[r] = bytes 4..7).
// On return row r holds what was column r.
__device__ __forceinline__ void transpose8x8(uint32_t (&lo)[8], uint32_t (&hi)[8]) {
  // Quadrants: TL = lo[0..3], TR = hi[0..3], BL = lo[4..7], BR = hi[4..7].
  transpose4x4(lo[0], lo[1], lo[2], lo[3]);
  transpose4x4(hi[0], hi[1], hi[2], hi[3]);
  transpose4x4(lo[4], lo[5], lo[6], lo[7]);
  transpose4x4(hi[4], hi[5], hi[6], hi[7]);
  // New row r < 4: lo = T(TL)[r], hi = T(BL)[r]; row r >= 4: lo = T(TR)[r-4], hi = T(BR)[r-4].
  uint32_t nlo[8], nhi[8];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    nlo[r] = lo[r];
    nhi[r] = lo[r + 4];
    nlo[r + 4] = hi[r];
    nhi[r + 4] = hi[r + 4];
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    lo[r] = nlo[r];
    hi[r] = nhi[r];
  }
}

// ---------------------------------------------------------------------------
// Dense LSB-first bit streams (bit k of a stream = bit k%8 of byte k/8, i.e. bit
// k%32 of little-endian word k/32).
// ---------------------------------------------------------------------------

// 64 bits of a 16-byte-aligned shared-memory row starting at bit `bitpos`.
// Two aligned 64-bit shared loads cover words wi..wi+2 (fewer bank conflicts than three
// 32-bit loads at a 2-word lane stride); reads at most 4 bytes past word wi + 2.
__device__ __forceinline__ void window64(const uint8_t* row, int bitpos, uint32_t& v0,
                                         uint32_t& v1) {
  const int wi = bitpos >> 5;
  const int sh = bitpos & 31;
  const uint2* p = reinterpret_cast<const uint2*>(row) + (wi >> 1);
  const uint2 a = p[0];
  const uint2 b = p[1];
  const bool odd = (wi & 1) != 0;
  const uint32_t w0 = odd ? a.y : a.x;
  const uint32_t w1 = odd ? b.x : a.y;
  const uint32_t w2 = odd ? b.y : b.x;
  v0 = __funnelshift_r(w0, w1, sh);
  v1 = __funnelshift_r(w1, w2, sh);
}

// Words q..q+4 of a 16-byte aligned shared row from two aligned 16-byte loads; reads at
// most 12 bytes past word q + 4.
__device__ __forceinline__ void words5(const uint32_t* src, int q, uint32_t (&s)[5]) {
  const int qa = q & ~3;
  const int d = q & 3;
  const uint4 x = *reinterpret_cast<const uint4*>(src + qa);
  const uint4 y = *reinterpret_cast<const uint4*>(src + qa + 4);
  const uint32_t w[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    s[k] = d == 0 ? w[k] : d == 1 ? w[k + 1] : d == 2 ? w[k + 2] : w[k + 3];
  }
}

__device__ __forceinline__ void spread8_rt(uint32_t v0, uint32_t v1, int bits, uint32_t& lo,
                                           uint32_t& hi) {
  if (bits == 8) {
    lo = v0;
    hi = v1;
    return;
  }
  const uint64_t v = (static_cast<uint64_t>(v1) << 32) | v0;
  const uint32_t m = (1u << bits) - 1u;
  lo = static_cast<uint32_t>(v & m) | (static_cast<uint32_t>((v >> bits) & m) << 8) |
       (static_cast<uint32_t>((v >> (2 * bits)) & m) << 16) |
       (static_cast<uint32_t>((v >> (3 * bits)) & m) << 24);
  hi = static_cast<uint32_t>((v >> (4 * bits)) & m) |
       (static_cast<uint32_t>((v >> (5 * bits)) & m) << 8) |
       (static_cast<uint32_t>((v >> (6 * bits)) & m) << 16) |
       (static_cast<uint32_t>((v >> (7 * bits)) & m) << 24);
}

// Inverse: pack 8 byte symbols (lo = symbols 0..3, hi = 4..7, already masked) into a
// 64-bit LSB-first field of 8*bits bits.
__device__ __forceinline__ uint64_t gather8(uint32_t lo, uint32_t hi, int bits) {
  if (bits == 8) return (static_cast<uint64_t>(hi) << 32) | lo;
  uint64_t v = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v |= static_cast<uint64_t>((lo >> (8 * i)) & 0xFFu) << (i * bits);
    v |= static_cast<uint64_t>((hi >> (8 * i)) & 0xFFu) << ((i + 4) * bits);
  }
  return v;
}

__device__ __forceinline__ uint32_t bit_range_mask(int lo, int hi) {
  // bits [lo, hi) of a word, 0 <= lo <= hi <= 32
  const uint32_t upper = hi >= 32 ? 0xFFFFFFFFu : ((1u << hi) - 1u);
  const uint32_t lower = lo >= 32 ? 0xFFFFFFFFu : ((1u << lo) - 1u);
  return upper & ~lower;
}

}  // namespace origami
