// Persistent, double-buffered kernels for contiguous canonical plane formats whose runs
// are not 16-byte aligned (ragged token counts): every chunk spans all T tokens, the
// chunks of a component are contiguous in canonical (head, channel) order and T*bits is a
// multiple of 8, so run (q, h, c) starts at stream bit comp_base[q]*8 + (h*D + c)*T*bits of
// its job. Aligned formats take the TMA tensor-map kernels (tma_kernels.cuh) instead.
//
// restore_bulk: one bulk (TMA) copy per run row of the 16-byte words covering its bits
//   (mbarrier completion, two stages) -> 64-bit bit windows -> 8x8 byte transposes + plane
//   merge in registers -> token rows in shared memory -> 16-byte stores through the block
//   table.
// pack_bulk: cp.async gather of token rows (two stages) -> split + transpose -> packed runs
//   in shared memory -> whole 16-byte stores of every vector. Each CTA walks a contiguous
//   range of tiles and carries the vector a run shares with the next tile in registers;
//   only the vectors shared across ranges or heads are merged with masked atomics.
// Both kernels walk contiguous tile ranges, so the 16-byte word two neighbouring runs share
// is read from L2 the second time.
#pragma once

#include "tile_kernels.cuh"
#include "tma_kernels.cuh"

namespace origami {

struct BulkArgs {
  uint8_t* packed;       // job 0's packed bytes; job j at packed + j * job_stride
  int64_t job_stride;
  int64_t packed_bytes;  // whole buffer
  int64_t comp_base[kMaxMaps];  // byte offset of component q within a job
  void* rows[kMaxJobs];
  const int64_t* block_ids[kMaxJobs];
  int64_t kv_stride, block_stride, token_stride, head_stride;
  int64_t block_size, num_blocks;
  int64_t T;
  int64_t write_tokens;  // restore: token rows below this are written (a prefix restore when < T)
  int32_t H, tiles_per_head, tiles_per_job, num_tiles;
  uint32_t* err;
};

template <int MODE, int D>
struct BulkGeo {
  using G = TmaGeo<MODE, D>;
  static constexpr int TT = G::TT;
  static constexpr int P = G::P;
  // run row stride in shared memory: the run's bytes plus one 16-byte word of alignment
  // slack (bits == 8) or two (narrower symbols: the 64-bit window reads 3 words)
  __host__ __device__ static constexpr int rs(int p) {
    return ((TT * G::bits(p) / 8 + 15) & ~15) + (G::bits(p) == 8 ? 16 : 32);
  }
  __host__ __device__ static constexpr int plane_off(int p) {
    return p == 0 ? 0 : (p == 1 ? D * rs(0) : D * (rs(0) + rs(1)));
  }
  static constexpr int in_bytes = D * (rs(0) + rs(1) + (P > 2 ? rs(2) : 0));
  static constexpr int bit0_bytes = P * D * 2;  // int16 first bit of each run inside its row
  static constexpr int rowoff_bytes = TT * 8;
  static constexpr int stage_bytes = ((in_bytes + bit0_bytes + 15) & ~15) + rowoff_bytes;
  static constexpr int rows_bytes = TT * D * 2;
  static constexpr int smem_bytes = 2 * stage_bytes + rows_bytes + 16 + 128 + 32;  // + over-read slack
};

template <int TT>
__device__ __forceinline__ void bulk_rowoff(const BulkArgs& a, const TmaTile& t, int64_t* rowoff) {
  const int32_t bs = static_cast<int32_t>(a.block_size);
  for (int i = threadIdx.x; i < TT; i += kThreads) {
    if (i >= t.n) {
      rowoff[i] = -1;
      continue;
    }
    const int32_t tg = static_cast<int32_t>(t.t0) + i;
    const int32_t bi = tg / bs;
    const int64_t blk = a.block_ids[t.job][bi];
    if (blk < 0 || blk >= a.num_blocks) {
      rowoff[i] = -1;
      if (a.err) atomicAdd(a.err, 1u);
    } else {
      rowoff[i] = t.kv * a.kv_stride + blk * a.block_stride + static_cast<int64_t>(tg - bi * bs) * a.token_stride +
                  static_cast<int64_t>(t.h) * a.head_stride;
    }
  }
}

template <int TT>
__device__ __forceinline__ TmaTile bulk_tile(const BulkArgs& a, int tile) {
  TmaTile t;
  t.job = tile / a.tiles_per_job;
  const int in_job = tile - t.job * a.tiles_per_job;
  const int tt = in_job % a.tiles_per_head;
  const int rest = in_job / a.tiles_per_head;
  t.h = rest % a.H;
  t.kv = rest / a.H;
  t.t0 = static_cast<int64_t>(tt) * TT;
  t.n = static_cast<int>(min64(TT, a.T - t.t0));
  return t;
}

// ---------------------------------------------------------------------------------------
// restore_bulk
// ---------------------------------------------------------------------------------------
template <int MODE, int D>
__global__ void __launch_bounds__(kThreads, 2) restore_bulk(const __grid_constant__ BulkArgs args) {
  using BG = BulkGeo<MODE, D>;
  using G = TmaGeo<MODE, D>;
  extern __shared__ __align__(128) uint8_t bulk_smem[];
  uint8_t* smem = bulk_smem + ((128 - (smem_u32(bulk_smem) & 127)) & 127);
  uint8_t* rows_sm = smem + 2 * BG::stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(rows_sm + BG::rows_bytes);
  const int tid = threadIdx.x;

  if (tid == 0) {
    mbar_init(&bars[0], kThreads);
    mbar_init(&bars[1], kThreads);
    fence_mbar_init();
  }
  __syncthreads();

  // Every thread arrives once per stage use (announcing its own bytes) and issues the
  // bulk copies of its run rows; words past the buffer end are read bytewise. The tile's
  // block-table rows go to registers and are written to its stage after the current
  // tile's work.
  RowoffRegs<BG::TT> next_rows;
  auto issue = [&](int s, int tile) {
    const TmaTile t = bulk_tile<BG::TT>(args, tile);
    uint8_t* sb = smem + s * BG::stage_bytes;
    int16_t* bit0 = reinterpret_cast<int16_t*>(sb + BG::in_bytes);
    const int64_t job_base = static_cast<int64_t>(t.job) * args.job_stride;
    uint32_t my_bytes = 0;
    for (int r = tid; r < BG::P * D; r += kThreads) {
      const int p = r / D;
      const int c = r - p * D;
      const int b = G::bits(p);
      const int64_t B = (job_base + args.comp_base[t.kv * BG::P + p]) * 8 +
                        (static_cast<int64_t>(t.h) * D + c) * args.T * b + t.t0 * b;
      const int64_t lo16 = (B >> 3) & ~static_cast<int64_t>(15);
      const int64_t hi16 = (((B + static_cast<int64_t>(t.n) * b + 7) >> 3) + 15) & ~static_cast<int64_t>(15);
      const int64_t full = min64((hi16 - lo16) >> 4, (args.packed_bytes - lo16) >> 4);
      if (full > 0) my_bytes += static_cast<uint32_t>(full) * 16u;
    }
    mbar_expect_tx(&bars[s], my_bytes);
    for (int r = tid; r < BG::P * D; r += kThreads) {
      const int p = r / D;
      const int c = r - p * D;
      const int b = G::bits(p);
      const int64_t B = (job_base + args.comp_base[t.kv * BG::P + p]) * 8 +
                        (static_cast<int64_t>(t.h) * D + c) * args.T * b + t.t0 * b;
      const int64_t lo16 = (B >> 3) & ~static_cast<int64_t>(15);
      const int64_t hi16 = (((B + static_cast<int64_t>(t.n) * b + 7) >> 3) + 15) & ~static_cast<int64_t>(15);
      const int64_t words = (hi16 - lo16) >> 4;
      const int64_t full = min64(words, (args.packed_bytes - lo16) >> 4);
      uint8_t* row = sb + BG::plane_off(p) + c * BG::rs(p);
      bit0[r] = static_cast<int16_t>(B - lo16 * 8);
      if (full > 0) bulk_load(row, args.packed + lo16, static_cast<uint32_t>(full) * 16u, &bars[s]);
      for (int64_t w = max64(full, 0); w < words; ++w) {
        const int64_t gofs = lo16 + 16 * w;
        uint32_t v[4] = {0u, 0u, 0u, 0u};
        for (int j = 0; j < 16; ++j) {
          if (gofs + j < args.packed_bytes) v[j >> 2] |= static_cast<uint32_t>(args.packed[gofs + j]) << (8 * (j & 3));
        }
        *reinterpret_cast<uint4*>(row + 16 * w) = make_uint4(v[0], v[1], v[2], v[3]);
      }
    }
    rowoff_load<BG::TT>(args, t, next_rows);
  };

  const int per = args.num_tiles / static_cast<int>(gridDim.x);
  const int extra = args.num_tiles % static_cast<int>(gridDim.x);
  const int first = static_cast<int>(blockIdx.x) * per + min(static_cast<int>(blockIdx.x), extra);
  const int last = first + per + (static_cast<int>(blockIdx.x) < extra ? 1 : 0);
  int tile = first;
  if (tile < last) {
    issue(0, tile);
    rowoff_store<BG::TT>(args.err, next_rows, reinterpret_cast<int64_t*>(smem + BG::stage_bytes - BG::rowoff_bytes));
  }
  uint32_t phases = 0u;
  const int a = tid % G::A;
  const int o = tid / G::A;

  for (int j = 0; tile < last; ++j, ++tile) {
    const int s = j & 1;
    const int next = tile + 1;
    if (next < last) issue(s ^ 1, next);
    if (stage_wait_or_bail(&bars[s], (phases >> s) & 1u, &bars[s ^ 1], (phases >> (s ^ 1)) & 1u, next < last,
                           args.err))
      return;
    phases ^= 1u << s;
    const TmaTile t = bulk_tile<BG::TT>(args, tile);
    uint8_t* rows = static_cast<uint8_t*>(args.rows[t.job]);
    const uint8_t* sb = smem + s * BG::stage_bytes;
    const int16_t* bit0 = reinterpret_cast<const int16_t*>(sb + BG::in_bytes);

    uint32_t out[8][4];
    uint32_t keep_lo[8], keep_hi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i][0] = out[i][1] = out[i][2] = out[i][3] = 0u;
#pragma unroll
    for (int p = 0; p < BG::P; ++p) {
      const int b = G::bits(p);
      uint32_t lo[8], hi[8];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int c = 8 * o + jj;
        const uint8_t* row = sb + BG::plane_off(p) + c * BG::rs(p);
        const int pos = bit0[p * D + c] + 8 * a * b;
        if (b == 8 && (pos & 63) == 0) {
          const uint2 v = *reinterpret_cast<const uint2*>(row + (pos >> 3));
          lo[jj] = v.x;
          hi[jj] = v.y;
        } else {
          uint32_t v0, v1;
          window64(row, pos, v0, v1);
          spread8_rt(v0, v1, b, lo[jj], hi[jj]);
        }
      }
      transpose8x8(lo, hi);
      if constexpr (MODE == kModeByte2) {
        if (p == 0) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            keep_lo[i] = lo[i];
            keep_hi[i] = hi[i];
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            out[i][0] = prmt(lo[i], keep_lo[i], 0x5140);
            out[i][1] = prmt(lo[i], keep_lo[i], 0x7362);
            out[i][2] = prmt(hi[i], keep_hi[i], 0x5140);
            out[i][3] = prmt(hi[i], keep_hi[i], 0x7362);
          }
        }
      } else {
        const int sh = G::shift(p);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          out[i][0] |= prmt(lo[i], 0u, 0x4140) << sh;
          out[i][1] |= prmt(lo[i], 0u, 0x4342) << sh;
          out[i][2] |= prmt(hi[i], 0u, 0x4140) << sh;
          out[i][3] |= prmt(hi[i], 0u, 0x4342) << sh;
        }
      }
    }
    const int phys = (o + a) & (G::O - 1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      *reinterpret_cast<uint4*>(rows_sm + (8 * a + i) * (D * 2) + phys * 16) =
          make_uint4(out[i][0], out[i][1], out[i][2], out[i][3]);
    }
    __syncthreads();
    const int64_t* rowoff = reinterpret_cast<const int64_t*>(sb + BG::stage_bytes - BG::rowoff_bytes);
    const int oc = tid % G::O;
    for (int r = tid / G::O; r < t.n; r += kThreads / G::O) {
      const int64_t off = rowoff[r];
      if (off < 0) continue;
      st_global_cs16(rows + (off + 8 * oc) * 2,
                     *reinterpret_cast<const uint4*>(rows_sm + r * (D * 2) + ((oc + (r >> 3)) & (G::O - 1)) * 16));
    }
    if (next < last)
      rowoff_store<BG::TT>(args.err, next_rows,
                           reinterpret_cast<int64_t*>(smem + (s ^ 1) * BG::stage_bytes + BG::stage_bytes - BG::rowoff_bytes));
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------
// pack_bulk
// ---------------------------------------------------------------------------------------
template <int MODE, int D>
struct PackBulkGeo {
  using G = TmaGeo<MODE, D>;
  // packed run row stride: the run's bytes rounded to 16, plus 16 when that is a multiple of
  // 128 bytes so that neighbouring channels start in different banks (the vector reads of
  // the last row run at most 16 bytes past it, into the tail slack)
  __host__ __device__ static constexpr int rs(int p) {
    return ((G::TT * G::bits(p) / 8 + 15) & ~15) + (((G::TT * G::bits(p) / 8 + 15) & ~15) % 128 == 0 ? 16 : 0);
  }
  __host__ __device__ static constexpr int plane_off(int p) {
    return p == 0 ? 0 : (p == 1 ? D * rs(0) : D * (rs(0) + rs(1)));
  }
  static constexpr int rows_bytes = G::TT * D * 2;
  static constexpr int rowoff_bytes = G::TT * 8;
  static constexpr int stage_bytes = rows_bytes + rowoff_bytes;
  static constexpr int out_bytes = D * (rs(0) + rs(1) + (G::P > 2 ? rs(2) : 0));
  static constexpr int smem_bytes = 2 * stage_bytes + out_bytes + 128 + 32;  // + over-read slack of words5
  static constexpr int runs_per_thread = (G::P * D + kThreads - 1) / kThreads;
};

// Word k of the 128-bit vector whose first bit sits at run bit `rel` (may be negative):
// the run's bits [0, len) that fall into the word, shifted into place, and their mask.
__device__ __forceinline__ void run_word(const uint32_t* src, int wr, int len, uint32_t& v, uint32_t& own) {
  const int q = wr >> 5;
  const int r = wr & 31;
  const int nsw = (len + 31) >> 5;
  const uint32_t lo = (q >= 0 && q < nsw) ? src[q] : 0u;
  const uint32_t hi = (q + 1 >= 0 && q + 1 < nsw) ? src[q + 1] : 0u;
  own = bit_range_mask(max(-wr, 0), min(max(len - wr, 0), 32));
  v = __funnelshift_r(lo, hi, r) & own;
}

template <int MODE, int D>
__global__ void __launch_bounds__(kThreads, 2) pack_bulk(const __grid_constant__ BulkArgs args) {
  using G = TmaGeo<MODE, D>;
  using PG = PackBulkGeo<MODE, D>;
  extern __shared__ __align__(128) uint8_t bulk_smem[];
  uint8_t* smem = bulk_smem + ((128 - (smem_u32(bulk_smem) & 127)) & 127);
  uint8_t* out_sm = smem + 2 * PG::stage_bytes;
  const int tid = threadIdx.x;

  auto gather = [&](int s, int tile) {
    const TmaTile t = bulk_tile<G::TT>(args, tile);
    const uint8_t* rows = static_cast<const uint8_t*>(args.rows[t.job]);
    uint8_t* sb = smem + s * PG::stage_bytes;
    int64_t* rowoff = reinterpret_cast<int64_t*>(sb + PG::rows_bytes);
    bulk_rowoff<G::TT>(args, t, rowoff);
    __syncthreads();
    const int oc = tid % G::O;
    for (int r = tid / G::O; r < t.n; r += kThreads / G::O) {
      const int64_t off = rowoff[r];
      uint8_t* dst = sb + r * (D * 2) + ((oc + (r >> 3)) & (G::O - 1)) * 16;
      if (off < 0) *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      else cp_async16(dst, rows + (off + 8 * oc) * 2);
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };

  // Each CTA takes a contiguous range of tiles, so consecutive tiles of one (job, kv, head)
  // continue the same runs: the 128-bit vector a run shares with the previous tile's run is
  // completed in registers (carry) and stored whole. Only vectors shared across CTA ranges
  // and head ends are merged with masked atomics.
  const int per = args.num_tiles / static_cast<int>(gridDim.x);
  const int extra = args.num_tiles % static_cast<int>(gridDim.x);
  const int first = static_cast<int>(blockIdx.x) * per + min(static_cast<int>(blockIdx.x), extra);
  const int last = first + per + (static_cast<int>(blockIdx.x) < extra ? 1 : 0);
  int tile = first;
  if (tile < last) gather(0, tile);
  const int a = tid % G::A;
  const int o = tid / G::A;
  uint32_t* dst32 = reinterpret_cast<uint32_t*>(args.packed);
  uint4 carry[PG::runs_per_thread];
#pragma unroll
  for (int k = 0; k < PG::runs_per_thread; ++k) carry[k] = make_uint4(0u, 0u, 0u, 0u);

  for (int j = 0; tile < last; ++j, ++tile) {
    const int s = j & 1;
    const int next = tile + 1;
    if (next < last) {
      gather(s ^ 1, next);
      asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    }
    __syncthreads();
    const TmaTile t = bulk_tile<G::TT>(args, tile);

    uint32_t x[8][4];
    {
      const int phys = (o + a) & (G::O - 1);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 v = *reinterpret_cast<const uint4*>(smem + s * PG::stage_bytes + (8 * a + i) * (D * 2) + phys * 16);
        x[i][0] = v.x;
        x[i][1] = v.y;
        x[i][2] = v.z;
        x[i][3] = v.w;
      }
    }
#pragma unroll
    for (int p = 0; p < G::P; ++p) {
      uint32_t lo[8], hi[8];
      if constexpr (MODE == kModeByte2) {
        const uint32_t sel = p == 0 ? 0x7531u : 0x6420u;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          lo[i] = prmt(x[i][0], x[i][1], sel);
          hi[i] = prmt(x[i][2], x[i][3], sel);
        }
      } else {
        const int sh = G::shift(p);
        const uint32_t m = (1u << G::bits(p)) - 1u;
        const uint32_t m2 = m | (m << 16);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          lo[i] = prmt((x[i][0] >> sh) & m2, (x[i][1] >> sh) & m2, 0x6420);
          hi[i] = prmt((x[i][2] >> sh) & m2, (x[i][3] >> sh) & m2, 0x6420);
        }
      }
      transpose8x8(lo, hi);
      const int b = G::bits(p);
      uint8_t* pbase = out_sm + PG::plane_off(p);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        uint8_t* row = pbase + (8 * o + jj) * PG::rs(p);
        if (b == 8) {
          *reinterpret_cast<uint2*>(row + 8 * a) = make_uint2(lo[jj], hi[jj]);
        } else {
          const uint64_t v = gather8(lo[jj], hi[jj], b);
#pragma unroll
          for (int q = 0; q < b; ++q) row[a * b + q] = static_cast<uint8_t>(v >> (8 * q));
        }
      }
    }
    __syncthreads();
    const int64_t job_base = static_cast<int64_t>(t.job) * args.job_stride;
    const bool cont_prev = tile > first && t.t0 > 0;
    const bool cont_next = tile + 1 < last && t.t0 + G::TT < args.T;
    // Edge vectors of every run: one thread per run, so the carry stays in its registers.
#pragma unroll
    for (int k = 0; k < PG::runs_per_thread; ++k) {
      const int r = tid + k * kThreads;
      if (r >= G::P * D) break;
      const int p = r / D;
      const int c = r - p * D;
      const int b = G::bits(p);
      const int len = t.n * b;
      const int64_t B = (job_base + args.comp_base[t.kv * G::P + p]) * 8 +
                        (static_cast<int64_t>(t.h) * D + c) * args.T * b + t.t0 * b;
      const int off = static_cast<int>(B & 127);
      const int vl = (off + len - 1) >> 7;
      const uint32_t* src = reinterpret_cast<const uint32_t*>(out_sm + PG::plane_off(p) + c * PG::rs(p));
      const uint4 cin = carry[k];
      for (int e = 0; e <= vl; e += max(vl, 1)) {
        const int rel = (e << 7) - off;
        if (rel >= 0 && rel + 128 <= len) continue;  // interior: whole store below
        uint32_t w[4], m[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) run_word(src, rel + 32 * q, len, w[q], m[q]);
        if (e == 0 && off != 0 && cont_prev) {
          w[0] |= cin.x;
          w[1] |= cin.y;
          w[2] |= cin.z;
          w[3] |= cin.w;
#pragma unroll
          for (int q = 0; q < 4; ++q) m[q] |= bit_range_mask(0, min(max(off - 32 * q, 0), 32));
        }
        if (rel + 128 > len && cont_next) {
          carry[k] = make_uint4(w[0], w[1], w[2], w[3]);
          continue;
        }
        uint32_t* dst = dst32 + 4 * ((B >> 7) + e);
        if ((m[0] & m[1] & m[2] & m[3]) == 0xFFFFFFFFu) {
          st_global_cs16(dst, make_uint4(w[0], w[1], w[2], w[3]));
          continue;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (m[q] == 0xFFFFFFFFu) {
            dst[q] = w[q];
          } else if (m[q] != 0u) {
            atomicAnd(dst + q, ~m[q]);
            atomicOr(dst + q, w[q]);
          }
        }
      }
    }
    // Interior vectors: whole 16-byte stores.
#pragma unroll
    for (int p = 0; p < G::P; ++p) {
      const int b = G::bits(p);
      const int Vmax = ((G::TT * b + 127) >> 7) + 1;
      const int len = t.n * b;
      const int64_t comp = (job_base + args.comp_base[t.kv * G::P + p]) * 8;
      for (int i = tid; i < D * Vmax; i += kThreads) {
        const int c = i / Vmax;
        const int v = i - c * Vmax;
        const int64_t B = comp + (static_cast<int64_t>(t.h) * D + c) * args.T * b + t.t0 * b;
        const int rel = (v << 7) - static_cast<int>(B & 127);
        if (rel < 0 || rel + 128 > len) continue;
        const uint32_t* src = reinterpret_cast<const uint32_t*>(out_sm + PG::plane_off(p) + c * PG::rs(p));
        const int q = rel >> 5;
        const int r = rel & 31;
        uint4 w;
        if (r == 0) {
          if ((q & 3) == 0) w = *reinterpret_cast<const uint4*>(src + q);
          else w = make_uint4(src[q], src[q + 1], src[q + 2], src[q + 3]);
        } else {
          uint32_t sw[5];
          words5(src, q, sw);
          w = make_uint4(__funnelshift_r(sw[0], sw[1], r), __funnelshift_r(sw[1], sw[2], r),
                         __funnelshift_r(sw[2], sw[3], r), __funnelshift_r(sw[3], sw[4], r));
        }
        st_global_cs16(dst32 + 4 * ((B >> 7) + v), w);
      }
    }
    __syncthreads();  // out_sm and stage s free for the next tile
  }
}

}  // namespace origami
