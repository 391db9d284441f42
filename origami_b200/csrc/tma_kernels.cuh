// Persistent, double-buffered tile kernels for the aligned plane format.
//
// Aligned format: every chunk spans all T tokens, the chunks of each (kv, plane)
// component are contiguous in canonical (head, channel) order, and T*bits is a multiple
// of 128 for every plane. Then component q is a dense 2-D byte array
// [H*D runs][T*bits/8 bytes] starting at offsets[q*S], and the runs of one tile (head h,
// tokens [t0, t0+TT)) are the box {TT*bits/8 bytes, D runs} at (t0*bits/8, h*D): one TMA
// copy per plane and tile.
//
// restore_tma: TMA 2-D loads of the packed runs (mbarrier completion, two stages: the
//   next tile's runs load while this one is transposed) -> 8x8 byte transposes + plane
//   merge in registers -> token rows in shared memory (16-byte chunks rotated by token
//   octet) -> 16-byte streaming stores through the block table.
// pack_tma: cp.async gather of the next tile's token rows (two stages) -> split +
//   transpose in registers -> dense packed runs in shared memory -> TMA 2-D stores.
//
// Every mbarrier wait is bounded; a CTA whose wait runs out flags bit 31 of the error
// word, waits once more (bounded) for its copies and returns. All threads agree on
// the outcome through __syncthreads_or, so no thread is left at a barrier.
#pragma once

#include <cuda.h>

#include "tile_kernels.cuh"

namespace origami {

constexpr int kMaxMaps = 2 * 3;  // K and V x at most 3 planes (the presets)
constexpr int kMaxJobs = 128;    // jobs (layers / requests) per launch

// Jobs share the chunk table and cache geometry; job j's packed runs are at coordinate
// j of the 3rd tensor-map dimension, its rows in rows[j] through block_ids[j].
struct TmaArgs {
  CUtensorMap maps[kMaxMaps];  // component q = kv * P + p: {T*bits/8, H*D, jobs}
  void* rows[kMaxJobs];
  const int64_t* block_ids[kMaxJobs];
  int64_t kv_stride, block_stride, token_stride, head_stride;
  int64_t block_size, num_blocks;
  int64_t T;
  int64_t write_tokens;  // restore: token rows below this are written (a prefix restore when < T)
  int32_t H, tiles_per_head, tiles_per_job, num_tiles;
  uint32_t* err;
};

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                             const void* smem_src) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3}], [%4];\n" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z), "r"(smem_u32(smem_src))
               : "memory");
}

__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
}
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

struct TmaTile {
  int job, kv, h;
  int64_t t0;
  int n;
};

template <int TT>
__device__ __forceinline__ TmaTile tma_tile(const TmaArgs& a, int tile) {
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

// Row offsets (elements) of a tile's token rows, -1 for rows whose block id is invalid.
template <int TT>
__device__ __forceinline__ void tma_rowoff(const TmaArgs& a, const TmaTile& t, int64_t* rowoff) {
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

// The same offsets in two halves, so the block-table loads of the next tile overlap the
// current tile's work: rowoff_load issues them into registers, rowoff_store writes
// them to shared memory later (-2 marks an invalid block id until it is counted there).
template <int TT>
struct RowoffRegs {
  static constexpr int kPer = (TT + kThreads - 1) / kThreads;
  int64_t v[kPer];
};

template <int TT, typename Args, typename Tile>
__device__ __forceinline__ void rowoff_load(const Args& a, const Tile& t, RowoffRegs<TT>& r) {
  const int32_t bs = static_cast<int32_t>(a.block_size);
#pragma unroll
  for (int k = 0; k < RowoffRegs<TT>::kPer; ++k) {
    const int i = static_cast<int>(threadIdx.x) + k * kThreads;
    int64_t off = -1;
    if (i < TT && i < t.n && t.t0 + i < a.write_tokens) {
      const int32_t tg = static_cast<int32_t>(t.t0) + i;
      const int32_t bi = tg / bs;
      const int64_t blk = a.block_ids[t.job][bi];
      off = (blk < 0 || blk >= a.num_blocks)
                ? -2
                : t.kv * a.kv_stride + blk * a.block_stride + static_cast<int64_t>(tg - bi * bs) * a.token_stride +
                      static_cast<int64_t>(t.h) * a.head_stride;
    }
    r.v[k] = off;
  }
}

template <int TT>
__device__ __forceinline__ void rowoff_store(uint32_t* err, RowoffRegs<TT>& r, int64_t* rowoff) {
#pragma unroll
  for (int k = 0; k < RowoffRegs<TT>::kPer; ++k) {
    const int i = static_cast<int>(threadIdx.x) + k * kThreads;
    if (i < TT) {
      if (r.v[k] == -2) {
        if (err) atomicAdd(err, 1u);
        r.v[k] = -1;
      }
      rowoff[i] = r.v[k];
    }
  }
}

template <int MODE, int D>
struct TmaGeo {
  static constexpr int TT = tile_tokens_for(D);
  static constexpr int A = TT / 8;
  static constexpr int O = D / 8;
  static constexpr int P = MODE == kModeByte2 ? 2 : 3;
  __host__ __device__ static constexpr int bits(int p) {
    return MODE == kModeByte2 ? 8
           : MODE == kModeBf16Bits ? (p == 0 ? 8 : (p == 1 ? 1 : 7))
                                   : (p == 0 ? 6 : (p == 1 ? 2 : 8));
  }
  __host__ __device__ static constexpr int shift(int p) {
    return MODE == kModeByte2 ? (p == 0 ? 8 : 0)
           : MODE == kModeBf16Bits ? (p == 0 ? 7 : (p == 1 ? 15 : 0))
                                   : (p == 0 ? 10 : (p == 1 ? 8 : 0));
  }
  __host__ __device__ static constexpr int run_bytes(int p) { return TT * bits(p) / 8; }
  __host__ __device__ static constexpr int plane_off(int p) {
    return p == 0 ? 0 : (p == 1 ? D * run_bytes(0) : D * (run_bytes(0) + run_bytes(1)));
  }
  static constexpr int in_bytes = D * 2 * TT;        // all planes of one tile (16 bits per element)
  static constexpr int rows_bytes = TT * D * 2;       // token rows of one tile
  static constexpr int rowoff_bytes = TT * 8;
  static constexpr int stage_bytes = in_bytes + rowoff_bytes;
  // [stage 0][stage 1][token rows][2 mbarriers] + 128 bytes of alignment slack
  static constexpr int smem_bytes = 2 * stage_bytes + rows_bytes + 16 + 128;
};

// Phase B of the restore kernels: thread (a, o) merges the planes of tokens 8a..8a+7 x
// channels 8o..8o+7 of one staged tile into out[token][4 words] (8 16-bit elements).
template <int MODE, int D>
__device__ __forceinline__ void tma_merge(const uint8_t* stage, int a, int o, uint32_t (&out)[8][4]) {
  using G = TmaGeo<MODE, D>;
  uint32_t keep_lo[8], keep_hi[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i][0] = out[i][1] = out[i][2] = out[i][3] = 0u;
#pragma unroll
  for (int p = 0; p < G::P; ++p) {
    const int bits = G::bits(p);
    const int rb = G::run_bytes(p);
    const uint8_t* pbase = stage + G::plane_off(p);
    uint32_t lo[8], hi[8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const uint8_t* row = pbase + (8 * o + jj) * rb;
      if (bits == 8) {
        const uint2 v = *reinterpret_cast<const uint2*>(row + 8 * a);
        lo[jj] = v.x;
        hi[jj] = v.y;
      } else {
        // 8 symbols = `bits` bytes at byte a*bits (runs are 16-byte aligned rows)
        uint32_t v0, v1;
        window64(row, 8 * a * bits, v0, v1);
        spread8_rt(v0, v1, bits, lo[jj], hi[jj]);
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
}

// ---------------------------------------------------------------------------------------
// restore_tma
// ---------------------------------------------------------------------------------------
template <int MODE, int D>
__global__ void __launch_bounds__(kThreads) restore_tma(const __grid_constant__ TmaArgs args) {
  using G = TmaGeo<MODE, D>;
  extern __shared__ __align__(128) uint8_t tma_smem[];
  // 128-byte aligned base for the TMA destinations (the launch adds 128 bytes of slack).
  uint8_t* smem = tma_smem + ((128 - (smem_u32(tma_smem) & 127)) & 127);
  uint8_t* rows_sm = smem + 2 * G::stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(rows_sm + G::rows_bytes);
  const int tid = threadIdx.x;

  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // The next tile's runs come by TMA; its block-table rows are loaded into registers here
  // and written to its stage after the current tile's work (rowoff_store).
  RowoffRegs<G::TT> next_rows;
  auto issue = [&](int s, int tile) {
    const TmaTile t = tma_tile<G::TT>(args, tile);
    if (tid == 0) {
      mbar_expect_tx(&bars[s], G::in_bytes);
#pragma unroll
      for (int p = 0; p < G::P; ++p) {
        tma_load_3d(smem + s * G::stage_bytes + G::plane_off(p), &args.maps[t.kv * G::P + p],
                    static_cast<int32_t>(t.t0 * G::bits(p) / 8), t.h * D, t.job, &bars[s]);
      }
    }
    rowoff_load<G::TT>(args, t, next_rows);
  };

  int tile = blockIdx.x;
  if (tile < args.num_tiles) {
    issue(0, tile);
    rowoff_store<G::TT>(args.err, next_rows, reinterpret_cast<int64_t*>(smem + G::in_bytes));
  }
  uint32_t phases = 0u;  // bit s = parity to wait for on stage s
  const int a = tid % G::A;
  const int o = tid / G::A;

  for (int j = 0; tile < args.num_tiles; ++j, tile += gridDim.x) {
    const int s = j & 1;
    const int next = tile + gridDim.x;
    if (next < args.num_tiles) issue(s ^ 1, next);
    if (stage_wait_or_bail(&bars[s], (phases >> s) & 1u, &bars[s ^ 1], (phases >> (s ^ 1)) & 1u,
                           next < args.num_tiles, args.err))
      return;
    phases ^= 1u << s;
    const TmaTile t = tma_tile<G::TT>(args, tile);
    uint8_t* rows = static_cast<uint8_t*>(args.rows[t.job]);

    // Phase B: 8 tokens x 8 channels per thread, planes merged in registers.
    uint32_t out[8][4];
    tma_merge<MODE, D>(smem + s * G::stage_bytes, a, o, out);
    // Token rows to shared memory (the previous tile's phase C finished at the loop-end barrier).
    const int phys = (o + a) & (G::O - 1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      *reinterpret_cast<uint4*>(rows_sm + (8 * a + i) * (D * 2) + phys * 16) =
          make_uint4(out[i][0], out[i][1], out[i][2], out[i][3]);
    }
    __syncthreads();
    // Phase C: rows to the paged cache.
    const int64_t* rowoff = reinterpret_cast<const int64_t*>(smem + s * G::stage_bytes + G::in_bytes);
    const int oc = tid % G::O;
    for (int r = tid / G::O; r < t.n; r += kThreads / G::O) {
      const int64_t off = rowoff[r];
      if (off < 0) continue;
      st_global_cs16(rows + (off + 8 * oc) * 2,
                     *reinterpret_cast<const uint4*>(rows_sm + r * (D * 2) + ((oc + (r >> 3)) & (G::O - 1)) * 16));
    }
    if (next < args.num_tiles)
      rowoff_store<G::TT>(args.err, next_rows, reinterpret_cast<int64_t*>(smem + (s ^ 1) * G::stage_bytes + G::in_bytes));
    __syncthreads();  // stage s and the row buffer are free again; stage s ^ 1's rows are written
  }
}

// ---------------------------------------------------------------------------------------
// pack_tma
// ---------------------------------------------------------------------------------------
template <int MODE, int D>
struct PackGeo {
  using G = TmaGeo<MODE, D>;
  static constexpr int rows_bytes = G::TT * D * 2;  // token rows of one tile (per stage)
  static constexpr int rowoff_bytes = G::TT * 8;
  static constexpr int stage_bytes = rows_bytes + rowoff_bytes;
  static constexpr int out_bytes = G::in_bytes;     // packed runs of one tile
  static constexpr int smem_bytes = 2 * stage_bytes + out_bytes + 128;
};

template <int MODE, int D>
__global__ void __launch_bounds__(kThreads) pack_tma(const __grid_constant__ TmaArgs args) {
  using G = TmaGeo<MODE, D>;
  using PG = PackGeo<MODE, D>;
  extern __shared__ __align__(128) uint8_t tma_smem[];
  uint8_t* smem = tma_smem + ((128 - (smem_u32(tma_smem) & 127)) & 127);
  uint8_t* out_sm = smem + 2 * PG::stage_bytes;
  const int tid = threadIdx.x;

  // Gather a tile's token rows with cp.async (8-channel chunks rotated by token octet).
  auto gather = [&](int s, int tile) {
    const TmaTile t = tma_tile<G::TT>(args, tile);
    const uint8_t* rows = static_cast<const uint8_t*>(args.rows[t.job]);
    uint8_t* sb = smem + s * PG::stage_bytes;
    int64_t* rowoff = reinterpret_cast<int64_t*>(sb + PG::rows_bytes);
    tma_rowoff<G::TT>(args, t, rowoff);
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

  int tile = blockIdx.x;
  if (tile < args.num_tiles) gather(0, tile);
  const int a = tid % G::A;
  const int o = tid / G::A;

  for (int j = 0; tile < args.num_tiles; ++j, tile += gridDim.x) {
    const int s = j & 1;
    const int next = tile + gridDim.x;
    if (next < args.num_tiles) {
      gather(s ^ 1, next);
      asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    }
    __syncthreads();
    const TmaTile t = tma_tile<G::TT>(args, tile);

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
    // The previous tile's TMA stores must have read the output buffer.
    if (tid == 0) tma_store_wait_read();
    __syncthreads();
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
        constexpr uint32_t dummy = 0;
        (void)dummy;
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
      const int bits = G::bits(p);
      const int rb = G::run_bytes(p);
      uint8_t* pbase = out_sm + G::plane_off(p);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        uint8_t* row = pbase + (8 * o + jj) * rb;
        if (bits == 8) {
          *reinterpret_cast<uint2*>(row + 8 * a) = make_uint2(lo[jj], hi[jj]);
        } else {
          const uint64_t v = gather8(lo[jj], hi[jj], bits);
#pragma unroll
          for (int q = 0; q < bits; ++q) row[a * bits + q] = static_cast<uint8_t>(v >> (8 * q));
        }
      }
    }
    fence_async_shared();
    __syncthreads();
    if (tid == 0) {
#pragma unroll
      for (int p = 0; p < G::P; ++p) {
        tma_store_3d(&args.maps[t.kv * G::P + p], static_cast<int32_t>(t.t0 * G::bits(p) / 8), t.h * D, t.job,
                     out_sm + G::plane_off(p));
      }
      tma_store_commit();
    }
  }
  if (tid == 0) tma_store_wait_all();
}

}  // namespace origami
