// Persistent layer kernels for the contiguous plane format, head_dim 128 / 256.
//
// Contiguous plane format: every chunk spans all T tokens and the chunks of each (kv,
// plane) component are contiguous in canonical (head, channel) order, so run (q, h, c)
// of job j starts at byte j*job_stride + comp_base[q] + (h*D + c)*T*bits/8. A tile is
// (job, kv, head h, a token range) x all D channels; thread (a, o) owns tokens 8a..8a+7 x
// channels 8o..8o+7 (one 8x8 block of 16-bit elements).
//
// restore_rows<MODE, D, RAGGED> (every plane preset)
//   aligned runs (T*bits a multiple of 128): one TMA tensor copy per plane and tile;
//     round-robin tiles (the CTAs running at once read neighbouring pieces of the same
//     runs); token rows staged in shared memory and stored as whole 256-byte rows.
//   ragged runs (any byte): one bulk copy per run of the 16-byte words covering it, each
//     warp announcing its bytes with one mbarrier arrive; a contiguous tile range per CTA
//     (the word two consecutive tiles of a run share is an L2 hit); token rows stored
//     straight from registers, three CTAs per SM.
//   Both: 64-bit bit windows -> 8x8 byte transposes + plane merge in registers.
// pack_rows<D> (byte planes, ragged runs)
//   Windows of TT token rows gathered with cp.async (two stages); each tile owns the last
//   TT - 16 of them and reads the first 16 again. Split + transpose into unshifted run
//   rows in shared memory; then each 16-byte chunk of a run's global 16-byte grid that
//   lies in the tile is realigned in registers and stored whole. Because the window
//   reaches 16 tokens back, the chunk straddling two tiles is written by the later one
//   from its own window: only the chunks at a run's two ends are partial.
//
// Every mbarrier wait is bounded (see restore_rows).
#pragma once

#include "bulk_kernels.cuh"
#include "tma_kernels.cuh"

namespace origami {

struct RowArgs {
  CUtensorMap maps[kMaxMaps];  // aligned restore: component q = kv * P + p, {T*bits/8, H*D, jobs}
  uint8_t* packed;             // job 0's packed bytes; job j at packed + j * job_stride
  int64_t job_stride;
  int64_t packed_bytes;         // from `packed` to the end of the buffer
  int64_t comp_base[kMaxMaps];  // byte offset of component q within a job
  int64_t run_bytes[4];         // T * bits(p) / 8
  void* rows[kMaxJobs];
  const int64_t* block_ids[kMaxJobs];
  int64_t kv_stride, block_stride, token_stride, head_stride;
  int64_t block_size, num_blocks;
  int64_t T;
  int64_t write_tokens;  // restore: token rows below this are written (a prefix restore when < T)
  int32_t H, tiles_per_head, tiles_per_job, num_tiles;
  uint32_t* err;
};

// Tile cursor: decoded once per CTA with divisions, then advanced by increments.
struct RowCursor {
  int job, kv, h, tt;
};

__device__ __forceinline__ RowCursor row_cursor(const RowArgs& a, int tile) {
  RowCursor c;
  c.job = tile / a.tiles_per_job;
  const int in_job = tile - c.job * a.tiles_per_job;
  const int rest = in_job / a.tiles_per_head;
  c.tt = in_job - rest * a.tiles_per_head;
  c.kv = rest / a.H;
  c.h = rest - c.kv * a.H;
  return c;
}

__device__ __forceinline__ void row_cursor_next(const RowArgs& a, RowCursor& c) {
  if (++c.tt == a.tiles_per_head) {
    c.tt = 0;
    if (++c.h == a.H) {
      c.h = 0;
      if (++c.kv == 2) {
        c.kv = 0;
        ++c.job;
      }
    }
  }
}

template <int TT>
__device__ __forceinline__ TmaTile row_tile(const RowArgs& a, const RowCursor& c) {
  TmaTile t;
  t.job = c.job;
  t.kv = c.kv;
  t.h = c.h;
  t.t0 = static_cast<int64_t>(c.tt) * TT;
  t.n = static_cast<int>(min64(TT, a.T - t.t0));
  return t;
}

// Writes the row offsets held in registers (rowoff_load) to the transposed table of
// restore_rows: token 8a + i at i * (A + 1) + a.
template <int TT>
__device__ __forceinline__ void rowoff_store_t(uint32_t* err, RowoffRegs<TT>& r, int64_t* rowoff) {
  constexpr int A = TT / 8;
#pragma unroll
  for (int k = 0; k < RowoffRegs<TT>::kPer; ++k) {
    const int i = static_cast<int>(threadIdx.x) + k * kThreads;
    if (i < TT) {
      if (r.v[k] == -2) {
        if (err) atomicAdd(err, 1u);
        r.v[k] = -1;
      }
      rowoff[(i & 7) * (A + 1) + (i >> 3)] = r.v[k];
    }
  }
}

// 16-byte words [w0, w1) of a staged run row whose bytes end past the packed buffer: the
// bytes inside the buffer, zeros after. Out of line: only the last runs of a buffer use it.
__device__ __noinline__ void ld_words_tail(uint8_t* row, const uint8_t* packed, int64_t lo16, int w0, int w1,
                                           int64_t packed_bytes) {
  for (int w = w0; w < w1; ++w) {
    const int64_t g = lo16 + 16 * w;
    uint32_t v[4] = {0u, 0u, 0u, 0u};
    for (int i = 0; i < 16; ++i) {
      if (g + i < packed_bytes) v[i >> 2] |= static_cast<uint32_t>(packed[g + i]) << (8 * (i & 3));
    }
    *reinterpret_cast<uint4*>(row + 16 * w) = make_uint4(v[0], v[1], v[2], v[3]);
  }
}

// Contiguous range of tiles of this CTA.
__device__ __forceinline__ void row_range(int num_tiles, int& first, int& last) {
  const int per = num_tiles / static_cast<int>(gridDim.x);
  const int extra = num_tiles % static_cast<int>(gridDim.x);
  const int b = static_cast<int>(blockIdx.x);
  first = b * per + min(b, extra);
  last = first + per + (b < extra ? 1 : 0);
}

// ---------------------------------------------------------------------------------------
// restore_rows
// ---------------------------------------------------------------------------------------
template <int MODE, int D, bool RAGGED>
struct RestoreRowsGeo {
  // aligned runs: token rows staged in shared memory and stored as whole rows; ragged runs
  // (larger stages): rows stored straight from registers, three CTAs per SM
  static constexpr bool STAGED = !RAGGED;
  using G = TmaGeo<MODE, D>;
  using BG = BulkGeo<MODE, D>;
  static constexpr int TT = G::TT;
  static constexpr int P = G::P;
  // run row stride: dense TMA rows, or the run's bytes plus alignment slack for bulk copies
  __host__ __device__ static constexpr int rs(int p) { return RAGGED ? BG::rs(p) : G::run_bytes(p); }
  __host__ __device__ static constexpr int plane_off(int p) { return RAGGED ? BG::plane_off(p) : G::plane_off(p); }
  static constexpr int in_bytes = RAGGED ? BG::in_bytes : G::in_bytes;
  static constexpr int rowoff_off = (in_bytes + 127) & ~127;
  // row offsets stored transposed: token 8a + i at i * (A + 1) + a, so the 16 lanes of a
  // half-warp (consecutive a, same i) read consecutive words
  static constexpr int rowoff_entries = 8 * (G::A + 1);
  static constexpr int stage_bytes = (rowoff_off + rowoff_entries * 8 + 127) & ~127;
  // staged stores: the tile's token rows in shared memory (16-byte chunks rotated by token
  // octet), written back as whole rows
  static constexpr int rows_bytes = STAGED ? TT * D * 2 : 0;
  // [stage 0][stage 1][token rows][2 mbarriers] + 128 bytes of alignment slack
  static constexpr int smem_bytes = 2 * stage_bytes + rows_bytes + 16 + 128;
  static constexpr int runs_per_thread = (P * D + kThreads - 1) / kThreads;
};

template <int MODE, int D, bool RAGGED>
__global__ void __launch_bounds__(kThreads, RAGGED ? 3 : 2) restore_rows(const __grid_constant__ RowArgs args) {
  using RG = RestoreRowsGeo<MODE, D, RAGGED>;
  constexpr bool STAGED = RG::STAGED;
  using G = TmaGeo<MODE, D>;
  constexpr int P = G::P;
  extern __shared__ __align__(128) uint8_t rows_smem[];
  uint8_t* smem = rows_smem + ((128 - (smem_u32(rows_smem) & 127)) & 127);
  uint8_t* rows_sm = smem + 2 * RG::stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(rows_sm + RG::rows_bytes);
  const int tid = threadIdx.x;
  const int lane = tid & 31;

  // Aligned runs: tiles blockIdx.x + k * gridDim.x, so the CTAs running at once read
  // neighbouring pieces of the same runs (DRAM page locality). Ragged runs: a contiguous
  // range per CTA, so the 16-byte word two consecutive tiles of a run share is an L2 hit.
  constexpr bool rr = !RAGGED;
  int first, last;
  row_range(args.num_tiles, first, last);
  if (rr) {
    first = blockIdx.x;
    last = args.num_tiles;
  }
  if (first >= last) return;
  if (tid == 0) {
    // aligned: one arrive (thread 0 with the tile's bytes); ragged: one arrive per warp
    mbar_init(&bars[0], RAGGED ? kThreads / 32 : 1);
    mbar_init(&bars[1], RAGGED ? kThreads / 32 : 1);
    fence_mbar_init();
  }
  __syncthreads();

  RowoffRegs<RG::TT> next_rows;
  auto rowoff_at = [&](int s) { return reinterpret_cast<int64_t*>(smem + s * RG::stage_bytes + RG::rowoff_off); };

  // Load a tile's packed runs into stage s; its block-table rows go to registers and are
  // written to the stage after the current tile's work (rowoff_store).
  auto issue = [&](int s, const TmaTile& t) {
    uint8_t* sb = smem + s * RG::stage_bytes;
    if constexpr (!RAGGED) {
      if (tid == 0) {
        mbar_expect_tx(&bars[s], G::in_bytes);
#pragma unroll
        for (int p = 0; p < P; ++p) {
          tma_load_3d(sb + G::plane_off(p), &args.maps[t.kv * P + p], static_cast<int32_t>(t.t0 * G::bits(p) / 8),
                      t.h * D, t.job, &bars[s]);
        }
      }
    } else {
      const int64_t job_base = static_cast<int64_t>(t.job) * args.job_stride;
      int64_t lo16[RG::runs_per_thread];
      int32_t words[RG::runs_per_thread], full[RG::runs_per_thread];
      uint32_t bytes = 0;
#pragma unroll
      for (int k = 0; k < RG::runs_per_thread; ++k) {
        const int r = tid + k * kThreads;
        words[k] = 0;
        full[k] = 0;
        lo16[k] = 0;
        if (r < P * D) {
          const int p = r / D;
          const int c = r - p * D;
          const int b = G::bits(p);
          const int64_t start = job_base + args.comp_base[t.kv * P + p] +
                                (static_cast<int64_t>(t.h) * D + c) * args.run_bytes[p] + t.t0 * b / 8;
          const int64_t end = start + static_cast<int64_t>(t.n) * b / 8;
          lo16[k] = start & ~static_cast<int64_t>(15);
          words[k] = static_cast<int32_t>(((end + 15) >> 4) - (start >> 4));
          // words that end past the buffer are read bytewise below
          full[k] = static_cast<int32_t>(min64(words[k], max64((args.packed_bytes - lo16[k]) >> 4, 0)));
          bytes += static_cast<uint32_t>(full[k]) * 16u;
        }
      }
      // every warp announces its bytes before any of its copies is issued
      const uint32_t warp_bytes = __reduce_add_sync(0xffffffffu, bytes);
      if (lane == 0) mbar_expect_tx(&bars[s], warp_bytes);
      __syncwarp();
#pragma unroll
      for (int k = 0; k < RG::runs_per_thread; ++k) {
        const int r = tid + k * kThreads;
        if (r < P * D) {
          const int p = r / D;
          const int c = r - p * D;
          uint8_t* row = sb + RG::plane_off(p) + c * RG::rs(p);
          if (full[k] > 0) bulk_load(row, args.packed + lo16[k], static_cast<uint32_t>(full[k]) * 16u, &bars[s]);
          if (full[k] < words[k]) ld_words_tail(row, args.packed, lo16[k], full[k], words[k], args.packed_bytes);
        }
      }
    }
    rowoff_load<RG::TT>(args, t, next_rows);
  };

  RowCursor cur = row_cursor(args, first);
  TmaTile t = row_tile<RG::TT>(args, cur);
  issue(0, t);
  rowoff_store_t<RG::TT>(args.err, next_rows, rowoff_at(0));
  uint32_t phases = 0u;  // bit s = parity to wait for on stage s
  const int a = tid % G::A;
  const int o = tid / G::A;

  const int step = rr ? static_cast<int>(gridDim.x) : 1;
  for (int tile = first, j = 0;; tile += step, ++j) {
    const int s = j & 1;
    const bool has_next = tile + step < last;
    TmaTile tn = t;
    if (has_next) {
      if (rr) cur = row_cursor(args, tile + step);
      else row_cursor_next(args, cur);
      tn = row_tile<RG::TT>(args, cur);
      issue(s ^ 1, tn);
    }
    if (stage_wait_or_bail(&bars[s], (phases >> s) & 1u, &bars[s ^ 1], (phases >> (s ^ 1)) & 1u, has_next, args.err))
      return;
    phases ^= 1u << s;

    // Planes -> 8 token rows x 8 channels in registers.
    const uint8_t* sb = smem + s * RG::stage_bytes;
    uint32_t out[8][4];
    uint32_t keep_lo[8], keep_hi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i][0] = out[i][1] = out[i][2] = out[i][3] = 0u;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const int b = G::bits(p);
      // first byte of channel c's run inside its staged row: (base + c * run_bytes) mod 16
      uint32_t base16 = 0u, step16 = 0u;
      if constexpr (RAGGED) {
        base16 = static_cast<uint32_t>(static_cast<int64_t>(t.job) * args.job_stride + args.comp_base[t.kv * P + p] +
                                       static_cast<int64_t>(t.h) * D * args.run_bytes[p] + t.t0 * b / 8);
        step16 = static_cast<uint32_t>(args.run_bytes[p]);
      }
      uint32_t lo[8], hi[8];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int c = 8 * o + jj;
        const uint8_t* row = sb + RG::plane_off(p) + c * RG::rs(p);
        if constexpr (RAGGED) {
          const int pos = static_cast<int>((base16 + static_cast<uint32_t>(c) * step16) & 15u) * 8 + 8 * a * b;
          uint32_t v0, v1;
          window64(row, pos, v0, v1);
          if (b == 8) {
            lo[jj] = v0;
            hi[jj] = v1;
          } else {
            spread8_rt(v0, v1, b, lo[jj], hi[jj]);
          }
        } else if (b == 8) {
          const uint2 v = *reinterpret_cast<const uint2*>(row + 8 * a);
          lo[jj] = v.x;
          hi[jj] = v.y;
        } else {
          uint32_t v0, v1;
          window64(row, 8 * a * b, v0, v1);
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
    uint8_t* rows = static_cast<uint8_t*>(args.rows[t.job]);
    const int64_t* rowoff = rowoff_at(s);
    if constexpr (STAGED) {
      // Token rows through shared memory, then whole rows to the cache.
      const int phys = (o + a) & (G::O - 1);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        *reinterpret_cast<uint4*>(rows_sm + (8 * a + i) * (D * 2) + phys * 16) =
            make_uint4(out[i][0], out[i][1], out[i][2], out[i][3]);
      }
      __syncthreads();
      const int oc = tid % G::O;
      for (int r = tid / G::O; r < t.n; r += kThreads / G::O) {
        const int64_t off = rowoff[(r & 7) * (G::A + 1) + (r >> 3)];
        if (off < 0) continue;
        st_global_cs16(rows + (off + 8 * oc) * 2,
                       *reinterpret_cast<const uint4*>(rows_sm + r * (D * 2) + ((oc + (r >> 3)) & (G::O - 1)) * 16));
      }
    } else {
      // Token rows straight to the cache: lanes (a, o) and (a, o + 1) write one 32-byte sector.
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t off = rowoff[i * (G::A + 1) + a];
        if (off >= 0)
          st_global_cs16(rows + (off + 8 * o) * 2, make_uint4(out[i][0], out[i][1], out[i][2], out[i][3]));
      }
    }
    if (!has_next) break;
    rowoff_store_t<RG::TT>(args.err, next_rows, rowoff_at(s ^ 1));
    __syncthreads();  // stage s free again; stage s ^ 1's block-table rows written
    t = tn;
  }
}

// ---------------------------------------------------------------------------------------
// pack_rows (byte planes: plane 0 = high byte, plane 1 = low byte)
// ---------------------------------------------------------------------------------------
template <int D>
struct PackRowsGeo {
  using G = TmaGeo<kModeByte2, D>;
  static constexpr int TT = G::TT;                // tokens of a tile's window
  static constexpr int LOOK = 16;                 // of which the first LOOK were the tile before's
  static constexpr int STEP = TT - LOOK;          // tokens a tile owns
  static constexpr int rows_bytes = TT * D * 2;   // token rows of one window
  static constexpr int stage_bytes = rows_bytes + TT * 8;
  // one row per (plane, channel): the window's TT bytes of the run + 16 bytes of slack (a
  // realigned 16-byte output chunk reads 32 aligned bytes)
  static constexpr int rs = TT + 16;
  static constexpr int out_bytes = 2 * D * rs;
  // [stage 0][stage 1][run rows] + 128 bytes of alignment slack (two CTAs per SM: measured
  // faster than three CTAs with the run rows written over the consumed stage)
  static constexpr int smem_bytes = 2 * stage_bytes + out_bytes + 128;
  static constexpr int chunks = STEP / 16;       // output chunks a tile writes (one more at a run's end)
  // (plane, channel mod 16) misalignment classes per warp
  static constexpr int classes_per_warp = 32 / (kThreads / 32);
};

// 16-byte cp.async that zero-fills the destination when src_bytes is 0.
__device__ __forceinline__ void cp_async16_zfill(void* smem_dst, const void* gmem_src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem_dst)), "l"(gmem_src),
               "r"(src_bytes)
               : "memory");
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// Bytes [lo, hi) of the 16-byte chunk v to the 16-byte aligned global chunk p, as naturally
// aligned 1/2/4/8-byte stores (bytes outside the range belong to a neighbouring tile or run).
__device__ __forceinline__ void st_range16(uint8_t* p, const uint4& v, int lo, int hi) {
  int k = lo;
  if ((k & 1) && k < hi) {
    p[k] = static_cast<uint8_t>(word_of(v, k >> 2) >> (8 * (k & 3)));
    k += 1;
  }
  if ((k & 2) && k + 2 <= hi) {
    *reinterpret_cast<uint16_t*>(p + k) = static_cast<uint16_t>(word_of(v, k >> 2) >> (8 * (k & 3)));
    k += 2;
  }
  if ((k & 4) && k + 4 <= hi) {
    *reinterpret_cast<uint32_t*>(p + k) = word_of(v, k >> 2);
    k += 4;
  }
  if (k + 8 <= hi) {
    *reinterpret_cast<uint2*>(p + k) = make_uint2(word_of(v, k >> 2), word_of(v, (k >> 2) + 1));
    k += 8;
  }
  if (k + 4 <= hi) {
    *reinterpret_cast<uint32_t*>(p + k) = word_of(v, k >> 2);
    k += 4;
  }
  if (k + 2 <= hi) {
    *reinterpret_cast<uint16_t*>(p + k) = static_cast<uint16_t>(word_of(v, k >> 2) >> (8 * (k & 3)));
    k += 2;
  }
  if (k < hi) p[k] = static_cast<uint8_t>(word_of(v, k >> 2) >> (8 * (k & 3)));
}

// 16 bytes starting at byte 16 - m (m in 0..15) of the 32-byte little-endian window
// (a, b): m is the same for the whole warp, so the switch does not diverge.
__device__ __forceinline__ uint4 realign16(const uint4& a, const uint4& b, int m) {
  const int k = 16 - m;
  const uint32_t sel = 0x3210u + 0x1111u * static_cast<uint32_t>(k & 3);
  switch (k >> 2) {
    case 0: return make_uint4(prmt(a.x, a.y, sel), prmt(a.y, a.z, sel), prmt(a.z, a.w, sel), prmt(a.w, b.x, sel));
    case 1: return make_uint4(prmt(a.y, a.z, sel), prmt(a.z, a.w, sel), prmt(a.w, b.x, sel), prmt(b.x, b.y, sel));
    case 2: return make_uint4(prmt(a.z, a.w, sel), prmt(a.w, b.x, sel), prmt(b.x, b.y, sel), prmt(b.y, b.z, sel));
    case 3: return make_uint4(prmt(a.w, b.x, sel), prmt(b.x, b.y, sel), prmt(b.y, b.z, sel), prmt(b.z, b.w, sel));
    default: return b;
  }
}

template <int D>
__global__ void __launch_bounds__(kThreads, 2) pack_rows(const __grid_constant__ RowArgs args) {
  using PG = PackRowsGeo<D>;
  using G = TmaGeo<kModeByte2, D>;
  constexpr int TT = G::TT;
  constexpr int A = G::A;
  constexpr int O = G::O;
  constexpr int U = D / 16;  // channels of one misalignment class per plane
  extern __shared__ __align__(128) uint8_t rows_smem[];
  uint8_t* smem = rows_smem + ((128 - (smem_u32(rows_smem) & 127)) & 127);
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t T = args.T;
  // tiles blockIdx.x + k * gridDim.x: the CTAs running at once write neighbouring pieces
  // of the same runs
  const int step = static_cast<int>(gridDim.x);
  const int first = static_cast<int>(blockIdx.x);
  if (first >= args.num_tiles) return;
  // tile tt of a (job, kv, head) owns tokens [tt * STEP, tt * STEP + STEP); its window
  // starts LOOK tokens earlier
  auto tile_at = [&](int tile) {
    const RowCursor c = row_cursor(args, tile);
    TmaTile t;
    t.job = c.job;
    t.kv = c.kv;
    t.h = c.h;
    t.t0 = static_cast<int64_t>(c.tt) * PG::STEP;
    t.n = static_cast<int>(min64(PG::STEP, T - t.t0));
    return t;
  };

  auto rowoff_at = [&](int s) { return reinterpret_cast<int64_t*>(smem + s * PG::stage_bytes + PG::rows_bytes); };
  auto fill_rowoff = [&](int s, const TmaTile& t) {
    int64_t* ro = rowoff_at(s);
    const int32_t bs = static_cast<int32_t>(args.block_size);
    for (int i = tid; i < TT; i += kThreads) {
      const int64_t tok = t.t0 - PG::LOOK + i;
      int64_t off = -1;
      if (tok >= 0 && tok < T) {
        const int32_t tg = static_cast<int32_t>(tok);
        const int32_t bi = tg / bs;
        const int64_t blk = args.block_ids[t.job][bi];
        if (blk < 0 || blk >= args.num_blocks) {
          if (args.err && i >= PG::LOOK) atomicAdd(args.err, 1u);  // counted by the tile that owns the token
        } else {
          off = t.kv * args.kv_stride + blk * args.block_stride + static_cast<int64_t>(tg - bi * bs) * args.token_stride +
                static_cast<int64_t>(t.h) * args.head_stride;
        }
      }
      ro[i] = off;
    }
  };
  // cp.async gather of a window's token rows (16-byte chunks rotated by token octet);
  // rows outside the run or with an invalid block id are zero-filled.
  auto gather = [&](int s, const TmaTile& t) {
    const uint8_t* rows = static_cast<const uint8_t*>(args.rows[t.job]);
    uint8_t* sb = smem + s * PG::stage_bytes;
    const int64_t* ro = rowoff_at(s);
    const int oc = tid % O;
#pragma unroll
    for (int r = tid / O; r < TT; r += kThreads / O) {
      const int64_t off = ro[r];
      uint8_t* dst = sb + r * (D * 2) + ((oc + (r >> 3)) & (O - 1)) * 16;
      cp_async16_zfill(dst, off < 0 ? rows : rows + (off + 8 * oc) * 2, off < 0 ? 0u : 16u);
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };

  TmaTile t = tile_at(first);
  fill_rowoff(0, t);
  __syncthreads();
  gather(0, t);
  TmaTile tn = t;
  if (first + step < args.num_tiles) {
    tn = tile_at(first + step);
    fill_rowoff(1, tn);
  }
  const int a = tid % A;
  const int o = tid / A;

  for (int tile = first, j = 0;; tile += step, ++j) {
    const int s = j & 1;
    const bool has_next = tile + step < args.num_tiles;
    __syncthreads();  // run rows and stage s ^ 1 free; stage s ^ 1's block-table rows written
    if (has_next) {
      gather(s ^ 1, tn);
      asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    }
    __syncthreads();  // stage s rows visible

    // Split + transpose: the window's bytes of every run into its row, unshifted.
    uint8_t* out_sm = smem + 2 * PG::stage_bytes;
    const uint8_t* in_sm = smem + s * PG::stage_bytes;
    uint32_t x[8][4];
    {
      const int phys = (o + a) & (O - 1);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 v = *reinterpret_cast<const uint4*>(in_sm + (8 * a + i) * (D * 2) + phys * 16);
        x[i][0] = v.x;
        x[i][1] = v.y;
        x[i][2] = v.z;
        x[i][3] = v.w;
      }
    }
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      uint32_t lo[8], hi[8];
      const uint32_t sel = p == 0 ? 0x7531u : 0x6420u;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        lo[i] = prmt(x[i][0], x[i][1], sel);
        hi[i] = prmt(x[i][2], x[i][3], sel);
      }
      transpose8x8(lo, hi);
      uint8_t* prow = out_sm + (p * D + 8 * o) * PG::rs + 8 * a;
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) *reinterpret_cast<uint2*>(prow + jj * PG::rs) = make_uint2(lo[jj], hi[jj]);
    }
    __syncthreads();  // run rows complete

    // Stores. Run (p, c)'s owned piece starts at global byte g = base_p + c * T; m = g mod
    // 16 depends, for a plane, only on c mod 16 (heads and tiles are multiples of 16 bytes
    // apart), so warp w takes the classes (p, k = c mod 16) numbered [4w, 4w + 4), U
    // channels each. Output chunk q (the run's global 16-byte grid) holds the run's
    // tokens [t0 - m + 16q, t0 - m + 16q + 16), i.e. window bytes [16 - m + 16q, ...): the
    // chunk before the piece reaches back into the window's first LOOK tokens, and the
    // chunk the piece ends in is the next tile's chunk 0. So every chunk is written whole
    // by one tile; only the chunks at a run's two ends are partial.
    const int64_t job_base = static_cast<int64_t>(t.job) * args.job_stride;
    const int64_t head_base = static_cast<int64_t>(t.h) * D * T + t.t0;
    const bool last = t.t0 + PG::STEP >= T;  // the run's last tile also writes chunk `chunks`
#pragma unroll
    for (int cls = 0; cls < PG::classes_per_warp; ++cls) {
      const int pk = warp * PG::classes_per_warp + cls;
      const int p = pk >> 4;
      const int k = pk & 15;
      const int64_t base = job_base + args.comp_base[t.kv * 2 + p] + head_base + k * T;  // channel k
      const int m = static_cast<int>(base & 15);
      const uint8_t* rows0 = out_sm + (p * D + k) * PG::rs;
      uint8_t* dst0 = args.packed + (base - m);
#pragma unroll
      for (int r0 = 0; r0 < U; r0 += 4) {
        const int u = r0 + (lane >> 3);
        const int q = lane & 7;
        const int64_t tok = t.t0 - m + 16 * q;  // first token of chunk q
        if ((q < PG::chunks || (q == PG::chunks && last)) && tok < T) {
          const uint8_t* row = rows0 + 16 * u * PG::rs + 16 * q;
          const uint4 v = realign16(*reinterpret_cast<const uint4*>(row), *reinterpret_cast<const uint4*>(row + 16), m);
          uint8_t* dst = dst0 + 16 * u * T + 16 * q;
          if (tok >= 0 && tok + 16 <= T) st_global_cs16(dst, v);
          else st_range16(dst, v, tok < 0 ? static_cast<int>(-tok) : 0, static_cast<int>(min64(16, T - tok)));
        }
      }
    }
    if (!has_next) break;
    if (tile + 2 * step < args.num_tiles) {
      // block-table rows of tile + 2 steps into stage s (its rows are read above, its
      // row-offset table is not)
      const TmaTile t2 = tile_at(tile + 2 * step);
      fill_rowoff(s, t2);
      t = tn;
      tn = t2;
    } else {
      t = tn;
    }
  }
}

}  // namespace origami
