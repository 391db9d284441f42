// Tile kernels: canonical chunk streams <-> token-major rows.
//
// A tile is (kv, head h, tokens [t0, t0 + TT)) x all D channels. On the packed side every
// (plane p, channel c) of the tile is one contiguous run of TT symbols inside the chunk
// that covers (h, c): Origami's canonical order is head > channel > token
// (csrc/origami/bitpack_layout_cuda.cu:115-124) with dense LSB-first symbols
// (bitpack_layout_cuda.cu:70-89). On the row side a token's D channels are contiguous
// (paged KV cache rows, or a [.., head, head_dim]-innermost uint8 symbol tensor).
//
// restore_tiles: packed runs -(cp.async)-> smem rows [p][c][bits] -> 8x8 byte transposes
//   in registers -> plane merge -> smem rows [t][c] (16-byte chunks rotated by token octet,
//   bank-conflict free) -> 16-byte streaming stores into the destination rows.
// pack_tiles: the inverse. Fully owned, aligned 16-byte vectors of a run are stored
//   whole; 32-bit words a run shares with its neighbour are merged with masked atomics,
//   so any bit alignment (ragged token counts, odd bit widths) is exact without a
//   zero-fill pass.
//
// Template parameters: ELEM (row element bytes: 2 = bf16/fp16 cache, 1 = uint8 symbols),
// MODE (plane preset with compile-time shifts and widths, or generic), DT (head_dim when
// it is 64/128/256 so every index division folds to shifts; 0 = runtime head_dim).
#pragma once

#include "common.cuh"

namespace origami {

enum PlaneMode : int {
  kModeGeneric = 0,  // runtime planes (and per-chunk bits for canonical ops)
  kModeByte2 = 1,    // 16-bit element -> hi byte (shift 8) + lo byte (shift 0)
  kModeBf16Bits = 2, // bf16 -> exponent (7,8), sign (15,1), mantissa (0,7)
  kModeFp16Bits = 3  // fp16 -> sign+exponent (10,6), mantissa high (8,2), mantissa low (0,8)
};

struct RowMeta {
  int64_t a;  // restore: 16-byte aligned start byte of the run (-1 = no chunk covers it)
              // pack:    first destination bit of the run (-1 = not covered)
  int32_t b;  // restore: 16-byte words to load;  pack: destination bit count incl. pad
  int32_t c;  // restore: (bits << 16) | first bit inside the loaded row;  pack: bits
};

struct TileArgs {
  // Row side: element (kv, t, h, c) lives at
  //   kv*kv_stride + blk*block_stride + (t % block_size)*token_stride + h*head_stride + c
  // with blk = block_ids[t / block_size] (or t / block_size when block_ids is null).
  void* rows;
  int64_t kv_stride, block_stride, token_stride, head_stride;
  int64_t block_size, num_blocks;
  const int64_t* block_ids;
  // Packed side.
  uint8_t* packed;
  int64_t packed_bytes;
  const int64_t* specs;       // [S][6]
  const int64_t* offsets;     // [num_kv * P * S + 1]
  const int64_t* chunk_bits;  // per chunk bits (canonical ops) or null (plane bits)
  int32_t S;
  // Geometry.
  int32_t num_kv, H, D;
  int64_t T;
  int64_t write_tokens;  // restore: token rows below this are written (a prefix restore when < T)
  int32_t TT, tiles_per_head;
  // Planes (bits[p] is the widest chunk's width when chunk_bits is set).
  int32_t P;
  int32_t shift[8];
  int32_t bits[8];
  // Shared memory layout (bytes from the start of dynamic shared memory).
  int32_t rowoff_off, meta_off, data_off;
  uint32_t* err;
};

template <int MODE>
__device__ __forceinline__ int mode_planes(const TileArgs& a) {
  if constexpr (MODE == kModeByte2) return 2;
  else if constexpr (MODE == kModeBf16Bits || MODE == kModeFp16Bits) return 3;
  else return a.P;
}

template <int MODE>
__device__ __forceinline__ int mode_shift(const TileArgs& a, int p) {
  if constexpr (MODE == kModeByte2) return p == 0 ? 8 : 0;
  else if constexpr (MODE == kModeBf16Bits) return p == 0 ? 7 : (p == 1 ? 15 : 0);
  else if constexpr (MODE == kModeFp16Bits) return p == 0 ? 10 : (p == 1 ? 8 : 0);
  else return a.shift[p];
}

template <int MODE>
__device__ __forceinline__ int mode_bits(const TileArgs& a, int p) {
  if constexpr (MODE == kModeByte2) return 8;
  else if constexpr (MODE == kModeBf16Bits) return p == 0 ? 8 : (p == 1 ? 1 : 7);
  else if constexpr (MODE == kModeFp16Bits) return p == 0 ? 6 : (p == 1 ? 2 : 8);
  else return a.bits[p];
}

// Tile geometry; compile-time constants when DT != 0.
template <int DT>
struct Geo {
  int D, TT, O, A;
  __device__ __forceinline__ explicit Geo(const TileArgs& a)
      : D(DT ? DT : a.D),
        TT(DT ? tile_tokens_for(DT) : a.TT),
        O((DT ? DT : a.D) >> 3),
        A((DT ? tile_tokens_for(DT) : a.TT) >> 3) {}
  // (x + y) mod O for x, y >= 0; O is a power of two when DT != 0.
  __device__ __forceinline__ int rot(int x, int y) const {
    if constexpr (DT != 0) return (x + y) & (O - 1);
    else return (x + y) % O;
  }
};

template <int MODE, int DT>
__device__ __forceinline__ int plane_stride(const TileArgs& a, const Geo<DT>& g, int p, bool restore) {
  return run_stride(g.TT, mode_bits<MODE>(a, p), restore);
}

template <int MODE, int DT>
__device__ __forceinline__ int plane_base(const TileArgs& a, const Geo<DT>& g, int p, bool restore) {
  int base = 0;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    if (q >= p) break;
    base += g.D * plane_stride<MODE, DT>(a, g, q, restore);
  }
  return base;
}

struct TileCoord {
  int kv, h, n;
  int64_t t0;
};

__device__ __forceinline__ TileCoord tile_coord(const TileArgs& args, int TT) {
  int tile = blockIdx.x;
  const int tt = tile % args.tiles_per_head;
  tile /= args.tiles_per_head;
  TileCoord tc;
  tc.h = tile % args.H;
  tc.kv = tile / args.H;
  tc.t0 = static_cast<int64_t>(tt) * TT;
  tc.n = static_cast<int>(min64(static_cast<int64_t>(TT), args.T - tc.t0));
  return tc;
}

// spec_of_c[c] = index of the spec covering (h, c), -1 when none does. rowoff[t] = element
// offset of token t0 + t of (kv, h) in the rows tensor, -1 when its block id is invalid
// (counted in args.err). One block-table lookup per token row and tile.
__device__ __forceinline__ void tile_setup(const TileArgs& args, const TileCoord& tc, int D, int16_t* spec_of_c,
                                           int64_t* rowoff) {
  for (int c = threadIdx.x; c < D; c += kThreads) spec_of_c[c] = -1;
  const int32_t bs = static_cast<int32_t>(args.block_size);
  for (int t = threadIdx.x; t < tc.n; t += kThreads) {
    const int32_t tg = static_cast<int32_t>(tc.t0) + t;
    if (tg >= args.write_tokens) {
      rowoff[t] = -1;
      continue;
    }
    const int32_t bi = tg / bs;
    const int64_t blk = args.block_ids ? args.block_ids[bi] : bi;
    if (blk < 0 || blk >= args.num_blocks) {
      rowoff[t] = -1;
      if (args.err) atomicAdd(args.err, 1u);
    } else {
      rowoff[t] = tc.kv * args.kv_stride + blk * args.block_stride +
                  static_cast<int64_t>(tg - bi * bs) * args.token_stride +
                  static_cast<int64_t>(tc.h) * args.head_stride;
    }
  }
  __syncthreads();
  for (int s = threadIdx.x; s < args.S; s += kThreads) {
    const int64_t* sp = args.specs + 6 * static_cast<int64_t>(s);
    if (sp[0] <= tc.h && tc.h < sp[1]) {
      for (int64_t c = sp[2]; c < sp[3]; ++c) spec_of_c[c] = static_cast<int16_t>(s);
    }
  }
  __syncthreads();
}

// Copy one 8-channel chunk of a token row between shared memory and global memory.
template <int ELEM>
__device__ __forceinline__ void store_chunk(uint8_t* gdst, const uint8_t* ssrc) {
  if constexpr (ELEM == 2) st_global_cs16(gdst, *reinterpret_cast<const uint4*>(ssrc));
  else st_global_cs8(gdst, *reinterpret_cast<const uint2*>(ssrc));
}

template <int ELEM>
__device__ __forceinline__ void load_chunk_async(uint8_t* sdst, const uint8_t* gsrc) {
  if constexpr (ELEM == 2) cp_async16(sdst, gsrc);
  else cp_async8(sdst, gsrc);
}

template <int ELEM>
__device__ __forceinline__ void zero_chunk(uint8_t* sdst) {
  if constexpr (ELEM == 2) *reinterpret_cast<uint4*>(sdst) = make_uint4(0u, 0u, 0u, 0u);
  else *reinterpret_cast<uint2*>(sdst) = make_uint2(0u, 0u);
}

// ---------------------------------------------------------------------------------------
// Restore: packed chunks -> rows
// ---------------------------------------------------------------------------------------
template <int ELEM, int MODE, int DT>
__global__ void __launch_bounds__(kThreads) restore_tiles(const TileArgs args) {
  extern __shared__ __align__(128) uint8_t smem[];
  int16_t* spec_of_c = reinterpret_cast<int16_t*>(smem);
  int64_t* rowoff = reinterpret_cast<int64_t*>(smem + args.rowoff_off);
  RowMeta* meta = reinterpret_cast<RowMeta*>(smem + args.meta_off);
  uint8_t* data = smem + args.data_off;
  const int tid = threadIdx.x;
  const Geo<DT> g(args);
  const int D = g.D;
  const int O = g.O;
  const int P = mode_planes<MODE>(args);
  const TileCoord tc = tile_coord(args, g.TT);

  tile_setup(args, tc, D, spec_of_c, rowoff);

  for (int r = tid; r < P * D; r += kThreads) {
    const int p = r / D;
    const int c = r - p * D;
    const int s = spec_of_c[c];
    RowMeta m;
    m.a = -1;
    m.b = 0;
    m.c = 8 << 16;
    if (s >= 0) {
      const int64_t* sp = args.specs + 6 * static_cast<int64_t>(s);
      const int64_t k = static_cast<int64_t>(tc.kv * P + p) * args.S + s;
      const int bits = args.chunk_bits ? static_cast<int>(args.chunk_bits[k]) : mode_bits<MODE>(args, p);
      const int64_t C = sp[3] - sp[2];
      const int64_t L = ((tc.h - sp[0]) * C + (c - sp[2])) * args.T + tc.t0;
      const int64_t B = args.offsets[k] * 8 + L * bits;
      const int64_t lo16 = (B >> 3) & ~static_cast<int64_t>(15);
      const int64_t hi16 = (((B + static_cast<int64_t>(tc.n) * bits + 7) >> 3) + 15) & ~static_cast<int64_t>(15);
      m.a = lo16;
      m.b = static_cast<int>((hi16 - lo16) >> 4);
      m.c = static_cast<int>(B - lo16 * 8) | (bits << 16);
    }
    meta[r] = m;
  }
  __syncthreads();

  // Phase A: stage the covering 16-byte words of every run, one bulk (TMA) copy per run
  // row; rows no chunk covers are zero-filled, words past the buffer end read bytewise.
  __shared__ __align__(8) uint64_t bar;
  if (tid == 0) {
    mbar_init(&bar, kThreads);
    fence_mbar_init();
  }
  __syncthreads();
  {
    uint32_t my_bytes = 0;  // announced before any of this thread's copies can complete
    for (int r = tid; r < P * D; r += kThreads) {
      const RowMeta m = meta[r];
      if (m.a < 0) continue;
      const int64_t full = min64(m.b, (args.packed_bytes - m.a) >> 4);
      if (full > 0) my_bytes += static_cast<uint32_t>(full) * 16u;
    }
    mbar_expect_tx(&bar, my_bytes);
    for (int r = tid; r < P * D; r += kThreads) {
      const int p = r / D;
      const int c = r - p * D;
      const int rs = plane_stride<MODE, DT>(args, g, p, true);
      uint8_t* row = data + plane_base<MODE, DT>(args, g, p, true) + c * rs;
      const RowMeta m = meta[r];
      if (m.a < 0) {
        for (int w = 0; w < (rs >> 4); ++w) *reinterpret_cast<uint4*>(row + 16 * w) = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      const int64_t full = min64(m.b, (args.packed_bytes - m.a) >> 4);
      if (full > 0) bulk_load(row, args.packed + m.a, static_cast<uint32_t>(full) * 16u, &bar);
      for (int64_t w = max64(full, 0); w < m.b; ++w) {  // words straddling the buffer end
        const int64_t gofs = m.a + 16 * w;
        uint32_t v[4] = {0u, 0u, 0u, 0u};
        for (int j = 0; j < 16; ++j) {
          if (gofs + j < args.packed_bytes) v[j >> 2] |= static_cast<uint32_t>(args.packed[gofs + j]) << (8 * (j & 3));
        }
        *reinterpret_cast<uint4*>(row + 16 * w) = make_uint4(v[0], v[1], v[2], v[3]);
      }
    }
  }
  if (stage_wait_or_bail(&bar, 0, nullptr, 0, false, args.err)) return;

  // Phase B: 8 tokens x 8 channels per thread.
  const int A = g.A;
  const bool have = tid < A * O;
  const int a = tid % A;
  const int o = tid / A;
  constexpr int WPT = ELEM == 2 ? 4 : 2;
  uint32_t out[8][WPT];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
#pragma unroll
    for (int k = 0; k < WPT; ++k) out[i][k] = 0u;
  }
  if (have) {
    uint32_t keep_lo[8], keep_hi[8];  // kModeByte2: plane 0 (high bytes)
#pragma unroll
    for (int p = 0; p < (MODE == kModeGeneric ? 8 : 3); ++p) {
      if (p >= P) break;
      uint32_t lo[8], hi[8];
      const int rs = plane_stride<MODE, DT>(args, g, p, true);
      const uint8_t* pbase = data + plane_base<MODE, DT>(args, g, p, true);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = 8 * o + j;
        const int mc = meta[p * D + c].c;
        const int bits = MODE == kModeGeneric ? (mc >> 16) : mode_bits<MODE>(args, p);
        const int bit0 = mc & 0xFFFF;
        const uint8_t* row = pbase + c * rs;
        if (bits == 8 && (bit0 & 63) == 0) {
          const uint2 v = *reinterpret_cast<const uint2*>(row + (bit0 >> 3) + 8 * a);
          lo[j] = v.x;
          hi[j] = v.y;
        } else {
          uint32_t v0, v1;
          window64(row, bit0 + 8 * a * bits, v0, v1);
          spread8_rt(v0, v1, bits, lo[j], hi[j]);
        }
      }
      transpose8x8(lo, hi);  // row i = token i: channels 0..3 in lo, 4..7 in hi
      if constexpr (ELEM == 1) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          out[i][0] |= lo[i];
          out[i][1] |= hi[i];
        }
      } else if constexpr (MODE == kModeByte2) {
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
        const int s = mode_shift<MODE>(args, p);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          out[i][0] |= prmt(lo[i], 0u, 0x4140) << s;
          out[i][1] |= prmt(lo[i], 0u, 0x4342) << s;
          out[i][2] |= prmt(hi[i], 0u, 0x4140) << s;
          out[i][3] |= prmt(hi[i], 0u, 0x4342) << s;
        }
      }
    }
  }
  __syncthreads();  // every packed run has been consumed; reuse the area for rows
  const int row_bytes = D * ELEM;
  if (have) {
    const int phys = g.rot(o, a);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint8_t* dst = data + (8 * a + i) * row_bytes + phys * (8 * ELEM);
      if constexpr (ELEM == 2) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(out[i][0], out[i][1], out[i][2], out[i][3]);
      } else {
        *reinterpret_cast<uint2*>(dst) = make_uint2(out[i][0], out[i][1]);
      }
    }
  }
  __syncthreads();

  // Phase C: rows to the destination.
  uint8_t* rows = static_cast<uint8_t*>(args.rows);
  if (kThreads % O == 0) {  // fixed chunk per thread, rows strided
    const int oc = tid % O;
    const int step = kThreads / O;
    for (int t = tid / O; t < tc.n; t += step) {
      const int64_t off = rowoff[t];
      if (off < 0) continue;
      store_chunk<ELEM>(rows + (off + 8 * oc) * ELEM, data + t * row_bytes + g.rot(oc, t >> 3) * (8 * ELEM));
    }
  } else {
    for (int i = tid; i < tc.n * O; i += kThreads) {
      const int t = i / O;
      const int oc = i - t * O;
      const int64_t off = rowoff[t];
      if (off < 0) continue;
      store_chunk<ELEM>(rows + (off + 8 * oc) * ELEM, data + t * row_bytes + g.rot(oc, t >> 3) * (8 * ELEM));
    }
  }
}

// ---------------------------------------------------------------------------------------
// Pack: rows -> packed chunks
// ---------------------------------------------------------------------------------------

// One destination 32-bit word of a run, `wr` = its first bit relative to the run start
// (the run owns bits [0, len); its first nsrc bits come from `src`, a 16-byte aligned
// shared row, the rest up to len is zero pad): plain store when the run owns the whole
// word, otherwise a masked atomic clear + set of the run's own bits (a neighbouring run
// owns the rest of the word).
__device__ __forceinline__ void put_word(uint32_t* dst, int wr, int len, int nsrc, const uint32_t* src) {
  const int q = wr >> 5;
  const int r = wr & 31;
  const int nsw = (nsrc + 31) >> 5;
  const uint32_t lo = (q >= 0 && q < nsw) ? src[q] : 0u;
  const uint32_t hi = (q + 1 >= 0 && q + 1 < nsw) ? src[q + 1] : 0u;
  const int first = max(-wr, 0);
  const uint32_t v = __funnelshift_r(lo, hi, r) & bit_range_mask(first, min(max(nsrc - wr, 0), 32));
  const uint32_t own = bit_range_mask(first, min(max(len - wr, 0), 32));
  if (own == 0xFFFFFFFFu) {
    *dst = v;
  } else if (own != 0u) {
    atomicAnd(dst, ~own);
    atomicOr(dst, v & own);
  }
}

template <int ELEM, int MODE, int DT>
__global__ void __launch_bounds__(kThreads) pack_tiles(const TileArgs args) {
  extern __shared__ __align__(128) uint8_t smem[];
  int16_t* spec_of_c = reinterpret_cast<int16_t*>(smem);
  int64_t* rowoff = reinterpret_cast<int64_t*>(smem + args.rowoff_off);
  RowMeta* meta = reinterpret_cast<RowMeta*>(smem + args.meta_off);
  uint8_t* data = smem + args.data_off;
  const int tid = threadIdx.x;
  const Geo<DT> g(args);
  const int D = g.D;
  const int O = g.O;
  const int P = mode_planes<MODE>(args);
  const TileCoord tc = tile_coord(args, g.TT);

  tile_setup(args, tc, D, spec_of_c, rowoff);

  for (int r = tid; r < P * D; r += kThreads) {
    const int p = r / D;
    const int c = r - p * D;
    const int s = spec_of_c[c];
    RowMeta m;
    m.a = -1;
    m.b = 0;
    m.c = 8;
    if (s >= 0) {
      const int64_t* sp = args.specs + 6 * static_cast<int64_t>(s);
      const int64_t k = static_cast<int64_t>(tc.kv * P + p) * args.S + s;
      const int bits = args.chunk_bits ? static_cast<int>(args.chunk_bits[k]) : mode_bits<MODE>(args, p);
      const int64_t C = sp[3] - sp[2];
      const int64_t L = ((tc.h - sp[0]) * C + (c - sp[2])) * args.T + tc.t0;
      const int64_t B = args.offsets[k] * 8 + L * bits;
      int64_t E = B + static_cast<int64_t>(tc.n) * bits;
      // The run that ends a chunk also owns the chunk's zero pad bits.
      if (tc.t0 + tc.n == args.T && c == sp[3] - 1 && tc.h == sp[1] - 1) E = (E + 7) & ~static_cast<int64_t>(7);
      m.a = B;
      m.b = static_cast<int>(E - B);
      m.c = bits;
    }
    meta[r] = m;
  }

  // Phase A: stage the tile's rows; 8-channel chunks rotated by token octet.
  const int row_bytes = D * ELEM;
  const uint8_t* rows = static_cast<const uint8_t*>(args.rows);
  if (kThreads % O == 0) {
    const int oc = tid % O;
    const int step = kThreads / O;
    for (int t = tid / O; t < tc.n; t += step) {
      const int64_t off = rowoff[t];
      uint8_t* dst = data + t * row_bytes + g.rot(oc, t >> 3) * (8 * ELEM);
      if (off < 0) zero_chunk<ELEM>(dst);
      else load_chunk_async<ELEM>(dst, rows + (off + 8 * oc) * ELEM);
    }
  } else {
    for (int i = tid; i < tc.n * O; i += kThreads) {
      const int t = i / O;
      const int oc = i - t * O;
      const int64_t off = rowoff[t];
      uint8_t* dst = data + t * row_bytes + g.rot(oc, t >> 3) * (8 * ELEM);
      if (off < 0) zero_chunk<ELEM>(dst);
      else load_chunk_async<ELEM>(dst, rows + (off + 8 * oc) * ELEM);
    }
  }
  cp_async_wait_all();
  __syncthreads();

  const int A = g.A;
  const bool have = tid < A * O;
  const int a = tid % A;
  const int o = tid / A;
  constexpr int WPT = ELEM == 2 ? 4 : 2;
  uint32_t x[8][WPT];
  if (have) {
    const int phys = g.rot(o, a);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint8_t* src = data + (8 * a + i) * row_bytes + phys * (8 * ELEM);
      if constexpr (ELEM == 2) {
        const uint4 v = *reinterpret_cast<const uint4*>(src);
        x[i][0] = v.x;
        x[i][1] = v.y;
        x[i][2] = v.z;
        x[i][3] = v.w;
      } else {
        const uint2 v = *reinterpret_cast<const uint2*>(src);
        x[i][0] = v.x;
        x[i][1] = v.y;
      }
    }
  }
  __syncthreads();  // rows consumed; reuse the area for packed runs

  if (have) {
#pragma unroll
    for (int p = 0; p < (MODE == kModeGeneric ? 8 : 3); ++p) {
      if (p >= P) break;
      uint32_t lo[8], hi[8];
      if constexpr (ELEM == 1) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          lo[i] = x[i][0];  // masked per chunk below
          hi[i] = x[i][1];
        }
      } else if constexpr (MODE == kModeByte2) {
        const uint32_t sel = p == 0 ? 0x7531u : 0x6420u;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          lo[i] = prmt(x[i][0], x[i][1], sel);
          hi[i] = prmt(x[i][2], x[i][3], sel);
        }
      } else {
        const int s = mode_shift<MODE>(args, p);
        const uint32_t m = (1u << mode_bits<MODE>(args, p)) - 1u;
        const uint32_t m2 = m | (m << 16);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          lo[i] = prmt((x[i][0] >> s) & m2, (x[i][1] >> s) & m2, 0x6420);
          hi[i] = prmt((x[i][2] >> s) & m2, (x[i][3] >> s) & m2, 0x6420);
        }
      }
      transpose8x8(lo, hi);  // row j = channel j: tokens 0..3 in lo, 4..7 in hi
      const int rs = plane_stride<MODE, DT>(args, g, p, false);
      uint8_t* pbase = data + plane_base<MODE, DT>(args, g, p, false);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = 8 * o + j;
        const int bits = MODE == kModeGeneric ? meta[p * D + c].c : mode_bits<MODE>(args, p);
        uint8_t* row = pbase + c * rs;
        if (bits == 8) {
          *reinterpret_cast<uint2*>(row + 8 * a) = make_uint2(lo[j], hi[j]);
        } else {
          const uint32_t mb = ((1u << bits) - 1u) * 0x01010101u;
          const uint64_t v = gather8(lo[j] & mb, hi[j] & mb, bits);
#pragma unroll 8
          for (int q = 0; q < bits; ++q) row[a * bits + q] = static_cast<uint8_t>(v >> (8 * q));
        }
      }
    }
  }
  __syncthreads();

  // Phase C: runs to the chunk stream in 16-byte destination vectors.
  uint32_t* dst32 = reinterpret_cast<uint32_t*>(args.packed);
#pragma unroll 1
  for (int p = 0; p < P; ++p) {
    const int maxbits = MODE == kModeGeneric ? args.bits[p] : mode_bits<MODE>(args, p);
    const int Vmax = ((g.TT * maxbits + 7 + 127) >> 7) + 1;
    const int cnt = D * Vmax;
    const int rs = plane_stride<MODE, DT>(args, g, p, false);
    const uint8_t* pbase = data + plane_base<MODE, DT>(args, g, p, false);
    const RowMeta* pm = meta + p * D;
    for (int i = tid; i < cnt; i += kThreads) {
      const int c = i / Vmax;
      const int v = i - c * Vmax;
      const RowMeta m = pm[c];
      if (m.a < 0) continue;
      const int len = m.b;                                     // run bits incl. pad
      const int rel = (v << 7) - static_cast<int>(m.a & 127);  // vector's first bit, run-relative
      if (rel >= len) continue;
      const int nsrc = tc.n * m.c;
      const int64_t V = (m.a >> 7) + v;
      const uint32_t* src = reinterpret_cast<const uint32_t*>(pbase + c * rs);
      if (rel >= 0 && rel + 128 <= nsrc && rel + 128 <= len) {
        // fully owned vector made of source bits only: whole 16-byte store, the run's bit
        // offset applied with funnel shifts (src[q + 4] holds source bits when r > 0)
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
        st_global_cs16(dst32 + 4 * V, w);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int wr = rel + 32 * k;
          if (wr + 32 <= 0 || wr >= len) continue;
          put_word(dst32 + 4 * V + k, wr, len, nsrc, src);
        }
      }
    }
  }
}

}  // namespace origami
