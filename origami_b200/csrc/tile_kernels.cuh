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
//   in registers -> plane merge -> smem rows [t][c] (rotated 16-byte chunks, bank-conflict
//   free) -> 16-byte streaming stores into the destination rows via the block table.
// pack_tiles: the inverse; partially owned 32-bit words at run edges are merged with
//   masked atomics so any bit alignment (ragged token counts, odd bit widths) is exact
//   without a zero-fill pass.
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
  int32_t TT, tiles_per_head;
  // Planes.
  int32_t P;
  int32_t shift[8];
  int32_t bits[8];
  // Shared memory layout.
  int32_t rs[8];          // row stride (bytes) of plane p's packed rows
  int32_t plane_base[8];  // offset of plane p's rows inside the data area
  int32_t meta_off, data_off;
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

struct TileCoord {
  int kv, h, n;
  int64_t t0;
};

__device__ __forceinline__ TileCoord tile_coord(const TileArgs& args) {
  int tile = blockIdx.x;
  const int tt = tile % args.tiles_per_head;
  tile /= args.tiles_per_head;
  TileCoord tc;
  tc.h = tile % args.H;
  tc.kv = tile / args.H;
  tc.t0 = static_cast<int64_t>(tt) * args.TT;
  tc.n = static_cast<int>(min64(static_cast<int64_t>(args.TT), args.T - tc.t0));
  return tc;
}

// spec_of_c[c] = index of the spec covering (h, c), -1 when none does.
__device__ __forceinline__ void scan_specs(const TileArgs& args, int h, int16_t* spec_of_c) {
  for (int c = threadIdx.x; c < args.D; c += kThreads) spec_of_c[c] = -1;
  __syncthreads();
  for (int s = threadIdx.x; s < args.S; s += kThreads) {
    const int64_t* sp = args.specs + 6 * static_cast<int64_t>(s);
    if (sp[0] <= h && h < sp[1]) {
      for (int64_t c = sp[2]; c < sp[3]; ++c) spec_of_c[c] = static_cast<int16_t>(s);
    }
  }
  __syncthreads();
}

__device__ __forceinline__ int64_t row_element(const TileArgs& args, int kv, int h, int64_t tg,
                                               int64_t& blk) {
  const int64_t bi = tg / args.block_size;
  blk = args.block_ids ? args.block_ids[bi] : bi;
  return kv * args.kv_stride + blk * args.block_stride + (tg - bi * args.block_size) * args.token_stride +
         static_cast<int64_t>(h) * args.head_stride;
}

// ---------------------------------------------------------------------------------------
// Restore: packed chunks -> rows
// ---------------------------------------------------------------------------------------
template <int ELEM, int MODE>
__global__ void __launch_bounds__(kThreads) restore_tiles(const TileArgs args) {
  extern __shared__ __align__(128) uint8_t smem[];
  int16_t* spec_of_c = reinterpret_cast<int16_t*>(smem);
  RowMeta* meta = reinterpret_cast<RowMeta*>(smem + args.meta_off);
  uint8_t* data = smem + args.data_off;
  const int tid = threadIdx.x;
  const int D = args.D;
  const int P = mode_planes<MODE>(args);
  const TileCoord tc = tile_coord(args);

  scan_specs(args, tc.h, spec_of_c);

  // Per-run metadata.
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

  // Phase A: stage the covering 16-byte words of every run.
  for (int p = 0; p < P; ++p) {
    const int W = args.rs[p] >> 4;
    const int cnt = D * W;
    uint8_t* pbase = data + args.plane_base[p];
    for (int i = tid; i < cnt; i += kThreads) {
      const int c = i / W;
      const int w = i - c * W;
      const RowMeta m = meta[p * D + c];
      uint8_t* dst = pbase + c * args.rs[p] + w * 16;
      if (m.a < 0) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      if (w >= m.b) continue;
      const int64_t g = m.a + 16 * static_cast<int64_t>(w);
      if (g + 16 <= args.packed_bytes) {
        cp_async16(dst, args.packed + g);
      } else {
        uint32_t v[4] = {0u, 0u, 0u, 0u};
        for (int j = 0; j < 16; ++j) {
          if (g + j < args.packed_bytes) v[j >> 2] |= static_cast<uint32_t>(args.packed[g + j]) << (8 * (j & 3));
        }
        *reinterpret_cast<uint4*>(dst) = make_uint4(v[0], v[1], v[2], v[3]);
      }
    }
  }
  cp_async_wait_all();
  __syncthreads();

  // Phase B: 8 tokens x 8 channels per thread.
  const int A = args.TT >> 3;
  const int O = D >> 3;
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
      const uint8_t* pbase = data + args.plane_base[p];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = 8 * o + j;
        const int mc = meta[p * D + c].c;
        const int bits = MODE == kModeGeneric ? (mc >> 16) : mode_bits<MODE>(args, p);
        const int bitpos = (mc & 0xFFFF) + 8 * a * bits;
        uint32_t v0, v1;
        window64(pbase + c * args.rs[p], bitpos, v0, v1);
        spread8_rt(v0, v1, bits, lo[j], hi[j]);
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
    const int phys = (o + a) % O;
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
  for (int i = tid; i < tc.n * O; i += kThreads) {
    const int t = i / O;
    const int oc = i - t * O;
    int64_t blk;
    const int64_t e = row_element(args, tc.kv, tc.h, tc.t0 + t, blk);
    if (blk < 0 || blk >= args.num_blocks) {
      if (oc == 0 && args.err) atomicAdd(args.err, 1u);
      continue;
    }
    const int phys = (oc + (t >> 3)) % O;
    const uint8_t* src = data + t * row_bytes + phys * (8 * ELEM);
    uint8_t* dst = rows + (e + 8 * oc) * ELEM;
    if constexpr (ELEM == 2) {
      st_global_cs16(dst, *reinterpret_cast<const uint4*>(src));
    } else {
      st_global_cs8(dst, *reinterpret_cast<const uint2*>(src));
    }
  }
}

// ---------------------------------------------------------------------------------------
// Pack: rows -> packed chunks
// ---------------------------------------------------------------------------------------
template <int ELEM, int MODE>
__global__ void __launch_bounds__(kThreads) pack_tiles(const TileArgs args) {
  extern __shared__ __align__(128) uint8_t smem[];
  int16_t* spec_of_c = reinterpret_cast<int16_t*>(smem);
  RowMeta* meta = reinterpret_cast<RowMeta*>(smem + args.meta_off);
  uint8_t* data = smem + args.data_off;
  const int tid = threadIdx.x;
  const int D = args.D;
  const int P = mode_planes<MODE>(args);
  const TileCoord tc = tile_coord(args);

  scan_specs(args, tc.h, spec_of_c);

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
  const int O = D >> 3;
  const int row_bytes = D * ELEM;
  const uint8_t* rows = static_cast<const uint8_t*>(args.rows);
  for (int i = tid; i < tc.n * O; i += kThreads) {
    const int t = i / O;
    const int oc = i - t * O;
    int64_t blk;
    const int64_t e = row_element(args, tc.kv, tc.h, tc.t0 + t, blk);
    uint8_t* dst = data + t * row_bytes + ((oc + (t >> 3)) % O) * (8 * ELEM);
    if (blk < 0 || blk >= args.num_blocks) {
      if (oc == 0 && args.err) atomicAdd(args.err, 1u);
      if constexpr (ELEM == 2) *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      else *reinterpret_cast<uint2*>(dst) = make_uint2(0u, 0u);
      continue;
    }
    const uint8_t* src = rows + (e + 8 * oc) * ELEM;
    if constexpr (ELEM == 2) cp_async16(dst, src);
    else cp_async8(dst, src);
  }
  cp_async_wait_all();
  __syncthreads();

  const int A = args.TT >> 3;
  const bool have = tid < A * O;
  const int a = tid % A;
  const int o = tid / A;
  constexpr int WPT = ELEM == 2 ? 4 : 2;
  uint32_t x[8][WPT];
  if (have) {
    const int phys = (o + a) % O;
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
          // one plane per symbol tensor; masking happens per chunk below
          lo[i] = x[i][0];
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
      uint8_t* pbase = data + args.plane_base[p];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = 8 * o + j;
        const int bits = MODE == kModeGeneric ? meta[p * D + c].c : mode_bits<MODE>(args, p);
        uint8_t* row = pbase + c * args.rs[p];
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

  // Phase C: runs to the chunk stream. Fully owned words: plain stores; words shared
  // with a neighbouring run: masked atomic clear + set of this run's bits only.
  uint32_t* dst32 = reinterpret_cast<uint32_t*>(args.packed);
  for (int p = 0; p < P; ++p) {
    const int maxbits = MODE == kModeGeneric ? 8 : mode_bits<MODE>(args, p);
    const int Wmax = ((args.TT * maxbits + 7 + 31) >> 5) + 1;
    const int cnt = D * Wmax;
    const uint8_t* pbase = data + args.plane_base[p];
    for (int i = tid; i < cnt; i += kThreads) {
      const int c = i / Wmax;
      const int w = i - c * Wmax;
      const RowMeta m = meta[p * D + c];
      if (m.a < 0) continue;
      const int64_t B = m.a;
      const int64_t E = B + m.b;
      const int64_t W = (B >> 5) + w;
      if (W > ((E - 1) >> 5)) continue;
      const int64_t rel = W * 32 - B;
      const int64_t nsrc = static_cast<int64_t>(tc.n) * m.c;
      const int64_t nsw = (nsrc + 31) >> 5;
      const uint32_t* src = reinterpret_cast<const uint32_t*>(pbase + c * args.rs[p]);
      const int64_t q = rel >> 5;
      const int r = static_cast<int>(rel & 31);
      const uint32_t lo = (q >= 0 && q < nsw) ? src[q] : 0u;
      const uint32_t hi = (q + 1 >= 0 && q + 1 < nsw) ? src[q + 1] : 0u;
      uint32_t v = __funnelshift_r(lo, hi, r);
      const int vlo = static_cast<int>(min64(max64(-rel, 0), 32));
      const int vhi = static_cast<int>(min64(max64(nsrc - rel, 0), 32));
      v &= bit_range_mask(vlo, vhi);
      const int olo = static_cast<int>(min64(max64(B - W * 32, 0), 32));
      const int ohi = static_cast<int>(min64(max64(E - W * 32, 0), 32));
      const uint32_t own = bit_range_mask(olo, ohi);
      if (own == 0xFFFFFFFFu) {
        dst32[W] = v;
      } else if (own != 0u) {
        atomicAnd(dst32 + W, ~own);
        atomicOr(dst32 + W, v & own);
      }
    }
  }
}

}  // namespace origami
