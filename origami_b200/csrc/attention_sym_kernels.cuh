// prefix_attention_sym: the fused prefix attention with the dequantization scales applied
// by the tensor cores (decode shapes: 8 query rows per CTA).
//
// A quantized element is s * scale + zero with s a small integer (exact in fp16 / bf16).
// So the K and V^T operand tiles hold the raw symbols s, converted with one lookup in a
// 256-entry byte table per 1, 2 or 4 symbols, the scales move to the small B operands of
// the MMAs and the zeros to per-row sums:
//   S^T_g = K_sym . (q (.) scale_g)^T  + (q . zero_g)        per K group g in the tile
//   S^T_R = K_val . q^T                                       real keys (sinks, suffix)
//   O^T_c = V_sym^T . (P (.) vscale_c)^T + sum_t P_t vzero_c  per value channel group c
// (KIVI: key scale / zero per (token group, channel), value scale / zero per (token,
// channel group); KVQuant: key per channel (one group), value per token (one channel
// group).) The groups' B operands are stacked along N, so each tile takes one chain of 8
// MMAs with N = 32 (3 key groups + the real block) for S and one with N = 16 (2 channel
// groups) for O. A key's softmax lane reads the S block of its group and adds q . zero of
// that group; a dim's output lane reads the O block of its channel group and adds the
// running sum of P * vzero, rescaled with O by the online softmax. Real-valued keys carry
// their values in the same tiles with scale 1 / zero 0 on the V side.
//
// The stream words of tile j + 1 (and its key-group and per-key metadata) are copied into
// shared memory with cp.async while tile j's MMAs and softmax run; the symbol decode then
// reads shared memory only. Row blocks, splits, online softmax and merge are
// prefix_attention's. Used when a 128-key tile spans at most 3 key groups and a head at
// most 2 value channel groups (KIVI group size >= 64; KVQuant always).
#pragma once

#include "attention_kernels.cuh"

namespace origami {

namespace attn {

constexpr int kSymNQ = 8;
constexpr int kSymMaxG = 3;                      // K groups per 128-key tile
constexpr int kSymMaxC = 2;                      // value channel groups per head
constexpr int kSymReal = kSymMaxG;               // S block of the real-valued keys
constexpr int kSymSCols = 8 * (kSymMaxG + 1);    // N of the S product
constexpr int kSymOCols = 8 * kSymMaxC;          // N of the O product
constexpr uint32_t kSymOCol = kSymSCols;         // first O column in TMEM
constexpr uint32_t kSymTmemCols = 64;
constexpr int kRowTile = kSBO;                   // one B operand block of 8 rows x 128
constexpr int kMetaWords = 65;                   // 128 fp16 values from a 2-byte aligned address

// Words staged per dim run of a 128-key tile: 128 symbols of `slot` bits plus the bit
// offset of the run's first symbol inside its word.
__host__ __device__ constexpr int sym_run_words(int slot) { return 4 * slot + 1; }

__device__ __forceinline__ void cp_async4(uint32_t* dst, uintptr_t src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

// Element (kv, key, dim d of head h) as the symbol tiles hold it: the raw symbol for a
// body key, the value for sink / suffix keys, 0 past kmax.
template <int CODEC>
__device__ float element_sym(const AttnArgs& a, int kv, int64_t key, int h, int d, int64_t kmax, float bias) {
  if (key > kmax) return 0.f;
  if (key < a.prefix && (CODEC == 1 || key >= a.sink)) {
    const int64_t bt = CODEC == 0 ? key - a.sink : key;
    int64_t idx;
    if (kv == 0) idx = (static_cast<int64_t>(d) * a.kv_heads + h) * a.body + bt;
    else if (CODEC == 0) idx = (static_cast<int64_t>(h) * kD + d) * a.body + bt;
    else idx = (static_cast<int64_t>(h) * a.prefix + key) * kD + d;
    return bias + static_cast<float>(symbol(a, kv, idx));
  }
  return element<CODEC>(a, kv, key, h, d, kmax);
}

// Byte table: the 16-bit values of the symbols packed in byte e, low symbol first
// (8 / slot_bits symbols per byte).
template <typename QT>
__device__ __forceinline__ uint2 sym_lut_entry(uint32_t e, int slot, uint32_t mask) {
  if (slot == 2)
    return make_uint2(pack2<QT>(static_cast<float>(e & mask), static_cast<float>((e >> 2) & mask)),
                      pack2<QT>(static_cast<float>((e >> 4) & mask), static_cast<float>((e >> 6) & mask)));
  if (slot == 4) return make_uint2(pack2<QT>(static_cast<float>(e & mask), static_cast<float>((e >> 4) & mask)), 0u);
  return make_uint2(pack2<QT>(static_cast<float>(e), 0.f), 0u);
}

// 8 consecutive symbols of a window as 4 words of 16-bit values through the byte table.
__device__ __forceinline__ uint4 sym8(const uint2* lut, const Win& w, int slot) {
  if (slot == 2) {
    const uint2 a = lut[w.lo & 0xFFu], b = lut[(w.lo >> 8) & 0xFFu];
    return make_uint4(a.x, a.y, b.x, b.y);
  }
  if (slot == 4)
    return make_uint4(lut[w.lo & 0xFFu].x, lut[(w.lo >> 8) & 0xFFu].x, lut[(w.lo >> 16) & 0xFFu].x,
                      lut[w.lo >> 24].x);
  uint32_t v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t word = k < 2 ? w.lo : w.hi;
    const uint32_t b0 = (word >> (16 * (k & 1))) & 0xFFu, b1 = (word >> (16 * (k & 1) + 8)) & 0xFFu;
    v[k] = (lut[b0].x & 0xFFFFu) | (lut[b1].x << 16);
  }
  return make_uint4(v[0], v[1], v[2], v[3]);
}

// 8 consecutive symbols of a window (low symbol first) as 4 words of 16-bit values
// bias + s, built with byte permutes: the bit pattern 0x4300 | s is 128 + s in bf16,
// 0x6400 | s is 1024 + s in fp16 (s below 128 / 1024: exact). bf16 with 8-bit symbols
// (s up to 255) goes through the byte table instead, with bias 0.
template <int SLOT, bool BF16>
__device__ __forceinline__ uint4 sym8_bias(const Win& w, const uint2* lut, uint32_t mask4) {
  if constexpr (SLOT == 2) {
    constexpr uint32_t C = BF16 ? 0x43004300u : 0x64006400u;
    const uint32_t m = w.lo & 0x3333u, e = (w.lo >> 2) & 0x3333u;  // even / odd symbols, 2 per byte
    const uint32_t t01 = __byte_perm(m, e, 0x4400), t23 = __byte_perm(m, e, 0x5511);
    return make_uint4((t01 & 0x00030003u) | C, ((t01 >> 4) & 0x00030003u) | C, (t23 & 0x00030003u) | C,
                      ((t23 >> 4) & 0x00030003u) | C);
  } else if constexpr (SLOT == 4) {
    constexpr uint32_t CR = BF16 ? 0x43434343u : 0x64646464u;
    const uint32_t y = w.lo & mask4, z = (w.lo >> 4) & mask4;  // even / odd symbols, 1 per byte
    const uint32_t t = __byte_perm(y, z, 0x5140), u = __byte_perm(y, z, 0x7362);
    return make_uint4(__byte_perm(t, CR, 0x4140), __byte_perm(t, CR, 0x4342), __byte_perm(u, CR, 0x4140),
                      __byte_perm(u, CR, 0x4342));
  } else {
    if constexpr (BF16) return sym8(lut, w, 8);
    constexpr uint32_t CR = 0x64646464u;
    return make_uint4(__byte_perm(w.lo, CR, 0x4140), __byte_perm(w.lo, CR, 0x4342), __byte_perm(w.hi, CR, 0x4140),
                      __byte_perm(w.hi, CR, 0x4342));
  }
}
template <bool BF16>
__host__ __device__ constexpr float sym_bias(int slot) {
  return BF16 ? (slot == 8 ? 0.f : 128.f) : 1024.f;
}

// 64 symbols of a staged run from bit `sh` of src[0] (8 octets; octet o goes to
// dst + o * stride when bit o of `octets` is set).
template <int SLOT, bool BF16>
__device__ __forceinline__ void decode_half_run(const uint32_t* src, uint32_t sh, uint32_t octets, uint8_t* dst,
                                                int stride, const uint2* lut, uint32_t mask4) {
  constexpr int NW = 2 * SLOT;
  uint32_t raw[NW + 1], n[NW];
#pragma unroll
  for (int i = 0; i <= NW; ++i) raw[i] = src[i];
#pragma unroll
  for (int i = 0; i < NW; ++i) n[i] = __funnelshift_r(raw[i], raw[i + 1], sh);
#pragma unroll
  for (int o = 0; o < 8; ++o) {
    if (!((octets >> o) & 1u)) continue;
    Win w;
    w.hi = 0u;
    if constexpr (SLOT == 2) {
      w.lo = n[o >> 1] >> (16 * (o & 1));
    } else if constexpr (SLOT == 4) {
      w.lo = n[o];
    } else {
      w.lo = n[2 * o];
      w.hi = n[2 * o + 1];
    }
    *reinterpret_cast<uint4*>(dst + o * stride) = sym8_bias<SLOT, BF16>(w, lut, mask4);
  }
}

// The 8 symbols at bit `pos` of a staged run (`pos` counted from the run's first word).
__device__ __forceinline__ Win staged_window(const uint32_t* run, uint32_t pos, bool narrow) {
  const uint32_t* w = run + (pos >> 5);
  const uint32_t sh = pos & 31u;
  Win r;
  r.lo = __funnelshift_r(w[0], w[1], sh);
  r.hi = narrow ? 0u : __funnelshift_r(w[1], w[2], sh);
  return r;
}

// Dims 8 dq .. 8 dq + 7 of a cache row whose element offset without the kv term, `off`,
// was resolved through the block table when the tile was staged (-1: block id out of
// range, the row reads as zeros as in cache_row8).
template <typename QT>
__device__ __forceinline__ void cache_row8_at(const AttnArgs& a, int kv, int64_t off, int dq, uint32_t (&w)[4]) {
  if (off < 0) {
    w[0] = w[1] = w[2] = w[3] = 0u;
    return;
  }
  const int64_t e = kv * a.kv_stride + off + 8 * dq;
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

// 8 x 8 block of keys kb.. x dims 8*dq.. in a non-body octet, as rows per key (real
// values for sink / suffix keys, bias + symbol for body keys, element by element at mixed
// octets).
template <typename QT, int CODEC>
__device__ __forceinline__ void real_rows8(const AttnArgs& a, int kv, int h, int64_t kb, int dq, int64_t kmax,
                                           float bias, const int64_t* rowsfx, int64_t k0, uint32_t (&m)[8][4]) {
  if (kb + 7 <= kmax && kb >= a.prefix) {
#pragma unroll
    for (int i = 0; i < 8; ++i) cache_row8_at<QT>(a, kv, rowsfx[kb + i - k0], dq, m[i]);
  } else if (CODEC == 0 && kb + 7 <= kmax && kb + 7 < a.sink) {
#pragma unroll
    for (int i = 0; i < 8; ++i) sink_row8<QT>(a, kv, kb + i, h, dq, m[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int w = 0; w < 4; ++w)
        m[i][w] = pack2<QT>(element_sym<CODEC>(a, kv, kb + i, h, 8 * dq + 2 * w, kmax, bias),
                            element_sym<CODEC>(a, kv, kb + i, h, 8 * dq + 2 * w + 1, kmax, bias));
  }
}

// 8 raw fp16 values p[i .. i+7] (one 16-byte load when `vec`).
__device__ __forceinline__ uint4 load8h(const __half* p, int64_t i, bool vec) {
  if (vec) return __ldg(reinterpret_cast<const uint4*>(p + i));
  const uint16_t* q = reinterpret_cast<const uint16_t*>(p) + i;
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) w[k] = static_cast<uint32_t>(__ldg(q + 2 * k)) | (static_cast<uint32_t>(__ldg(q + 2 * k + 1)) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// KVQuant V^T tile (MN-major: dims contiguous per key) from the head's staged symbols:
// dim octet u_lo of keys u_hi + 16 r, body octets [ob_lo, ob_hi) only.
template <int SLOT, bool BF16>
__device__ __forceinline__ void decode_kvq_v(const uint32_t* rawv, uint32_t sh0, int u_lo, int u_hi, int ob_lo,
                                             int ob_hi, uint8_t* vt_sm, const uint2* lut, uint32_t mask4) {
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int tl = u_hi + 16 * r;
    if ((tl >> 3) < ob_lo || (tl >> 3) >= ob_hi) continue;
    const Win w = staged_window(rawv, sh0 + static_cast<uint32_t>((tl * kD + 8 * u_lo) * SLOT), SLOT != 8);
    *reinterpret_cast<uint4*>(vt_sm + u_lo * kSBO + (tl >> 3) * kLBO + (tl & 7) * 16) = sym8_bias<SLOT, BF16>(w, lut, mask4);
  }
}

// Barrier 1 over warps 0..3 (the softmax warps) with an OR vote.
__device__ __forceinline__ bool named_sync_or_softmax(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n barrier.cta.red.or.pred p, 1, 128, q;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0u;
}

// First tile of split sp when the nkt tiles are shared by cost: a body tile costs 4, a tile
// holding sink keys 5 (rows from the sink tensors) and one holding paged-cache keys 7
// (rows through the block table), in line with their measured times; split sp starts at
// the tile boundary whose cost(tiles < t) * splits is nearest to sp * cost(all).
template <int CODEC>
__device__ __forceinline__ int sym_split_begin(const AttnArgs& a, int sp, int nkt) {
  if (sp <= 0) return 0;
  if (sp >= a.splits) return nkt;
  const int64_t fs = min(static_cast<int64_t>(nkt), a.prefix / kKT);  // first tile with cache keys
  const int64_t ns = CODEC == 0 ? min(fs, (a.sink + kKT - 1) / kKT) : 0;  // tiles with sink keys before it
  auto cost = [&](int64_t t) { return 4 * t + min(t, ns) + 3 * max(static_cast<int64_t>(0), t - fs); };
  const int64_t goal = static_cast<int64_t>(sp) * cost(nkt);
  int lo = 0, hi = nkt;  // cost(hi) * splits >= goal
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (cost(mid) * a.splits >= goal) hi = mid;
    else lo = mid + 1;
  }
  // the nearer of the two boundaries around the goal (fewer uneven splits than rounding up)
  if (lo > 0 && goal - cost(lo - 1) * a.splits < cost(lo) * a.splits - goal) --lo;
  return lo;
}

// Key range, body range and key groups of tile kt.
struct SymTile {
  int64_t k0, kend, b_lo, b_hi, g_lo;
  int n_g;
  bool has_body, has_real;
};
template <int CODEC>
__device__ __forceinline__ SymTile sym_tile(const AttnArgs& a, int kt, int64_t kmax) {
  SymTile t;
  t.k0 = static_cast<int64_t>(kt) * kKT;
  t.kend = min(t.k0 + kKT, kmax + 1);
  t.b_lo = max(t.k0, static_cast<int64_t>(CODEC == 0 ? a.sink : 0));
  t.b_hi = min(t.kend, a.prefix);  // body keys [b_lo, b_hi)
  t.has_body = t.b_lo < t.b_hi;
  t.has_real = !(t.has_body && t.b_lo == t.k0 && t.b_hi == t.kend);
  t.g_lo = 0;
  t.n_g = t.has_body ? 1 : 0;
  if (CODEC == 0 && t.has_body) {
    const uint32_t gs = static_cast<uint32_t>(a.group_size);
    t.g_lo = static_cast<uint32_t>(t.b_lo - a.sink) / gs;
    t.n_g = static_cast<int>(static_cast<uint32_t>(t.b_hi - 1 - a.sink) / gs - t.g_lo + 1);
  }
  return t;
}

}  // namespace attn

// Shared memory of prefix_attention_sym; the staged stream words at the end depend on the
// slot width.
struct AttnSymSmem {
  static constexpr int a_off = 0;                                              // K tile (MN-major: keys x dims)
  static constexpr int v_off = a_off + attn::kTileBytes;                       // V^T tile
  static constexpr int lut_off = v_off + attn::kTileBytes;                     // 256 x uint2
  static constexpr int bq_off = lut_off + 256 * 8;                             // [32 x 128]: q (.) scale_g, q
  static constexpr int ps_off = bq_off + (attn::kSymMaxG + 1) * attn::kRowTile;  // [16 x 128]: P (.) vscale_c
  static constexpr int f_off = ps_off + attn::kSymMaxC * attn::kRowTile;
  // floats: red[4][8], redz[2][4][8], m_run, l_run, alpha, m_new [8], cz[4][8], zacc[2][8],
  // cs[4][8]
  static constexpr int n_floats = 4 * 8 + 8 * 8 + 4 * 8 + 4 * 8 + 2 * 8 + 4 * 8;
  static constexpr int cend_off = f_off + n_floats * 4;                        // [8] int64
  static constexpr int rowsfx_off = cend_off + 8 * 8;                          // [128] int64: suffix rows
  static constexpr int bars_off = rowsfx_off + 128 * 8;                        // 2 mbarriers, TMEM slot, 2 flags
  static constexpr int raw_off = bars_off + 32;
  // staged words: K runs [128][rw] + 2, V runs [128][rw] + 2, key-group rows [3][2][65],
  // per-key value scale / zero [128][2][2]
  __host__ __device__ static constexpr int raw_words(int slot) {
    return 2 * (128 * attn::sym_run_words(slot) + 2) + attn::kSymMaxG * 2 * attn::kMetaWords + 128 * 4;
  }
  __host__ __device__ static constexpr int bytes(int slot) { return raw_off + 4 * raw_words(slot) + 128; }
};
static_assert(AttnSymSmem::raw_off % 16 == 0, "staged words 16-byte aligned");
static_assert(AttnSymSmem::bytes(4) + 1024 <= 233472 / 2, "two CTAs per SM up to 4-bit slots");

// grid = kv_heads * row_blocks * splits CTAs of 256 threads, 8 query rows per CTA; dynamic
// shared memory AttnSymSmem::bytes(SLOT). SLOT = a.slot_bits (2, 4 or 8).
template <typename QT, int CODEC, int SLOT>
__global__ void __launch_bounds__(attn::kThreadsA, 2) prefix_attention_sym(const __grid_constant__ AttnArgs a) {
  using namespace attn;
  using L = AttnSymSmem;
  constexpr int NQ = kSymNQ;
  extern __shared__ __align__(128) uint8_t sym_smem[];
  uint8_t* sm = sym_smem + ((128 - (smem_u32(sym_smem) & 127)) & 127);
  uint8_t* kt_sm = sm + L::a_off;
  uint8_t* vt_sm = sm + L::v_off;
  uint2* lut = reinterpret_cast<uint2*>(sm + L::lut_off);
  uint8_t* bq_sm = sm + L::bq_off;
  uint8_t* ps_sm = sm + L::ps_off;
  float* red = reinterpret_cast<float*>(sm + L::f_off);  // [4][NQ]
  float* redz = red + 4 * NQ;                            // [2][4][NQ]
  float* m_run = redz + 8 * NQ;
  float* l_run = m_run + NQ;
  float* alpha = l_run + NQ;
  float* m_new = alpha + NQ;
  float* cz = m_new + NQ;         // [4][NQ]: q . zero of the tile's key groups (block 3: 0)
  float* zacc = cz + 4 * NQ;      // [2][NQ]: running sum of p * value zero per channel group
  float* cs = zacc + 2 * NQ;      // [4][NQ]: sum of q (.) scale (as rounded) of the tile's key groups
  int64_t* cend = reinterpret_cast<int64_t*>(sm + L::cend_off);
  int64_t* rowsfx = reinterpret_cast<int64_t*>(sm + L::rowsfx_off);  // the tile's suffix rows, by key - k0
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::bars_off);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
  uint32_t* last_flag = tslot + 1;
  uint32_t* fail_flag = tslot + 2;  // a softmax warp's wait for S ran out
  constexpr int slot = SLOT;
  constexpr int rw = sym_run_words(SLOT);
  uint32_t* rawk = reinterpret_cast<uint32_t*>(sm + L::raw_off);  // [128][rw] + 2
  uint32_t* rawv = rawk + 128 * rw + 2;                           // [128][rw] + 2 (KVQuant: one run)
  uint32_t* kmw = rawv + 128 * rw + 2;                            // [3][2][65]
  uint32_t* vmw = kmw + kSymMaxG * 2 * kMetaWords;                // [128][2][2]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sp = static_cast<int>(blockIdx.x % a.splits);
  const int rest = static_cast<int>(blockIdx.x / a.splits);
  const int rb = rest % a.row_blocks;
  const int h = rest / a.row_blocks;
  const int row0 = rb * NQ;
  const int last_row = min(a.rows, row0 + NQ) - 1;
  const int64_t kmax = min(a.seq_len - 1, a.q_start + last_row / a.group);
  const int nkt = static_cast<int>(kmax / kKT) + 1;
  const int t_begin = sym_split_begin<CODEC>(a, sp, nkt);
  const int t_end = sym_split_begin<CODEC>(a, sp + 1, nkt);
  constexpr bool kBf16 = is_bf16<QT>();
  constexpr uint32_t idesc_s = instr_desc(kBf16, kSymSCols) | (1u << 15);  // MN-major K tile
  constexpr uint32_t idesc_o = CODEC == 0 ? instr_desc(kBf16, kSymOCols) : (instr_desc(kBf16, kSymOCols) | (1u << 15));
  const int64_t C = static_cast<int64_t>(a.kv_heads) * kD;
  const int64_t run = CODEC == 0 ? a.body : a.prefix;  // tokens per K (and KIVI V) dim run
  // value channel groups of this head (KIVI); KVQuant has one
  const int64_t cg_first = CODEC == 0 ? static_cast<int64_t>(h) * kD / a.group_size : 0;
  const int n_cg = CODEC == 0 ? static_cast<int>((static_cast<int64_t>(h) * kD + kD - 1) / a.group_size - cg_first + 1) : 1;
  const int64_t vgroups = CODEC == 0 ? (C + a.group_size - 1) / a.group_size : 1;
  // this thread's fill units: K and KIVI V: key octet tid & 15 of dims (tid >> 4) + 16 r;
  // KVQuant V: dim octet tid & 15 of keys (tid >> 4) + 16 r
  const int u_lo = tid & 15, u_hi = tid >> 4;
  // stream bounds are read from the parameters where used (no registers held across the loop)
#define SYM_S_LO(k) reinterpret_cast<uintptr_t>(a.stream[k])
#define SYM_S_HI(k) reinterpret_cast<uintptr_t>(a.stream_end[k])
  constexpr float bias = sym_bias<kBf16>(SLOT);  // symbol tiles hold bias + s
  const uint32_t mask4 = static_cast<uint32_t>(a.sym_mask & 0xF) * 0x01010101u;
  // warps 4..7 stage: thread st = tid - 128 copies words e = st + 128 k of the [128][rw]
  // staged runs, e = dim * rw + i advanced without division (128 = q128 * rw + r128)
  constexpr int kStageThreads = kThreadsA / 2;
  const int st = tid - kStageThreads;
  constexpr int q128 = kStageThreads / rw, r128 = kStageThreads % rw;
  const int st_d0 = st >= 0 ? st / rw : 0, st_i0 = st >= 0 ? st % rw : 0;

  // Stage the words tile kt decodes (warps 4..7; one cp.async group per thread). Per dim run, the
  // 4 * slot + 1 words that hold the tile's 128 symbols (K; KIVI V) or the 512 * slot + 1
  // words of the head's 128 x 128 symbols (KVQuant V); the key groups' scale / zero rows
  // (KIVI); each body key's value scale / zero. Words outside a stream are skipped: their
  // bits belong to no body key of the tile.
  auto stage = [&](int kt) {
    const SymTile t = sym_tile<CODEC>(a, kt, kmax);
    {  // paged-cache keys (at or past the prefix): their rows through the block table
      const int64_t key = t.k0 + st;
      if (key >= a.prefix && key <= kmax) {
        const int64_t bi = key / a.block_size;
        const int64_t pb = __ldg(a.block_table + bi);
        rowsfx[st] = (pb < 0 || pb >= a.num_blocks)
                         ? -1
                         : pb * a.block_stride + (key - bi * a.block_size) * a.token_stride + static_cast<int64_t>(h) * kD;
      }
    }
    if (!t.has_body) return;
    const int64_t koff = CODEC == 0 ? t.k0 - a.sink : t.k0;  // stream token of the tile's key 0
    {  // K runs: dim d starts at bit s_lo * 8 + ((d * H + h) * run + koff) * slot
      const int64_t step = static_cast<int64_t>(a.kv_heads) * run * slot;  // bits between dim runs
      int64_t bit = static_cast<int64_t>(SYM_S_LO(0)) * 8 + (static_cast<int64_t>(st_d0 * a.kv_heads + h) * run + koff) * slot;
      int i = st_i0;
#pragma unroll 1
      for (int e = st; e < 128 * rw; e += kStageThreads) {
        const uintptr_t wa = static_cast<uintptr_t>(bit >> 5) * 4 + 4u * static_cast<uint32_t>(i);
        if (wa + 4 > SYM_S_LO(0) && wa < SYM_S_HI(0)) cp_async4(rawk + e, wa);
        i += r128;
        bit += q128 * step;
        if (i >= rw) {
          i -= rw;
          bit += step;
        }
      }
    }
    if (CODEC == 0) {  // KIVI V runs: dim d starts at bit s_lo * 8 + ((h * 128 + d) * body + koff) * slot
      const int64_t step = a.body * slot;
      int64_t bit = static_cast<int64_t>(SYM_S_LO(1)) * 8 + ((static_cast<int64_t>(h) * kD + st_d0) * a.body + koff) * slot;
      int i = st_i0;
#pragma unroll 1
      for (int e = st; e < 128 * rw; e += kStageThreads) {
        const uintptr_t wa = static_cast<uintptr_t>(bit >> 5) * 4 + 4u * static_cast<uint32_t>(i);
        if (wa + 4 > SYM_S_LO(1) && wa < SYM_S_HI(1)) cp_async4(rawv + e, wa);
        i += r128;
        bit += q128 * step;
        if (i >= rw) {
          i -= rw;
          bit += step;
        }
      }
    } else {
      const int64_t bit = static_cast<int64_t>(SYM_S_LO(1)) * 8 + (static_cast<int64_t>(h) * a.prefix + t.k0) * kD * slot;
      const uintptr_t w0 = static_cast<uintptr_t>(bit >> 5) * 4;
      const int nw = 512 * slot + 1;
#pragma unroll 1
      for (int e = st; e < nw; e += kStageThreads) {
        const uintptr_t wa = w0 + 4u * static_cast<uint32_t>(e);
        if (wa + 4 > SYM_S_LO(1) && wa < SYM_S_HI(1)) cp_async4(rawv + e, wa);
      }
    }
    if (CODEC == 0) {  // key group rows: [gi][scale, zero][65 words]
#pragma unroll 1
      for (int e = st; e < t.n_g * 2 * kMetaWords; e += kStageThreads) {
        const int gi = e / (2 * kMetaWords), r = e - gi * 2 * kMetaWords;
        const int side = r >= kMetaWords ? 1 : 0, i = r - side * kMetaWords;
        const uintptr_t A = reinterpret_cast<uintptr_t>(side ? a.zero[0] : a.scale[0]) +
                            2 * static_cast<uintptr_t>((t.g_lo + gi) * C + static_cast<int64_t>(h) * kD);
        if (i < 64 + ((A & 3) ? 1 : 0)) cp_async4(kmw + e, (A & ~static_cast<uintptr_t>(3)) + 4u * i);
      }
    }
    {  // value scale / zero of the body keys: key k0 + st
      const int64_t key = t.k0 + st;
      if (key >= t.b_lo && key < t.b_hi) {
        const int64_t idx = CODEC == 0 ? (key - a.sink) * vgroups + cg_first : key;
#pragma unroll
        for (int side = 0; side < 2; ++side) {
          const uintptr_t A = reinterpret_cast<uintptr_t>(side ? a.zero[1] : a.scale[1]) + 2 * static_cast<uintptr_t>(idx);
          const uintptr_t A4 = A & ~static_cast<uintptr_t>(3);
          cp_async4(vmw + (st * 2 + side) * 2, A4);
          if ((A & 3) + 2 * (CODEC == 0 ? n_cg : 1) > 4) cp_async4(vmw + (st * 2 + side) * 2 + 1, A4 + 4);
        }
      }
    }
  };

  // Programmatic dependent launch: the next kernel on the stream may start its own setup
  // now; this one sets up shared memory and TMEM, then waits for the kernels before it
  // (their results, the workspace they share) before its first global access. Without the
  // launch attribute both instructions are no-ops.
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
    *fail_flag = 0u;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tslot)),
                 "r"(kSymTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  // byte table, zeroed B blocks of the groups and channel groups, per-row causal ends,
  // running sums
  if constexpr (kBf16 && SLOT == 8)  // the byte table serves bf16 8-bit symbols only
    lut[tid] = sym_lut_entry<QT>(static_cast<uint32_t>(tid), slot, static_cast<uint32_t>((1 << a.sym_len) - 1));
  for (int e = tid; e < (kSymMaxG * kRowTile) / 16; e += kThreadsA)
    reinterpret_cast<uint4*>(bq_sm)[e] = make_uint4(0u, 0u, 0u, 0u);
  for (int e = tid; e < (kSymMaxC * kRowTile) / 16; e += kThreadsA)
    reinterpret_cast<uint4*>(ps_sm)[e] = make_uint4(0u, 0u, 0u, 0u);
  if (tid < NQ) {
    const int row = row0 + tid;
    m_run[tid] = -INFINITY;
    l_run[tid] = 0.f;
    cend[tid] = row < a.rows ? min(a.seq_len - 1, a.q_start + row / a.group) : -1;
  }
  if (tid < 10 * NQ) cz[tid] = 0.f;  // cz, zacc, cs
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  // first tile's staged words; q rows (real block)
  if (warp >= 4) {
    if (t_begin < t_end) stage(t_begin);
    cp_async_commit();
  }
  uint8_t* bq_real = bq_sm + kSymReal * kRowTile;
  if (tid < NQ * 16) {
    const int n = tid >> 4, c = tid & 15;
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
    *reinterpret_cast<uint4*>(bq_real + c * kLBO + n * 16) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  __syncthreads();
  // B operands of a key group: threads 0..127 write q (.) scale (one 8-dim chunk c of one
  // row n each), threads 128..255 sum q . zero over the row into cz
  const bool zero_side = tid >= 128;
  const int qb_n = (tid & 127) >> 4, qb_c = tid & 15;
  const __half* qb_meta = zero_side ? a.zero[0] : a.scale[0];
  const bool kmis = (reinterpret_cast<uintptr_t>(qb_meta) & 3) != 0;  // group rows start 2 bytes into a word
  auto build_qb = [&](int gi, uint4 mv) {
    const uint4 qv = *reinterpret_cast<const uint4*>(bq_real + qb_c * kLBO + qb_n * 16);
    const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
    const uint32_t mw[4] = {mv.x, mv.y, mv.z, mv.w};
    if (!zero_side) {  // q (.) scale, and its sum over the row (the bias of the symbols)
      uint32_t o[4];
      float qs = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&mw[k]));
        const float q0 = bits_to_float(static_cast<uint16_t>(qw[k] & 0xFFFFu), kBf16);
        const float q1 = bits_to_float(static_cast<uint16_t>(qw[k] >> 16), kBf16);
        o[k] = pack2<QT>(q0 * f.x, q1 * f.y);
        qs += bits_to_float(static_cast<uint16_t>(o[k] & 0xFFFFu), kBf16) + bits_to_float(static_cast<uint16_t>(o[k] >> 16), kBf16);
      }
      *reinterpret_cast<uint4*>(bq_sm + gi * kRowTile + qb_c * kLBO + qb_n * 16) = make_uint4(o[0], o[1], o[2], o[3]);
#pragma unroll
      for (int x = 1; x < 16; x <<= 1) qs += __shfl_xor_sync(0xffffffffu, qs, x);
      if (qb_c == 0) cs[gi * NQ + qb_n] = qs;
    } else {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&mw[k]));
        acc = __fmaf_rn(bits_to_float(static_cast<uint16_t>(qw[k] & 0xFFFFu), kBf16), f.x, acc);
        acc = __fmaf_rn(bits_to_float(static_cast<uint16_t>(qw[k] >> 16), kBf16), f.y, acc);
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (qb_c == 0) cz[gi * NQ + qb_n] = acc;
    }
  };
  if (CODEC == 1) build_qb(0, load8h(qb_meta, static_cast<int64_t>(h) * kD + 8 * qb_c, a.meta_vec != 0));
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
    const SymTile t = sym_tile<CODEC>(a, kt, kmax);
    const int64_t k0 = t.k0;
    const int n_g = t.n_g;
    const uint32_t koff = static_cast<uint32_t>(CODEC == 0 ? k0 - a.sink : k0);  // low bits suffice below
    cp_async_wait_all();
    __syncthreads();  // this tile's staged words are visible to every thread

    // K tile (MMA 1 of the previous tile has completed): body units from the staged runs
    // through the byte table, keys contiguous; other octets as 8 x 8 blocks transposed to
    // keys-contiguous
    // body octets of the tile (octet o = keys k0 + 8 o ..): [ob_lo, ob_hi)
    const int ob_lo = static_cast<int>((t.b_lo - k0 + 7) >> 3);
    const int ob_hi = t.has_body ? static_cast<int>((t.b_hi - k0) >> 3) : 0;
    // this thread's body octets among octets 8 kh .. 8 kh + 7 of its dim dd
    const int kh = tid >> 7, dd = tid & 127;
    uint32_t octs = 0u;
    {
      const int lo = max(ob_lo - 8 * kh, 0), hi = min(ob_hi - 8 * kh, 8);
      if (hi > lo) octs = ((0xFFu >> (8 - (hi - lo))) << lo) & 0xFFu;
    }
    if (octs) {
      const uint32_t b0 = static_cast<uint32_t>(SYM_S_LO(0)) * 8u +
                          (static_cast<uint32_t>(dd * a.kv_heads + h) * static_cast<uint32_t>(run) + koff) *
                              static_cast<uint32_t>(slot);
      const uint32_t pos0 = (b0 & 31u) + 64u * static_cast<uint32_t>(kh * slot);
      const uint32_t* src = rawk + dd * rw + (pos0 >> 5);
      uint8_t* dst = kt_sm + 8 * kh * kSBO + (dd >> 3) * kLBO + (dd & 7) * 16;
      decode_half_run<SLOT, kBf16>(src, pos0 & 31u, octs, dst, kSBO, lut, mask4);
    }
    {
      const int dq = u_lo, ko = u_hi;  // the 8 x 8 block (dims 8 dq.., keys 8 ko..) of this thread
      const int64_t kb = k0 + 8 * ko;
      if (ko < ob_lo || ko >= ob_hi) {
        uint32_t m[8][4];
        real_rows8<QT, CODEC>(a, 0, h, kb, dq, kmax, bias, rowsfx, k0, m);
        transpose8x8_u16(m);  // rows per dim
#pragma unroll
        for (int i = 0; i < 8; ++i)
          *reinterpret_cast<uint4*>(kt_sm + ko * kSBO + dq * kLBO + i * 16) = make_uint4(m[i][0], m[i][1], m[i][2], m[i][3]);
      }
    }
    // B operands of this tile's key groups (their previous reader, MMA 1, is done)
    if (CODEC == 0) {
#pragma unroll
      for (int gi = 0; gi < kSymMaxG; ++gi) {
        if (gi < n_g) {
          const uint32_t* w = kmw + (gi * 2 + (zero_side ? 1 : 0)) * kMetaWords + 4 * qb_c;
          const uint4 mv = kmis ? make_uint4(__funnelshift_r(w[0], w[1], 16), __funnelshift_r(w[1], w[2], 16),
                                             __funnelshift_r(w[2], w[3], 16), __funnelshift_r(w[3], w[4], 16))
                                : make_uint4(w[0], w[1], w[2], w[3]);
          build_qb(gi, mv);
        }
      }
    }
    // this key's S block and value-side multipliers from the staged metadata
    const int64_t key = k0 + tid;
    int blk = kSymReal;
    float vsc[kSymMaxC] = {1.f, 1.f}, vze[kSymMaxC] = {0.f, 0.f};
    if (warp < 4 && key >= t.b_lo && key < t.b_hi) {
      const int64_t bt = CODEC == 0 ? key - a.sink : key;
      blk = CODEC == 0 ? static_cast<int>(static_cast<uint32_t>(bt) / static_cast<uint32_t>(a.group_size) -
                                          static_cast<uint32_t>(t.g_lo))
                       : 0;
      const int64_t idx = CODEC == 0 ? bt * vgroups + cg_first : key;
      const uint32_t os = static_cast<uint32_t>((reinterpret_cast<uintptr_t>(a.scale[1]) + 2 * idx) & 3);
      const uint32_t oz = static_cast<uint32_t>((reinterpret_cast<uintptr_t>(a.zero[1]) + 2 * idx) & 3);
      const uint8_t* ps8 = reinterpret_cast<const uint8_t*>(vmw + tid * 4) + os;
      const uint8_t* pz8 = reinterpret_cast<const uint8_t*>(vmw + tid * 4 + 2) + oz;
#pragma unroll
      for (int c = 0; c < kSymMaxC; ++c) {
        if (c < n_cg) {
          vsc[c] = __half2float(*reinterpret_cast<const __half*>(ps8 + 2 * c));
          vze[c] = __half2float(*reinterpret_cast<const __half*>(pz8 + 2 * c));
        }
      }
    }
    if (j > 0) {  // V^T tile and the P operands: MMA 2 of the previous tile
      const bool ok = mbar_wait_bounded(&bars[1], ph2);
      ph2 ^= 1u;
      if (__syncthreads_or(!ok)) {
        failed = true;
        break;
      }
    }
    // V^T tile from the staged words: KIVI K-major (one dim run per thread, keys
    // contiguous), KVQuant MN-major (dim octet u_lo of keys u_hi + 16 r)
    if (CODEC == 0) {
      if (octs) {
        const uint32_t b0 = static_cast<uint32_t>(SYM_S_LO(1)) * 8u +
                            (static_cast<uint32_t>(h * kD + dd) * static_cast<uint32_t>(a.body) + koff) *
                                static_cast<uint32_t>(slot);
        const uint32_t pos0 = (b0 & 31u) + 64u * static_cast<uint32_t>(kh * slot);
        const uint32_t* src = rawv + dd * rw + (pos0 >> 5);
        uint8_t* dst = vt_sm + (dd >> 3) * kSBO + 8 * kh * kLBO + (dd & 7) * 16;
        decode_half_run<SLOT, kBf16>(src, pos0 & 31u, octs, dst, kLBO, lut, mask4);
      }
    } else if (ob_hi > ob_lo) {
      const uint32_t b0 = static_cast<uint32_t>(SYM_S_LO(1)) * 8u +
                          static_cast<uint32_t>((static_cast<int64_t>(h) * a.prefix + k0) * kD) * static_cast<uint32_t>(slot);
      decode_kvq_v<SLOT, kBf16>(rawv, b0 & 31u, u_lo, u_hi, ob_lo, ob_hi, vt_sm, lut, mask4);
    }
    {
      const int dq = u_lo, ko = u_hi;
      const int64_t kb = k0 + 8 * ko;
      if (ko < ob_lo || ko >= ob_hi) {
        uint32_t m[8][4];
        real_rows8<QT, CODEC>(a, 1, h, kb, dq, kmax, bias, rowsfx, k0, m);  // rows per key
        if (CODEC == 0) transpose8x8_u16(m);              // K-major V^T: rows per dim
#pragma unroll
        for (int i = 0; i < 8; ++i)
          *reinterpret_cast<uint4*>(vt_sm + dq * kSBO + ko * kLBO + i * 16) = make_uint4(m[i][0], m[i][1], m[i][2], m[i][3]);
      }
    }
    proxy_fence();
    tc_fence_before();
    __syncthreads();  // tiles and B operands written; the staged words are free
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int s = 0; s < kD / 16; ++s)
        mma_f16(tmem, smem_desc(smem_u32(kt_sm) + 2 * s * kLBO), smem_desc(smem_u32(bq_sm) + 2 * s * kLBO), idesc_s,
                s > 0 ? 1u : 0u);
      mma_commit(&bars[0]);
    }
    // warps 4..7 stage tile kt + 1 while warps 0..3 wait for S and run the softmax
    bool s_ok = true;
    if (warp >= 4) {
      if (kt + 1 < t_end) stage(kt + 1);
      cp_async_commit();
    } else {
      s_ok = !named_sync_or_softmax(!mbar_wait_bounded(&bars[0], ph1));
      if (!s_ok && tid == 0) *fail_flag = 1u;
      tc_fence_after();
    }
    ph1 ^= 1u;

    if (warp < 4 && s_ok) {
      // S^T row of this key from its block (the same columns of every block are loaded by
      // the whole warp, then each lane keeps its own), plus q . zero of its key group
      float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int gi = 0; gi < n_g; ++gi) {
        float v[8];
        tmem_ld8(tmem + lane_base + 8 * gi, v);
        if (blk == gi)
#pragma unroll
          for (int n = 0; n < 8; ++n) s[n] = v[n];
      }
      if (t.has_real) {
        float v[8];
        tmem_ld8(tmem + lane_base + 8 * kSymReal, v);
        if (blk == kSymReal)
#pragma unroll
          for (int n = 0; n < 8; ++n) s[n] = v[n];
      }
      if (blk < kSymReal)
#pragma unroll
        for (int n = 0; n < 8; ++n) s[n] += cz[blk * NQ + n] - bias * cs[blk * NQ + n];
      float x[8];
#pragma unroll
      for (int n = 0; n < 8; ++n) x[n] = key <= cend[n] ? s[n] * a.scale_log2 : -INFINITY;
      const int ridx = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
      {
        const float r = warp_reduce8<true>(x, lane);
        if ((lane & 3) == 0) red[warp * NQ + ridx] = r;
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
      // P (.) vscale_c into the B operand; per row, sum p * vzero minus bias times the
      // rounded P (.) vscale of the body keys (their V values carry the bias)
      const float kbias = blk == kSymReal ? 0.f : bias;
      float p[8], z0[8], z1[8];
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        p[n] = x[n] == -INFINITY ? 0.f : exp2f(x[n] - m_new[n]);
        float pr[kSymMaxC] = {0.f, 0.f};
#pragma unroll
        for (int c = 0; c < kSymMaxC; ++c) {
          if (c < n_cg) {
            const uint16_t u = from_float<QT>(p[n] * vsc[c]);
            *reinterpret_cast<uint16_t*>(ps_sm + c * kRowTile + tile_off(n, tid)) = u;
            pr[c] = bits_to_float(u, kBf16);
          }
        }
        z0[n] = __fmaf_rn(p[n], vze[0], -kbias * pr[0]);
        z1[n] = __fmaf_rn(p[n], vze[1], -kbias * pr[1]);
      }
      {
        const float r = warp_reduce8<false>(p, lane);
        const float r0 = warp_reduce8<false>(z0, lane);
        const float r1 = n_cg > 1 ? warp_reduce8<false>(z1, lane) : 0.f;
        if ((lane & 3) == 0) {
          red[warp * NQ + ridx] = r;
          redz[warp * NQ + ridx] = r0;
          redz[4 * NQ + warp * NQ + ridx] = r1;
        }
      }
      named_sync_softmax();
      if (tid < NQ) {
        l_run[tid] = l_run[tid] * alpha[tid] + (red[tid] + red[NQ + tid]) + (red[2 * NQ + tid] + red[3 * NQ + tid]);
        m_run[tid] = m_new[tid];
      } else if (tid >= 32 && tid < 32 + kSymMaxC * NQ) {
        const int c = (tid - 32) >> 3, n = tid & 7;
        const float* rz = redz + c * 4 * NQ;
        zacc[c * NQ + n] = zacc[c * NQ + n] * alpha[n] + ((rz[n] + rz[NQ + n]) + (rz[2 * NQ + n] + rz[3 * NQ + n]));
      }
    }
    const bool rescale = __syncthreads_or(tid < NQ && alpha[tid] != 1.f) && j > 0;
    if (*fail_flag) {
      failed = true;
      break;
    }
    if (warp >= 4 && rescale) {
      for (int c = 0; c < n_cg; ++c) {
        float o[8];
        tmem_ld8(tmem + lane_base + kSymOCol + 8 * c, o);
#pragma unroll
        for (int n = 0; n < 8; ++n) o[n] *= alpha[n];
        tmem_st8(tmem + lane_base + kSymOCol + 8 * c, o);
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
        mma_f16(tmem + kSymOCol, smem_desc(smem_u32(vt_sm) + 2 * s * kLBO), smem_desc(smem_u32(ps_sm) + 2 * s * kLBO),
                idesc_o, (j > 0 || s > 0) ? 1u : 0u);
      mma_commit(&bars[1]);
    }
  }
  cp_async_wait_all();  // no copy outlives the loop (a failed wait leaves the next tile's in flight)
  const bool any_tiles = t_end > t_begin;
  if (!failed && any_tiles) {
    const bool ok = mbar_wait_bounded(&bars[1], ph2);
    ph2 ^= 1u;
    failed = __syncthreads_or(!ok);
  }
  if (failed) {
    if (tid == 0 && a.err) atomicOr(a.err, kWaitTimeoutFlag);
    mbar_wait_bounded(&bars[0], ph1 ^ 1u);
    mbar_wait_bounded(&bars[1], ph2 ^ 1u);
  } else {
    tc_fence_after();
    // this lane's dim reads the O block of its value channel group, plus that group's
    // running sum of p * value zero
    const int d = (warp & 3) * 32 + lane;
    const int cidx = CODEC == 0 ? static_cast<int>((static_cast<int64_t>(h) * kD + d) / a.group_size - cg_first) : 0;
    float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (warp >= 4 && any_tiles) {
      for (int c = 0; c < n_cg; ++c) {
        float v[8];
        tmem_ld8(tmem + lane_base + kSymOCol + 8 * c, v);
        if (c == cidx)
#pragma unroll
          for (int n = 0; n < 8; ++n) o[n] = v[n];
      }
#pragma unroll
      for (int n = 0; n < 8; ++n) o[n] += zacc[cidx * NQ + n];
    }
    if (a.splits == 1) {
      if (warp >= 4) {
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const int row = row0 + n;
          if (row < a.rows) {
            const int64_t q = row / a.group;
            const int64_t qh = static_cast<int64_t>(h) * a.group + row % a.group;
            a.output[(q * a.q_heads + qh) * kD + d] = from_float<QT>(o[n] / l_run[n]);
          }
        }
      }
    } else {
      const int64_t blkid = (static_cast<int64_t>(h) * a.row_blocks + rb) * a.splits + sp;
      if (warp >= 4) {
#pragma unroll
        for (int n = 0; n < 8; ++n) a.ws_o[(blkid * NQ + n) * kD + d] = o[n];
      }
      if (tid < NQ) {
        a.ws_ml[(blkid * NQ + tid) * 2] = m_run[tid];
        a.ws_ml[(blkid * NQ + tid) * 2 + 1] = l_run[tid];
      }
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        const uint32_t prev = atomicInc(&a.counters[static_cast<int64_t>(h) * a.row_blocks + rb],
                                        static_cast<uint32_t>(a.splits - 1));
        *last_flag = prev == static_cast<uint32_t>(a.splits - 1) ? 1u : 0u;
      }
      __syncthreads();
      if (*last_flag) split_merge<QT, NQ>(a, h, rb, row0, reinterpret_cast<float*>(kt_sm));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kSymTmemCols));
  }
#undef SYM_S_LO
#undef SYM_S_HI
}

}  // namespace origami
