/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle for the origami_b200 hot path.
 *
 * A plain-C restatement of Origami's layout / bitpack path used as the parity checker
 * by tests/, __graft_entry__.smoke() and bench.py's CPU baseline. Nothing in the
 * product (origami_b200/) links or calls it.
 *
 * Parity pins:
 *   - canonical unpack restates csrc/origami/bitpack_layout_cuda.cu:70-128
 *     (unpack_symbol + unpack_canonical_kernel) with the zero-filled output of
 *     bitpack_layout_cuda.cpp:367-374 and the source layout of cpp:84-147 / cu:52-68;
 *     it is checked against the reference kernel itself on the B200 (tests/golden);
 *   - canonical pack is the exact inverse (the reference ships only a stub,
 *     lossless/native_cpu.py:137-151): dense LSB-first symbols, ceil(n*bits/8)
 *     bytes per chunk (cpp:183-185), pad bits zero;
 *   - gather / scatter restate torch.index_select / index_copy_ along the block
 *     dimension (worker.py:1881-1897, benchmark_utils.py:434-444);
 *   - the plane split (x >> shift) & mask is new arithmetic with no reference
 *     counterpart: parity unpinned, invariant merge(split(x)) == x.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_OK 0
#define ORACLE_BAD -1

void oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* bitpack_layout_cuda.cu:70-89 */
static uint8_t unpack_symbol(const uint8_t* src, int64_t src_bytes, int64_t symbol_index, int bits) {
  if (bits == 8) return src[symbol_index];
  const int64_t bit_pos = symbol_index * (int64_t)bits;
  const int64_t byte_idx = bit_pos >> 3;
  const int shift = (int)(bit_pos & 7);
  uint16_t packed = 0;
  if (byte_idx < src_bytes) packed = src[byte_idx];
  if (byte_idx + 1 < src_bytes) packed = (uint16_t)(packed | ((uint16_t)src[byte_idx + 1] << 8));
  return (uint8_t)((packed >> shift) & ((1u << bits) - 1u));
}

/* Row-major strides of the source shape (cpp:103-106) and source_index (cu:52-68). */
static void strides_of(const int64_t* shape, int rank, int64_t* stride) {
  stride[rank - 1] = 1;
  for (int i = rank - 2; i >= 0; --i) stride[i] = stride[i + 1] * shape[i + 1];
}

static int64_t source_index(const int64_t* stride, const int64_t* axes, int rank, int64_t t, int64_t h, int64_t c) {
  int64_t coords[4] = {0, 0, 0, 0};
  coords[axes[0]] = t;
  coords[axes[1]] = h;
  coords[axes[2]] = c;
  if (axes[3] != -1) coords[axes[3]] = 0;
  int64_t index = 0;
  for (int a = 0; a < rank; ++a) index += coords[a] * stride[a];
  return index;
}

static int64_t numel_of(const int64_t* shape, int rank) {
  int64_t n = 1;
  for (int i = 0; i < rank; ++i) n *= shape[i];
  return n;
}

/* unpack_canonical_kernel (cu:91-128) over every chunk, output pre-zeroed (cpp:370-374). */
int oracle_unpack_canonical(const uint8_t* flat, const int64_t* offsets, const int64_t* bits, const int64_t* specs,
                            int64_t num_chunks, const int64_t* shape, int rank, const int64_t* axes, uint8_t* out) {
  int64_t stride[4];
  strides_of(shape, rank, stride);
  memset(out, 0, (size_t)numel_of(shape, rank));
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t k = 0; k < num_chunks; ++k) {
    const int64_t* r = specs + 6 * k;
    const int64_t token_span = r[5] - r[4];
    const int64_t channel_span = r[3] - r[2];
    const int64_t per_head = channel_span * token_span;
    const int64_t symbols = (r[1] - r[0]) * per_head;
    const uint8_t* src = flat + offsets[k];
    const int64_t src_bytes = offsets[k + 1] - offsets[k];
    const int b = (int)bits[k];
    for (int64_t local = 0; local < symbols; ++local) {
      const int64_t head_offset = local / per_head;
      const int64_t rem = local - head_offset * per_head;
      const int64_t channel_offset = rem / token_span;
      const int64_t token_offset = rem - channel_offset * token_span;
      out[source_index(stride, axes, rank, r[4] + token_offset, r[0] + head_offset, r[2] + channel_offset)] =
          unpack_symbol(src, src_bytes, local, b);
    }
  }
  return ORACLE_OK;
}

/* Inverse of the above: symbol `local` of chunk k goes to stream bits
 * [local*bits, (local+1)*bits) of the chunk, LSB first; pad bits are zero. */
int oracle_pack_canonical(const uint8_t* symbols, const int64_t* offsets, const int64_t* bits, const int64_t* specs,
                          int64_t num_chunks, const int64_t* shape, int rank, const int64_t* axes, uint8_t* flat) {
  int64_t stride[4];
  strides_of(shape, rank, stride);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t k = 0; k < num_chunks; ++k) {
    const int64_t* r = specs + 6 * k;
    const int64_t token_span = r[5] - r[4];
    const int64_t channel_span = r[3] - r[2];
    const int64_t per_head = channel_span * token_span;
    const int64_t n = (r[1] - r[0]) * per_head;
    const int b = (int)bits[k];
    const uint32_t mask = (1u << b) - 1u;
    uint8_t* dst = flat + offsets[k];
    memset(dst, 0, (size_t)(offsets[k + 1] - offsets[k]));
    for (int64_t local = 0; local < n; ++local) {
      const int64_t head_offset = local / per_head;
      const int64_t rem = local - head_offset * per_head;
      const int64_t channel_offset = rem / token_span;
      const int64_t token_offset = rem - channel_offset * token_span;
      const uint32_t s =
          symbols[source_index(stride, axes, rank, r[4] + token_offset, r[0] + head_offset, r[2] + channel_offset)] &
          mask;
      const int64_t bit_pos = local * b;
      const int64_t byte_idx = bit_pos >> 3;
      const int sh = (int)(bit_pos & 7);
      const uint32_t v = s << sh;
      dst[byte_idx] |= (uint8_t)(v & 0xFFu);
      if (sh + b > 8) dst[byte_idx + 1] |= (uint8_t)(v >> 8);
    }
  }
  return ORACLE_OK;
}

/* ---------------------------------------------------------------------------------
 * Paged cache geometry: layout 0 = [2, NB, bs, H, D], layout 1 = [NB, 2, bs, H, D].
 * ------------------------------------------------------------------------------- */
static int64_t row_offset(int layout, int64_t NB, int64_t bs, int64_t H, int64_t D, int kv, int64_t blk,
                          int64_t slot, int64_t h) {
  const int64_t slab = bs * H * D;
  const int64_t base = layout == 0 ? ((int64_t)kv * NB + blk) * slab : (blk * 2 + kv) * slab;
  return base + slot * H * D + h * D; /* in elements */
}

/* index_select(cache, block_dim, ids) (worker.py:1881-1897). */
int oracle_gather_blocks(const uint8_t* cache, int layout, int64_t NB, int64_t bs, int64_t H, int64_t D, int elem,
                         const int64_t* ids, int64_t nb, uint8_t* out) {
  const int64_t slab = bs * H * D * elem;
  for (int64_t j = 0; j < nb; ++j)
    if (ids[j] < 0 || ids[j] >= NB) return ORACLE_BAD;
#pragma omp parallel for
  for (int64_t j = 0; j < nb; ++j) {
    for (int kv = 0; kv < 2; ++kv) {
      const int64_t src = (layout == 0 ? ((int64_t)kv * NB + ids[j]) : (ids[j] * 2 + kv)) * slab;
      const int64_t dst = (layout == 0 ? ((int64_t)kv * nb + j) : (j * 2 + kv)) * slab;
      memcpy(out + dst, cache + src, (size_t)slab);
    }
  }
  return ORACLE_OK;
}

/* index_copy_(block_dim, ids, value) (benchmark_utils.py:434-444). */
int oracle_scatter_blocks(const uint8_t* in, int layout, int64_t NB, int64_t bs, int64_t H, int64_t D, int elem,
                          const int64_t* ids, int64_t nb, uint8_t* cache) {
  const int64_t slab = bs * H * D * elem;
  for (int64_t j = 0; j < nb; ++j)
    if (ids[j] < 0 || ids[j] >= NB) return ORACLE_BAD;
  for (int64_t j = 0; j < nb; ++j) {
    for (int kv = 0; kv < 2; ++kv) {
      const int64_t dst = (layout == 0 ? ((int64_t)kv * NB + ids[j]) : (ids[j] * 2 + kv)) * slab;
      const int64_t src = (layout == 0 ? ((int64_t)kv * nb + j) : (j * 2 + kv)) * slab;
      memcpy(cache + dst, in + src, (size_t)slab);
    }
  }
  return ORACLE_OK;
}

/* ---------------------------------------------------------------------------------
 * Plane format of one layer (new arithmetic, parity unpinned):
 *   for kv in {K, V}: x[t, h, c] = 16-bit element of token t < T read through the block
 *   table; for plane p: symbols (x >> shift[p]) & ((1 << bits[p]) - 1) in a [T, H, D]
 *   tensor, packed canonically with the layer's specs into component q = kv*P + p,
 *   chunk k = q*S + s at byte offset offsets[k].
 * ------------------------------------------------------------------------------- */
static void kv_tokens(const uint16_t* cache, int layout, int64_t NB, int64_t bs, int64_t H, int64_t D,
                      const int64_t* ids, int64_t T, int kv, uint16_t* x) {
#pragma omp parallel for
  for (int64_t t = 0; t < T; ++t) {
    const int64_t blk = ids[t / bs];
    memcpy(x + t * H * D, cache + row_offset(layout, NB, bs, H, D, kv, blk, t % bs, 0), (size_t)(H * D * 2));
  }
}

int oracle_pack_layer(const uint16_t* cache, int layout, int64_t NB, int64_t bs, int64_t H, int64_t D,
                      const int64_t* ids, int64_t T, int P, const int32_t* shift, const int32_t* bits,
                      const int64_t* specs, int64_t S, const int64_t* offsets, uint8_t* packed) {
  for (int64_t j = 0; j < (T + bs - 1) / bs; ++j)
    if (ids[j] < 0 || ids[j] >= NB) return ORACLE_BAD;
  const int64_t n = T * H * D;
  uint16_t* x = (uint16_t*)malloc((size_t)n * 2);
  uint8_t* sym = (uint8_t*)malloc((size_t)n);
  int64_t* chunk_bits = (int64_t*)malloc((size_t)S * 8);
  if (!x || !sym || !chunk_bits) {
    free(x); free(sym); free(chunk_bits);
    return ORACLE_BAD;
  }
  const int64_t shape[3] = {T, H, D};
  const int64_t axes[4] = {0, 1, 2, -1};
  for (int kv = 0; kv < 2; ++kv) {
    kv_tokens(cache, layout, NB, bs, H, D, ids, T, kv, x);
    for (int p = 0; p < P; ++p) {
      const uint32_t m = (1u << bits[p]) - 1u;
#pragma omp parallel for
      for (int64_t i = 0; i < n; ++i) sym[i] = (uint8_t)((x[i] >> shift[p]) & m);
      for (int64_t s = 0; s < S; ++s) chunk_bits[s] = bits[p];
      oracle_pack_canonical(sym, offsets + (int64_t)(kv * P + p) * S, chunk_bits, specs, S, shape, 3, axes, packed);
    }
  }
  free(x);
  free(sym);
  free(chunk_bits);
  return ORACLE_OK;
}

int oracle_restore_layer(const uint8_t* packed, int P, const int32_t* shift, const int32_t* bits,
                         const int64_t* specs, int64_t S, const int64_t* offsets, uint16_t* cache, int layout,
                         int64_t NB, int64_t bs, int64_t H, int64_t D, const int64_t* ids, int64_t T) {
  for (int64_t j = 0; j < (T + bs - 1) / bs; ++j)
    if (ids[j] < 0 || ids[j] >= NB) return ORACLE_BAD;
  const int64_t n = T * H * D;
  uint16_t* x = (uint16_t*)malloc((size_t)n * 2);
  uint8_t* sym = (uint8_t*)malloc((size_t)n);
  int64_t* chunk_bits = (int64_t*)malloc((size_t)S * 8);
  if (!x || !sym || !chunk_bits) {
    free(x); free(sym); free(chunk_bits);
    return ORACLE_BAD;
  }
  const int64_t shape[3] = {T, H, D};
  const int64_t axes[4] = {0, 1, 2, -1};
  for (int kv = 0; kv < 2; ++kv) {
    memset(x, 0, (size_t)n * 2);
    for (int p = 0; p < P; ++p) {
      for (int64_t s = 0; s < S; ++s) chunk_bits[s] = bits[p];
      oracle_unpack_canonical(packed, offsets + (int64_t)(kv * P + p) * S, chunk_bits, specs, S, shape, 3, axes, sym);
#pragma omp parallel for
      for (int64_t i = 0; i < n; ++i) x[i] = (uint16_t)(x[i] | ((uint16_t)sym[i] << shift[p]));
    }
#pragma omp parallel for
    for (int64_t t = 0; t < T; ++t) {
      const int64_t blk = ids[t / bs];
      memcpy(cache + row_offset(layout, NB, bs, H, D, kv, blk, t % bs, 0), x + t * H * D, (size_t)(H * D * 2));
    }
  }
  free(x);
  free(sym);
  free(chunk_bits);
  return ORACLE_OK;
}

/* ---------------------------------------------------------------------------------
 * Quantized restore paths (CacheGen, KIVI): restatements of
 *   cachegen_unpack_dequantize_to_kv_cache_kernel  (bitpack_layout_cuda.cu:348-423),
 *   cachegen_unpack_dequantize_kernel               (bitpack_layout_cuda.cu:141-185),
 *   kivi_dequantize_to_kv_cache_kernel             (bitpack_layout_cuda.cu:577-683).
 * The float steps are the reference's, one IEEE single operation each (this file is
 * compiled with -ffp-contract=off): CacheGen ((s - c) / c) * max, KIVI fmaf(s, scale,
 * zero) (nvcc contracts the reference's s * scale + zero into one fused multiply-add).
 * Pinned against the reference kernels' own outputs (tests/golden/ref_quant_vectors.npz).
 * ------------------------------------------------------------------------------- */
#include <math.h>

static uint32_t f32_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

static float bits_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* IEEE-754 binary16 -> binary32 (exact). */
float oracle_half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  if (exp == 0x1Fu) return bits_f32(sign | 0x7F800000u | (man << 13));
  if (exp != 0) return bits_f32(sign | ((exp + 112u) << 23) | (man << 13));
  if (man == 0) return bits_f32(sign);
  /* subnormal: value = man * 2^-24 */
  int e = -14;
  while ((man & 0x400u) == 0) {
    man <<= 1;
    --e;
  }
  man &= 0x3FFu;
  return bits_f32(sign | ((uint32_t)(e + 127) << 23) | (man << 13));
}

/* binary32 -> binary16, round to nearest even; NaN -> 0x7FFF (canonical). */
uint16_t oracle_float_to_half(float f) {
  const uint32_t u = f32_bits(f);
  const uint32_t sign = (u >> 16) & 0x8000u;
  const uint32_t a = u & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return 0x7FFFu;
  if (a >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* >= 65520 rounds to inf */
  if (a >= 0x38800000u) {                                     /* normal half */
    const uint32_t r = a - 0x38000000u;                       /* rebias exponent 127 -> 15 */
    const uint32_t q = r >> 13, rem = r & 0x1FFFu;
    const uint32_t out = q + (rem > 0x1000u || (rem == 0x1000u && (q & 1u)));
    return (uint16_t)(sign | out);
  }
  if (a < 0x33000000u) return (uint16_t)sign; /* below half the smallest subnormal */
  {
    /* subnormal half: value / 2^-24, rounded to nearest even */
    const uint32_t e = a >> 23;
    const uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
    const int shift = (int)(126 - e); /* m * 2^(e-150) / 2^-24 = m >> (126 - e), 14..24 */
    const uint32_t q = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    const uint32_t out = q + (rem > half || (rem == half && (q & 1u)));
    return (uint16_t)(sign | out);
  }
}

/* binary32 -> bfloat16, round to nearest even; NaN -> 0x7FFF (canonical). */
uint16_t oracle_float_to_bf16(float f) {
  const uint32_t u = f32_bits(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FFFu;
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

static float meta_at(const void* p, int is_half, int64_t i) {
  return is_half ? oracle_half_to_float(((const uint16_t*)p)[i]) : ((const float*)p)[i];
}

static uint16_t out_at(float v, int out_is_bf16) {
  return out_is_bf16 ? oracle_float_to_bf16(v) : oracle_float_to_half(v);
}

/* unpack_symbol_direct (cu:295-312): dense LSB-first, bytes past src_bytes read as 0 */
static uint8_t symbol_direct(const uint8_t* src, int64_t src_bytes, int64_t index, int bits) {
  if (bits == 8) return index < src_bytes ? src[index] : 0;
  const int64_t bit = index * bits, byte = bit >> 3;
  uint32_t w = byte < src_bytes ? src[byte] : 0u;
  if (byte + 1 < src_bytes) w |= (uint32_t)src[byte + 1] << 8;
  return (uint8_t)((w >> (bit & 7)) & ((1u << bits) - 1u));
}

/* The reference reads 8-bit symbols unchecked (src[index], cu:74-76 and 295-297): a short
 * 8-bit stream runs on into the rest of the bytestream. Narrower symbols stop at the
 * stream's own length. Past the bytestream (undefined in the reference) both read 0. */
static int64_t read_limit(int bits, int64_t stream_bytes, int64_t to_bytestream_end) {
  return bits == 8 ? to_bytestream_end : stream_bytes;
}

static int64_t cache_index(int blocks_first, int64_t num_cache_blocks, int64_t block_size, int64_t heads,
                           int64_t head_dim, int64_t blk, int64_t kv, int64_t offset, int64_t head, int64_t dim) {
  if (blocks_first) return ((((blk * 2 + kv) * block_size + offset) * heads + head) * head_dim + dim);
  return ((((kv * num_cache_blocks + blk) * block_size + offset) * heads + head) * head_dim + dim);
}

/* cu:348-423. Returns the number of (kv, token, head) rows skipped for bad block ids. */
int64_t oracle_cachegen_to_cache(const uint8_t* bytestream, int64_t bytestream_bytes, int64_t key_offset,
                                 int64_t key_bytes,
                                 int64_t value_offset, int64_t value_bytes, int key_bits, int value_bits,
                                 int64_t key_bins, int64_t value_bins, const void* max_key, const void* max_value,
                                 int max_is_half, uint16_t* cache, int out_is_bf16, int blocks_first,
                                 int64_t num_cache_blocks, const int64_t* block_ids, int64_t block_count,
                                 int64_t block_size, int64_t tokens, int64_t heads, int64_t head_dim) {
  const int64_t channels = heads * head_dim;
  int64_t skipped = 0;
  for (int64_t lb = 0; lb < block_count; ++lb) {
    for (int64_t kv = 0; kv < 2; ++kv) {
      for (int64_t off = 0; off < block_size; ++off) {
        const int64_t token = lb * block_size + off;
        if (token >= tokens) continue;
        const int64_t blk = block_ids[lb];
        if (blk < 0 || blk >= num_cache_blocks) {
          skipped += heads;
          continue;
        }
        const int is_value = kv != 0;
        const uint8_t* stream = bytestream + (is_value ? value_offset : key_offset);
        const int bits = is_value ? value_bits : key_bits;
        const int64_t stream_bytes =
            read_limit(bits, is_value ? value_bytes : key_bytes, bytestream_bytes - (is_value ? value_offset : key_offset));
        const int64_t bins = is_value ? value_bins : key_bins;
        const float center = (float)(bins / 2 - 1);
        const float max_abs = meta_at(is_value ? max_value : max_key, max_is_half, token);
        for (int64_t ch = 0; ch < channels; ++ch) {
          const uint8_t s = symbol_direct(stream, stream_bytes, token * channels + ch, bits);
          const float q = ((float)s - center) / center;
          const float value = q * max_abs;
          cache[cache_index(blocks_first, num_cache_blocks, block_size, heads, head_dim, blk, kv, off,
                            ch / head_dim, ch % head_dim)] = out_at(value, out_is_bf16);
        }
      }
    }
  }
  return skipped;
}

/* cu:141-185: fp16 output [layers, 2, heads, tokens, head_dim]. */
void oracle_cachegen_unpack(const uint8_t* bytestream, int64_t bytestream_bytes, const int64_t* offsets,
                            const int64_t* bits_per_layer,
                            const int64_t* key_bins, const int64_t* value_bins, const void* max_key,
                            const void* max_value, int max_is_half, uint16_t* out, int64_t layers, int64_t tokens,
                            int64_t heads, int64_t head_dim) {
  const int64_t channels = heads * head_dim;
  for (int64_t sidx = 0; sidx < 2 * layers; ++sidx) {
    const int is_value = sidx >= layers;
    const int64_t layer = is_value ? sidx - layers : sidx;
    const int bits = (int)bits_per_layer[sidx];
    const int64_t base = offsets[sidx];
    const int64_t len = read_limit(bits, offsets[sidx + 1] - base, bytestream_bytes - base);
    const int64_t bins = is_value ? value_bins[layer] : key_bins[layer];
    const float center = (float)(bins / 2 - 1);
    for (int64_t t = 0; t < tokens; ++t) {
      const float max_abs = meta_at(is_value ? max_value : max_key, max_is_half, layer * tokens + t);
      for (int64_t ch = 0; ch < channels; ++ch) {
        const uint8_t s = symbol_direct(bytestream + base, len, t * channels + ch, bits);
        const float value = (((float)s - center) / center) * max_abs;
        const int64_t h = ch / head_dim, d = ch % head_dim;
        out[(((layer * 2 + is_value) * heads + h) * tokens + t) * head_dim + d] = oracle_float_to_half(value);
      }
    }
  }
}

/* cu:577-683. Returns the number of (kv, token, head) rows skipped for bad block ids. */
int64_t oracle_kivi_to_cache(const uint8_t* bytestream, int64_t bytestream_bytes, int64_t key_offset,
                             int64_t key_bytes, int64_t value_offset,
                             int64_t value_bytes, int bits, int64_t group_size, int64_t sink_tokens,
                             const void* key_scale, const void* key_zero, const void* value_scale,
                             const void* value_zero, const void* key_sink, const void* value_sink, int meta_is_half,
                             uint16_t* cache, int out_is_bf16, int blocks_first, int64_t num_cache_blocks,
                             const int64_t* block_ids, int64_t block_count, int64_t block_size, int64_t tokens,
                             int64_t heads, int64_t head_dim) {
  const int64_t channels = heads * head_dim;
  const int64_t body_tokens = tokens - sink_tokens;
  const int64_t value_groups = (channels + group_size - 1) / group_size;
  int64_t skipped = 0;
  for (int64_t lb = 0; lb < block_count; ++lb) {
    for (int64_t kv = 0; kv < 2; ++kv) {
      for (int64_t off = 0; off < block_size; ++off) {
        const int64_t token = lb * block_size + off;
        if (token >= tokens) continue;
        const int64_t blk = block_ids[lb];
        if (blk < 0 || blk >= num_cache_blocks) {
          skipped += heads;
          continue;
        }
        const int is_value = kv != 0;
        for (int64_t ch = 0; ch < channels; ++ch) {
          const int64_t head = ch / head_dim, dim = ch % head_dim;
          float value;
          if (token < sink_tokens) {
            value = meta_at(is_value ? value_sink : key_sink, meta_is_half, token * channels + ch);
          } else {
            const int64_t bt = token - sink_tokens;
            const int64_t index = is_value ? ((head * head_dim + dim) * body_tokens + bt)
                                           : ((dim * heads + head) * body_tokens + bt);
            const uint8_t* stream = bytestream + (is_value ? value_offset : key_offset);
            const int64_t limit = read_limit(bits, is_value ? value_bytes : key_bytes,
                                             bytestream_bytes - (is_value ? value_offset : key_offset));
            const uint8_t s = symbol_direct(stream, limit, index, bits);
            int64_t m;
            if (is_value) m = bt * value_groups + ch / group_size;
            else m = (bt / group_size) * channels + ch;
            const float sc = meta_at(is_value ? value_scale : key_scale, meta_is_half, m);
            const float ze = meta_at(is_value ? value_zero : key_zero, meta_is_half, m);
            value = fmaf((float)s, sc, ze);
          }
          cache[cache_index(blocks_first, num_cache_blocks, block_size, heads, head_dim, blk, kv, off, head, dim)] =
              out_at(value, out_is_bf16);
        }
      }
    }
  }
  return skipped;
}

/* ---- fused prefix attention (cu:853-1091, cpp:716-890) ---------------------------- */

/* origami_fused_unpack_symbol (cu:853-871): 3-bit symbols are two nibbles per byte, low
 * nibble first; the other widths are dense (unpack_symbol_direct). */
static uint32_t fused_symbol(const uint8_t* src, int64_t src_bytes, int64_t index, int bits) {
  if (bits == 3) {
    const int64_t byte = index >> 1;
    if (byte >= src_bytes) return 0u;
    return (uint32_t)((src[byte] >> ((index & 1) * 4)) & 0x07);
  }
  return symbol_direct(src, src_bytes, index, bits);
}

typedef struct {
  const uint8_t* bytestream;
  int64_t key_offset, key_bytes, value_offset, value_bytes;
  int codec, bits;
  int64_t group_size, sink_tokens, prefix_tokens;
  const uint16_t *key_scale, *key_zero, *value_scale, *value_zero, *key_sink, *value_sink;
  const uint16_t* kv_cache;
  int cache_bf16, blocks_first;
  int64_t num_cache_blocks, block_size, kv_heads;
  const int32_t* block_table;
} fused_src;

static float h2f(uint16_t h) { return oracle_half_to_float(h); }

/* One K (kv = 0) or V (kv = 1) element as the reference kernel reads it (cu:936-972 and
 * 1017-1069), in fp32; s * scale + zero contracts to one fma as nvcc compiles it. */
static float fused_element(const fused_src* s, int kv, int64_t token, int64_t kv_head, int64_t dim) {
  const int64_t D = 128, channels = s->kv_heads * D, channel = kv_head * D + dim;
  if (token < s->prefix_tokens) {
    const uint8_t* st = s->bytestream + (kv ? s->value_offset : s->key_offset);
    const int64_t sb = kv ? s->value_bytes : s->key_bytes;
    if (s->codec == 0) {
      if (token < s->sink_tokens) return h2f((kv ? s->value_sink : s->key_sink)[token * channels + channel]);
      const int64_t body = s->prefix_tokens - s->sink_tokens, bt = token - s->sink_tokens;
      if (!kv) {
        const uint32_t sym = fused_symbol(st, sb, (dim * s->kv_heads + kv_head) * body + bt, s->bits);
        const int64_t m = (bt / s->group_size) * channels + channel;
        return fmaf((float)sym, h2f(s->key_scale[m]), h2f(s->key_zero[m]));
      }
      const int64_t groups = (channels + s->group_size - 1) / s->group_size;
      const uint32_t sym = fused_symbol(st, sb, (kv_head * D + dim) * body + bt, s->bits);
      const int64_t m = bt * groups + channel / s->group_size;
      return fmaf((float)sym, h2f(s->value_scale[m]), h2f(s->value_zero[m]));
    }
    if (!kv) {
      const uint32_t sym = fused_symbol(st, sb, (dim * s->kv_heads + kv_head) * s->prefix_tokens + token, s->bits);
      return fmaf((float)sym, h2f(s->key_scale[channel]), h2f(s->key_zero[channel]));
    }
    const uint32_t sym = fused_symbol(st, sb, (kv_head * s->prefix_tokens + token) * D + dim, s->bits);
    return fmaf((float)sym, h2f(s->value_scale[token]), h2f(s->value_zero[token]));
  }
  const int64_t pb = s->block_table[token / s->block_size];
  if (pb < 0 || pb >= s->num_cache_blocks) return 0.f;
  const int64_t off = token % s->block_size;
  const int64_t i = s->blocks_first ? ((((pb * 2 + kv) * s->block_size + off) * s->kv_heads + kv_head) * D + dim)
                                    : ((((kv * s->num_cache_blocks + pb) * s->block_size + off) * s->kv_heads + kv_head) * D + dim);
  const uint16_t b = s->kv_cache[i];
  return s->cache_bf16 ? bits_f32((uint32_t)b << 16) : h2f(b);
}

/* The reference kernel per (query token, query head): 4 warps score a 4-token tile (lane l
 * sums dims l, l+32, l+64, l+96 with fma, then the shuffle-down tree folds the lanes), one
 * thread updates the running max / sum with expf, and dim d accumulates
 * acc * old_weight + sum_w weight_w * v_w. */
void oracle_fused_prefix_attention(const uint8_t* bytestream, int64_t key_offset, int64_t key_bytes,
                                   int64_t value_offset, int64_t value_bytes, int codec, int bits, int64_t group_size,
                                   int64_t sink_tokens, const uint16_t* key_scale, const uint16_t* key_zero,
                                   const uint16_t* value_scale, const uint16_t* value_zero, const uint16_t* key_sink,
                                   const uint16_t* value_sink, const uint16_t* query, int query_bf16,
                                   const uint16_t* kv_cache, int cache_bf16, int blocks_first, int64_t num_cache_blocks,
                                   int64_t block_size, int64_t kv_heads, const int32_t* block_table,
                                   int64_t prefix_tokens, int64_t query_start, int64_t sequence_length,
                                   int64_t query_tokens, int64_t query_heads, float softmax_scale, uint16_t* output) {
  const fused_src s = {bytestream, key_offset, key_bytes, value_offset, value_bytes, codec, bits, group_size,
                       codec == 0 ? sink_tokens : 0, prefix_tokens, key_scale, key_zero, value_scale, value_zero,
                       key_sink, value_sink, kv_cache, cache_bf16, blocks_first, num_cache_blocks, block_size,
                       kv_heads, block_table};
  const int64_t D = 128, group = query_heads / kv_heads;
  const float NEG_INF = -__builtin_inff();
#pragma omp parallel for collapse(2) schedule(dynamic)
  for (int64_t qt = 0; qt < query_tokens; ++qt) {
    for (int64_t qh = 0; qh < query_heads; ++qh) {
      const int64_t kvh = qh / group;
      int64_t causal_end = query_start + qt;
      if (causal_end > sequence_length - 1) causal_end = sequence_length - 1;
      float q[128], acc[128];
      for (int64_t d = 0; d < D; ++d) {
        const uint16_t b = query[(qt * query_heads + qh) * D + d];
        q[d] = query_bf16 ? bits_f32((uint32_t)b << 16) : h2f(b);
        acc[d] = 0.f;
      }
      float run_max = NEG_INF, run_sum = 0.f;
      for (int64_t base = 0; base <= causal_end; base += 4) {
        float scores[4], weights[4];
        for (int w = 0; w < 4; ++w) {
          const int64_t token = base + w;
          if (token > causal_end) {
            scores[w] = NEG_INF;
            continue;
          }
          float lane[32];
          for (int l = 0; l < 32; ++l) {
            float dot = 0.f;
            for (int64_t d = l; d < D; d += 32) dot = fmaf(q[d], fused_element(&s, 0, token, kvh, d), dot);
            lane[l] = dot;
          }
          for (int off = 16; off > 0; off >>= 1) {
            float next[32];
            for (int l = 0; l < 32; ++l) next[l] = lane[l] + (l + off < 32 ? lane[l + off] : lane[l]);
            memcpy(lane, next, sizeof(lane));
          }
          scores[w] = lane[0] * softmax_scale;
        }
        float tile_max = scores[0];
        for (int w = 1; w < 4; ++w) tile_max = fmaxf(tile_max, scores[w]);
        const float next_max = fmaxf(run_max, tile_max);
        const float old_weight = expf(run_max - next_max);
        float tile_sum = 0.f;
        for (int w = 0; w < 4; ++w) {
          weights[w] = base + w <= causal_end ? expf(scores[w] - next_max) : 0.f;
          tile_sum += weights[w];
        }
        run_sum = fmaf(run_sum, old_weight, tile_sum);
        run_max = next_max;
        for (int64_t d = 0; d < D; ++d) {
          float tile_acc = 0.f;
          for (int w = 0; w < 4; ++w) {
            const int64_t token = base + w;
            if (token > causal_end) continue;
            tile_acc = fmaf(weights[w], fused_element(&s, 1, token, kvh, d), tile_acc);
          }
          acc[d] = fmaf(acc[d], old_weight, tile_acc);
        }
      }
      for (int64_t d = 0; d < D; ++d) output[(qt * query_heads + qh) * D + d] = out_at(acc[d] / run_sum, query_bf16);
    }
  }
}
