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
