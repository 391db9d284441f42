// C ABI of the quantized restore paths (declarations: include/origami_b200.h): the
// reference extension's argument checks (bitpack_layout_cuda.cpp:402-700, same messages),
// kernel selection and launches. Kernels: quant_kernels.cuh.
#include <algorithm>
#include <cstdint>

#include "host_common.h"
#include "quant_kernels.cuh"

namespace {

using namespace origami_host;

constexpr const char* kBitsMsg = "Origami CUDA bitpack supports only 1..8 bit symbols";

bool bits_ok(int64_t b) { return b >= 1 && b <= 8; }

// Bytes of a stream the kernels may read. The reference reads 8-bit symbols without a
// bounds check (unpack_symbol_direct, bitpack_layout_cuda.cu:295-297), so a short 8-bit
// stream continues into the bytes that follow it in the bytestream; narrower symbols stop
// at the stream's own length and read zeros past it. Past the bytestream both read zeros.
int64_t read_limit(int64_t bits, int64_t stream_bytes, int64_t to_bytestream_end) {
  return bits == 8 ? to_bytestream_end : stream_bytes;
}

// Paged-cache geometry for the to-cache ops (cpp:517-546): any 2-byte cache, aligned or
// not (unaligned caches take the scalar kernels).
int32_t cache_geom(const origami_paged_kv* kv, int32_t cache_dtype, PagedGeom& g) {
  if (cache_dtype != ORIGAMI_DTYPE_F16 && cache_dtype != ORIGAMI_DTYPE_BF16)
    return fail(ORIGAMI_ERR_INVALID, "kv_cache must be float16 or bfloat16");
  if (kv == nullptr || kv->d_data == nullptr) return fail(ORIGAMI_ERR_INVALID, "kv cache is null");
  if (kv->layout != ORIGAMI_KV_FIRST && kv->layout != ORIGAMI_BLOCKS_FIRST)
    return fail(ORIGAMI_ERR_INVALID,
                "kv_cache must be [num_blocks,2,block,heads,dim] or [2,num_blocks,block,heads,dim]");
  if (kv->elem_bytes != 2) return fail(ORIGAMI_ERR_INVALID, "kv_cache must be float16 or bfloat16");
  if (kv->num_blocks <= 0 || kv->num_heads <= 0 || kv->head_dim <= 0)
    return fail(ORIGAMI_ERR_INVALID, "kv cache dimensions must be positive");
  if (kv->block_size <= 0) return fail(ORIGAMI_ERR_INVALID, "kv_cache block size must be positive");
  const int64_t HD = kv->num_heads * kv->head_dim;
  const int64_t slab = kv->block_size * HD;
  g.token_stride = HD;
  g.head_stride = kv->head_dim;
  g.kv_stride = kv->layout == ORIGAMI_KV_FIRST ? kv->num_blocks * slab : slab;
  g.block_stride = kv->layout == ORIGAMI_KV_FIRST ? slab : 2 * slab;
  return ORIGAMI_OK;
}

int32_t check_blocks(const origami_paged_kv* kv, const int64_t* d_block_ids, int64_t num_ids, int64_t tokens) {
  if (num_ids <= 0 || d_block_ids == nullptr) return fail(ORIGAMI_ERR_INVALID, "block_ids must be non-empty");
  if (tokens > num_ids * kv->block_size) return fail(ORIGAMI_ERR_INVALID, "tokens exceed destination block capacity");
  return ORIGAMI_OK;
}

int32_t grid_for(const void* fn, int smem, int64_t want, int& grid) {
  int resident = 0;
  const int32_t rc = persistent_slots(fn, smem, resident);
  if (rc) return rc;
  grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, resident)));
  return ORIGAMI_OK;
}

// Launch with programmatic dependent launch: the kernel's CTAs may be scheduled while the
// kernel before it on the stream finishes; the kernel waits for it (griddepcontrol.wait)
// before touching global memory.
template <typename Args>
int32_t launch_dependent(void (*fn)(Args), int grid, int smem, cudaStream_t st, const Args& a, const char* what) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, a);
  if (e != cudaSuccess) return cuda_fail(e, what);
  return after_launch(what);
}

// ---------------------------------------------------------------------------------------
template <typename MAXT, typename OUT, bool VEC>
int32_t launch_cg(const origami::CgArgs& a, cudaStream_t st) {
  void (*fn)(origami::CgArgs) = origami::cachegen_to_cache<MAXT, OUT, VEC>;
  int grid = 0;
  const int32_t rc = grid_for(reinterpret_cast<const void*>(fn), 0, (2 * a.tokens + 7) / 8, grid);
  if (rc) return rc;
  return launch_dependent(fn, grid, 0, st, a, "cachegen_to_cache launch");
}

// Staged rows (symbols of at most 5 bits, 16-byte vector rows); null when the stages
// would not fit.
template <typename MAXT, typename OUT>
int32_t launch_cg_staged(const origami::CgArgs& a, const uint8_t* buf_end, cudaStream_t st, bool& launched) {
  launched = false;
  const int64_t rb = static_cast<int64_t>(a.nvec) * std::max(a.bits[0], a.bits[1]);
  const int stage_bytes = origami::CgStageGeo::bytes_for(rb);
  if (2LL * stage_bytes > 96 * 1024) return ORIGAMI_OK;
  void (*fn)(origami::CgArgs, int, const uint8_t*) = origami::cachegen_staged<MAXT, OUT>;
  const int smem = 2 * stage_bytes;
  int grid = 0;
  const int64_t groups = 2 * ((a.tokens + origami::kCgGroupRows - 1) / origami::kCgGroupRows);
  const int32_t rc = grid_for(reinterpret_cast<const void*>(fn), smem, groups, grid);
  if (rc) return rc;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  launched = true;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, a, stage_bytes, buf_end);
  if (e != cudaSuccess) return cuda_fail(e, "cachegen_staged launch");
  return after_launch("cachegen_staged launch");
}

template <typename MAXT, typename OUT>
int32_t launch_cg_vec(bool vec, const origami::CgArgs& a, const uint8_t* buf_end, cudaStream_t st) {
  if (vec && a.bits[0] <= 5 && a.bits[1] <= 5) {
    bool launched = false;
    const int32_t rc = launch_cg_staged<MAXT, OUT>(a, buf_end, st, launched);
    if (rc || launched) return rc;
  }
  return vec ? launch_cg<MAXT, OUT, true>(a, st) : launch_cg<MAXT, OUT, false>(a, st);
}

template <typename MAXT, bool VEC>
int32_t launch_cg_unpack(const origami::CgUnpackArgs& a, int64_t streams, cudaStream_t st) {
  void (*fn)(origami::CgUnpackArgs) = origami::cachegen_unpack<MAXT, VEC>;
  int resident = 0;
  const int32_t rc = persistent_slots(reinterpret_cast<const void*>(fn), 0, resident);
  if (rc) return rc;
  const int64_t rows = a.tokens * a.heads;
  const int64_t per_stream = std::max<int64_t>(1, 2 * resident / streams);
  const dim3 grid(static_cast<unsigned>(std::min<int64_t>({(rows + 7) / 8, per_stream, 65535})),
                  static_cast<unsigned>(streams));
  fn<<<grid, kThreads, 0, st>>>(a);
  return after_launch("cachegen_unpack launch");
}

// ---------------------------------------------------------------------------------------
// log2(v) when v is a power of two, else -1.
int32_t ilog2_exact(int64_t v) {
  if (v <= 0 || (v & (v - 1)) != 0) return -1;
  int32_t s = 0;
  while ((int64_t{1} << s) < v) ++s;
  return s;
}

template <typename META, typename OUT, int D, bool UNI>
int32_t launch_kivi_tiles(origami::KiviArgs a, cudaStream_t st) {
  using G = origami::KiviGeo<D, META>;
  void (*fn)(origami::KiviArgs) = origami::kivi_to_cache<META, OUT, D, UNI>;
  a.tiles_per_head = static_cast<int32_t>((a.tokens + G::TT - 1) / G::TT);
  const int64_t tiles = 2LL * a.H * a.tiles_per_head;
  if (tiles > 0x7FFFFFFF) return fail(ORIGAMI_ERR_UNSUPPORTED, "too many tiles");
  a.num_tiles = static_cast<int32_t>(tiles);
  int grid = 0;
  const int32_t rc = grid_for(reinterpret_cast<const void*>(fn), G::smem_bytes, tiles, grid);
  if (rc) return rc;
  return launch_dependent(fn, grid, G::smem_bytes, st, a, "kivi_to_cache launch");
}

template <typename META, typename OUT, int D>
int32_t launch_kivi2(origami::KiviArgs a, cudaStream_t st) {
  using G = origami::Kivi2Geo<D, META>;
  void (*fn)(origami::KiviArgs) = origami::kivi2_to_cache<META, OUT, D>;
  a.tiles_per_head = static_cast<int32_t>((a.tokens + G::TT - 1) / G::TT);
  const int64_t tiles = 2LL * a.H * a.tiles_per_head;
  if (tiles > 0x7FFFFFFF) return fail(ORIGAMI_ERR_UNSUPPORTED, "too many tiles");
  a.num_tiles = static_cast<int32_t>(tiles);
  int grid = 0;
  const int32_t rc = grid_for(reinterpret_cast<const void*>(fn), G::smem_bytes, tiles, grid);
  if (rc) return rc;
  return launch_dependent(fn, grid, G::smem_bytes, st, a, "kivi2_to_cache launch");
}

template <typename META, typename OUT>
int32_t launch_kivi(const origami::KiviArgs& a, bool tiled, cudaStream_t st) {
  if (tiled) {
    const bool uni = a.group_size % 8 == 0;
    const bool pow2_group = (a.group_size & (a.group_size - 1)) == 0;
    if (uni && pow2_group && a.bits == 2) {
      // 2-bit symbols (the KIVI default): table lookups without a transpose
      switch (a.D) {
        case 64: return launch_kivi2<META, OUT, 64>(a, st);
        case 128: return launch_kivi2<META, OUT, 128>(a, st);
        case 256: return launch_kivi2<META, OUT, 256>(a, st);
        default: break;
      }
    }
    switch (a.D) {
      case 64:
        return uni ? launch_kivi_tiles<META, OUT, 64, true>(a, st) : launch_kivi_tiles<META, OUT, 64, false>(a, st);
      case 128:
        return uni ? launch_kivi_tiles<META, OUT, 128, true>(a, st) : launch_kivi_tiles<META, OUT, 128, false>(a, st);
      case 256:
        return uni ? launch_kivi_tiles<META, OUT, 256, true>(a, st) : launch_kivi_tiles<META, OUT, 256, false>(a, st);
      default:
        break;
    }
  }
  void (*fn)(origami::KiviArgs) = origami::kivi_to_cache_elem<META, OUT>;
  int grid = 0;
  const int64_t total = 2 * a.tokens * static_cast<int64_t>(a.H) * a.D;
  const int32_t rc = grid_for(reinterpret_cast<const void*>(fn), 0, (total + kThreads - 1) / kThreads, grid);
  if (rc) return rc;
  fn<<<grid, kThreads, 0, st>>>(a);
  return after_launch("kivi_to_cache_elem launch");
}

}  // namespace

extern "C" {

int32_t origami_cachegen_unpack_dequantize_to_kv_cache(
    const uint8_t* d_bytestream, int64_t bytestream_bytes, int64_t key_offset, int64_t key_bytes,
    int64_t value_offset, int64_t value_bytes, int64_t key_bits, int64_t value_bits, int64_t key_bins,
    int64_t value_bins, const void* d_max_key, int64_t max_key_numel, const void* d_max_value,
    int64_t max_value_numel, int32_t max_dtype, const origami_paged_kv* cache, int32_t cache_dtype,
    const int64_t* d_block_ids, int64_t num_block_ids, int64_t tokens, uint32_t* d_error_count,
    origami_stream_t stream) {
  PagedGeom g{};
  if (cache_dtype != ORIGAMI_DTYPE_F16 && cache_dtype != ORIGAMI_DTYPE_BF16)
    return fail(ORIGAMI_ERR_INVALID, "kv_cache must be float16 or bfloat16");
  if (max_dtype != ORIGAMI_DTYPE_F16 && max_dtype != ORIGAMI_DTYPE_F32)
    return fail(ORIGAMI_ERR_INVALID, "max tensors must be float16 or float32");
  if (!bits_ok(key_bits) || !bits_ok(value_bits)) return fail(ORIGAMI_ERR_INVALID, kBitsMsg);
  if (cache == nullptr) return fail(ORIGAMI_ERR_INVALID, "kv cache is null");
  if (tokens <= 0 || cache->num_heads <= 0 || cache->head_dim <= 0)
    return fail(ORIGAMI_ERR_INVALID, "tokens, heads, and head_dim must be positive");
  if (key_bins <= 1 || value_bins <= 1) return fail(ORIGAMI_ERR_INVALID, "CacheGen bins must be greater than one");
  if (key_offset < 0 || key_bytes < 0 || value_offset < 0 || value_bytes < 0)
    return fail(ORIGAMI_ERR_INVALID, "invalid CacheGen stream offsets");
  if (key_offset + key_bytes > bytestream_bytes || value_offset + value_bytes > bytestream_bytes)
    return fail(ORIGAMI_ERR_INVALID, "CacheGen stream ranges exceed bytestream length");
  if (max_key_numel < tokens || max_value_numel < tokens)
    return fail(ORIGAMI_ERR_INVALID, "max tensors must contain at least tokens values");
  int32_t rc = cache_geom(cache, cache_dtype, g);
  if (rc) return rc;
  if ((rc = check_blocks(cache, d_block_ids, num_block_ids, tokens))) return rc;
  if (d_bytestream == nullptr && bytestream_bytes > 0) return fail(ORIGAMI_ERR_INVALID, "bytestream is null");
  if (d_max_key == nullptr || d_max_value == nullptr) return fail(ORIGAMI_ERR_INVALID, "max tensors are null");

  origami::CgArgs a{};
  a.stream[0] = d_bytestream + key_offset;
  a.stream[1] = d_bytestream + value_offset;
  a.stream_bytes[0] = read_limit(key_bits, key_bytes, bytestream_bytes - key_offset);
  a.stream_bytes[1] = read_limit(value_bits, value_bytes, bytestream_bytes - value_offset);
  a.bits[0] = static_cast<int32_t>(key_bits);
  a.bits[1] = static_cast<int32_t>(value_bits);
  a.bins[0] = key_bins;
  a.bins[1] = value_bins;
  a.maxv[0] = d_max_key;
  a.maxv[1] = d_max_value;
  a.cache = static_cast<uint8_t*>(cache->d_data);
  a.ids = d_block_ids;
  a.kv_stride = g.kv_stride;
  a.block_stride = g.block_stride;
  a.token_stride = g.token_stride;
  a.num_blocks = cache->num_blocks;
  a.block_size = cache->block_size;
  a.tokens = tokens;
  a.heads = static_cast<int32_t>(cache->num_heads);
  const int64_t C = cache->num_heads * cache->head_dim;
  if (C > 0x7FFFFFFF) return fail(ORIGAMI_ERR_UNSUPPORTED, "heads * head_dim must be below 2^31");
  if (tokens > 0x7FFFFFFF || cache->block_size > 0x7FFFFFFF)
    return fail(ORIGAMI_ERR_UNSUPPORTED, "tokens and block_size must be below 2^31");
  a.C = static_cast<int32_t>(C);
  const bool vec = C % 8 == 0 && aligned(cache->d_data, 16);
  a.nvec = vec ? static_cast<int32_t>(C / 8) : a.C;
  a.err = d_error_count;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool bf16 = cache_dtype == ORIGAMI_DTYPE_BF16;
  const uint8_t* buf_end = d_bytestream + bytestream_bytes;
  if (max_dtype == ORIGAMI_DTYPE_F16)
    return bf16 ? launch_cg_vec<__half, __nv_bfloat16>(vec, a, buf_end, st)
                : launch_cg_vec<__half, __half>(vec, a, buf_end, st);
  return bf16 ? launch_cg_vec<float, __nv_bfloat16>(vec, a, buf_end, st)
              : launch_cg_vec<float, __half>(vec, a, buf_end, st);
}

int32_t origami_cachegen_unpack_dequantize(
    const uint8_t* d_bytestream, int64_t bytestream_bytes, const int64_t* d_offsets, const int64_t* h_offsets,
    int64_t num_offsets, const int64_t* d_bits_per_layer, const int64_t* h_bits_per_layer, int64_t num_bits,
    const int64_t* d_key_bins, int64_t num_key_bins, const int64_t* d_value_bins, int64_t num_value_bins,
    const void* d_max_key, int64_t max_key_numel, const void* d_max_value, int64_t max_value_numel,
    int32_t max_dtype, int64_t tokens, int64_t heads, int64_t head_dim, void* d_output, int64_t output_bytes,
    origami_stream_t stream) {
  if (max_dtype != ORIGAMI_DTYPE_F16 && max_dtype != ORIGAMI_DTYPE_F32)
    return fail(ORIGAMI_ERR_INVALID, "max tensors must be float16 or float32");
  if (num_bits % 2 != 0) return fail(ORIGAMI_ERR_INVALID, "bits_per_layer length must be even");
  const int64_t layers = num_bits / 2;
  if (num_key_bins != layers) return fail(ORIGAMI_ERR_INVALID, "key_bins length must match layers");
  if (num_value_bins != layers) return fail(ORIGAMI_ERR_INVALID, "value_bins length must match layers");
  if (num_offsets != num_bits + 1)
    return fail(ORIGAMI_ERR_INVALID, "offsets length must be bits_per_layer length + 1");
  if (max_key_numel != layers * tokens) return fail(ORIGAMI_ERR_INVALID, "max_key must have layers * tokens values");
  if (max_value_numel != layers * tokens)
    return fail(ORIGAMI_ERR_INVALID, "max_value must have layers * tokens values");
  if (tokens <= 0 || heads <= 0 || head_dim <= 0)
    return fail(ORIGAMI_ERR_INVALID, "tokens, heads, and head_dim must be positive");
  if (num_bits > 0 && h_bits_per_layer == nullptr) return fail(ORIGAMI_ERR_INVALID, "bits_per_layer is null");
  for (int64_t i = 0; i < num_bits; ++i)
    if (!bits_ok(h_bits_per_layer[i])) return fail(ORIGAMI_ERR_INVALID, kBitsMsg);
  // The reference reads the streams wherever offsets point; here they must lie inside the
  // bytestream.
  if (h_offsets == nullptr) return fail(ORIGAMI_ERR_INVALID, "offsets are null");
  for (int64_t i = 0; i < num_bits; ++i)
    if (h_offsets[i] < 0 || h_offsets[i + 1] < h_offsets[i] || h_offsets[i + 1] > bytestream_bytes)
      return fail(ORIGAMI_ERR_INVALID, "offsets must be non-decreasing and inside the bytestream");
  const int64_t out_elems = layers * 2 * heads * tokens * head_dim;
  if (output_bytes < 2 * out_elems || (out_elems > 0 && d_output == nullptr))
    return fail(ORIGAMI_ERR_INVALID, "output buffer holds %lld bytes, %lld needed", (long long)output_bytes,
                (long long)(2 * out_elems));
  if (layers == 0) return ORIGAMI_OK;
  if (2 * layers > 65535) return fail(ORIGAMI_ERR_UNSUPPORTED, "at most 32767 layers per call");

  origami::CgUnpackArgs a{};
  a.bytestream = d_bytestream;
  a.bytestream_bytes = bytestream_bytes;
  a.offsets = d_offsets;
  a.bits = d_bits_per_layer;
  a.key_bins = d_key_bins;
  a.value_bins = d_value_bins;
  a.max_key = d_max_key;
  a.max_value = d_max_value;
  a.out = static_cast<__half*>(d_output);
  a.layers = layers;
  a.tokens = tokens;
  a.heads = heads;
  a.head_dim = head_dim;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = head_dim % 8 == 0 && aligned(d_output, 16);
  if (max_dtype == ORIGAMI_DTYPE_F16)
    return vec ? launch_cg_unpack<__half, true>(a, 2 * layers, st) : launch_cg_unpack<__half, false>(a, 2 * layers, st);
  return vec ? launch_cg_unpack<float, true>(a, 2 * layers, st) : launch_cg_unpack<float, false>(a, 2 * layers, st);
}

int32_t origami_kivi_dequantize_to_kv_cache(
    const uint8_t* d_bytestream, int64_t bytestream_bytes, int64_t key_offset, int64_t key_bytes,
    int64_t value_offset, int64_t value_bytes, int64_t bits, int64_t group_size, int64_t sink_tokens,
    const void* d_key_scale, const void* d_key_zero, const void* d_value_scale, const void* d_value_zero,
    const void* d_key_sink, const void* d_value_sink, const int64_t* meta_numel, int32_t meta_dtype,
    const origami_paged_kv* cache, int32_t cache_dtype, const int64_t* d_block_ids, int64_t num_block_ids,
    int64_t tokens, uint32_t* d_error_count, origami_stream_t stream) {
  if (cache_dtype != ORIGAMI_DTYPE_F16 && cache_dtype != ORIGAMI_DTYPE_BF16)
    return fail(ORIGAMI_ERR_INVALID, "kv_cache must be float16 or bfloat16");
  if (meta_dtype != ORIGAMI_DTYPE_F16 && meta_dtype != ORIGAMI_DTYPE_F32)
    return fail(ORIGAMI_ERR_INVALID, "KIVI metadata tensors must be float16 or float32");
  if (!bits_ok(bits)) return fail(ORIGAMI_ERR_INVALID, kBitsMsg);
  if (group_size <= 0) return fail(ORIGAMI_ERR_INVALID, "KIVI group_size must be positive");
  if (sink_tokens < 0 || sink_tokens > tokens) return fail(ORIGAMI_ERR_INVALID, "KIVI sink_tokens must be in [0, tokens]");
  if (cache == nullptr) return fail(ORIGAMI_ERR_INVALID, "kv cache is null");
  if (tokens <= 0 || cache->num_heads <= 0 || cache->head_dim <= 0)
    return fail(ORIGAMI_ERR_INVALID, "tokens, heads, and head_dim must be positive");
  if (key_offset < 0 || key_bytes < 0 || value_offset < 0 || value_bytes < 0)
    return fail(ORIGAMI_ERR_INVALID, "invalid KIVI stream offsets");
  if (key_offset + key_bytes > bytestream_bytes || value_offset + value_bytes > bytestream_bytes)
    return fail(ORIGAMI_ERR_INVALID, "KIVI stream ranges exceed bytestream length");
  if (meta_numel == nullptr) return fail(ORIGAMI_ERR_INVALID, "meta_numel is null");
  const int64_t body = tokens - sink_tokens;
  const int64_t channels = cache->num_heads * cache->head_dim;
  const int64_t key_groups = (body + group_size - 1) / group_size;
  const int64_t value_groups = (channels + group_size - 1) / group_size;
  if (meta_numel[0] < key_groups * channels || meta_numel[1] < key_groups * channels)
    return fail(ORIGAMI_ERR_INVALID, "KIVI key metadata is too small");
  if (meta_numel[2] < body * value_groups || meta_numel[3] < body * value_groups)
    return fail(ORIGAMI_ERR_INVALID, "KIVI value metadata is too small");
  if (meta_numel[4] < sink_tokens * channels || meta_numel[5] < sink_tokens * channels)
    return fail(ORIGAMI_ERR_INVALID, "KIVI sink metadata is too small");
  PagedGeom g{};
  int32_t rc = cache_geom(cache, cache_dtype, g);
  if (rc) return rc;
  if ((rc = check_blocks(cache, d_block_ids, num_block_ids, tokens))) return rc;
  if (channels > 0x7FFFFFFF || cache->head_dim > 0x7FFFFFFF)
    return fail(ORIGAMI_ERR_UNSUPPORTED, "heads * head_dim must be below 2^31");
  if (tokens > 0x7FFFFFFF || cache->block_size > 0x7FFFFFFF)
    return fail(ORIGAMI_ERR_UNSUPPORTED, "tokens and block_size must be below 2^31");

  origami::KiviArgs a{};
  a.stream[0] = d_bytestream + key_offset;
  a.stream[1] = d_bytestream + value_offset;
  a.stream_bytes[0] = read_limit(bits, key_bytes, bytestream_bytes - key_offset);
  a.stream_bytes[1] = read_limit(bits, value_bytes, bytestream_bytes - value_offset);
  a.scale[0] = d_key_scale;
  a.zero[0] = d_key_zero;
  a.scale[1] = d_value_scale;
  a.zero[1] = d_value_zero;
  a.sink[0] = d_key_sink;
  a.sink[1] = d_value_sink;
  a.cache = static_cast<uint8_t*>(cache->d_data);
  a.ids = d_block_ids;
  a.kv_stride = g.kv_stride;
  a.block_stride = g.block_stride;
  a.token_stride = g.token_stride;
  a.head_stride = g.head_stride;
  a.num_blocks = cache->num_blocks;
  a.block_size = cache->block_size;
  a.tokens = tokens;
  a.num_ids = num_block_ids;
  a.sink_tokens = sink_tokens;
  a.body_tokens = body;
  a.group_size = group_size;
  a.value_groups = value_groups;
  a.bits = static_cast<int32_t>(bits);
  a.H = static_cast<int32_t>(cache->num_heads);
  a.D = static_cast<int32_t>(cache->head_dim);
  a.err = d_error_count;
  a.group_shift = ilog2_exact(group_size);
  a.block_shift = ilog2_exact(cache->block_size);
  const bool tiled = sink_tokens % 8 == 0 && aligned(cache->d_data, 16);
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool bf16 = cache_dtype == ORIGAMI_DTYPE_BF16;
  if (meta_dtype == ORIGAMI_DTYPE_F16)
    return bf16 ? launch_kivi<__half, __nv_bfloat16>(a, tiled, st) : launch_kivi<__half, __half>(a, tiled, st);
  return bf16 ? launch_kivi<float, __nv_bfloat16>(a, tiled, st) : launch_kivi<float, __half>(a, tiled, st);
}

}  // extern "C"
