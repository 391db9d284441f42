// C ABI of the fused prefix attention (attention_kernels.cuh): validation with the
// reference's checks and messages (bitpack_layout_cuda.cpp:716-890), the split plan, the
// workspace size and the launch.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "../../include/origami_b200.h"
#include "attention_kernels.cuh"
#include "attention_sym_kernels.cuh"
#include "host_common.h"

using namespace origami_host;

namespace {

struct AttnPlan {
  int nq = 8;        // query rows per CTA
  int rows = 0;      // query_tokens * group
  int row_blocks = 0;
  int splits = 1;
  int64_t ws_bytes = 0, counters_bytes = 0, o_bytes = 0;
};

constexpr int64_t kAlign = 256;
int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

int32_t sm_count(int& sms) {
  static std::mutex mu;
  static std::vector<std::pair<int, int>> cache;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& x : cache)
    if (x.first == dev) {
      sms = x.second;
      return ORIGAMI_OK;
    }
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
    return cuda_fail(e, "cudaDeviceGetAttribute");
  cache.push_back({dev, sms});
  return ORIGAMI_OK;
}

// Rows per CTA grow with the query rows of a KV head (8 .. 64); the key range is split
// over CTAs until about two CTAs per SM are busy, at most one split per 128-key tile.
int32_t make_plan(int64_t query_tokens, int64_t query_heads, int64_t kv_heads, int64_t query_start,
                  int64_t sequence_length, bool sym, AttnPlan& p) {
  const int64_t group = query_heads / kv_heads;
  const int64_t rows = query_tokens * group;
  if (rows > 0x3FFFFFFF) return fail(ORIGAMI_ERR_UNSUPPORTED, "too many query rows");
  p.rows = static_cast<int>(rows);
  p.nq = sym ? origami::attn::kSymNQ : rows <= 8 ? 8 : rows <= 16 ? 16 : rows <= 32 ? 32 : 64;
  p.row_blocks = static_cast<int>((rows + p.nq - 1) / p.nq);
  int sms = 0;
  const int32_t rc = sm_count(sms);
  if (rc) return rc;
  const int64_t base = kv_heads * p.row_blocks;
  const int64_t first_tiles = std::min(sequence_length - 1, query_start) / origami::attn::kKT + 1;
  int64_t splits = (2 * static_cast<int64_t>(sms) + base - 1) / base;
  // the merging CTA stages splits x NQ (max, sum) pairs in its 2 x 36 KB of tile memory
  splits = std::max<int64_t>(1, std::min<int64_t>({splits, first_tiles, static_cast<int64_t>(4096 / p.nq)}));
  if (base * splits > 0x7FFFFFFF) return fail(ORIGAMI_ERR_UNSUPPORTED, "attention grid too large");
  p.splits = static_cast<int>(splits);
  if (p.splits > 1) {
    p.counters_bytes = round_up(base * 4, kAlign);
    p.o_bytes = round_up(base * splits * p.nq * origami::attn::kD * 4, kAlign);
    p.ws_bytes = p.counters_bytes + p.o_bytes + round_up(base * splits * p.nq * 2 * 4, kAlign);
  }
  return ORIGAMI_OK;
}

template <typename QT, int CODEC, int NQ>
int32_t launch(const origami::AttnArgs& a, int64_t ctas, cudaStream_t st) {
  const void* fn = reinterpret_cast<const void*>(&origami::prefix_attention<QT, CODEC, NQ>);
  const int smem = origami::AttnSmem<NQ>::bytes;
  int resident = 0;
  int32_t rc = persistent_slots(fn, smem, resident);  // raises the kernel's shared-memory limit
  if (rc) return rc;
  origami::prefix_attention<QT, CODEC, NQ><<<static_cast<unsigned>(ctas), origami::attn::kThreadsA, smem, st>>>(a);
  return after_launch("prefix_attention launch");
}

template <typename QT, int CODEC>
int32_t launch_nq(int nq, const origami::AttnArgs& a, int64_t ctas, cudaStream_t st) {
  switch (nq) {
    case 8: return launch<QT, CODEC, 8>(a, ctas, st);
    case 16: return launch<QT, CODEC, 16>(a, ctas, st);
    case 32: return launch<QT, CODEC, 32>(a, ctas, st);
    default: return launch<QT, CODEC, 64>(a, ctas, st);
  }
}

// The symbol-operand kernel (attention_sym_kernels.cuh) takes decode shapes (at most 32
// query rows per KV head, 8 per CTA) whose groups fit its operand slots: KVQuant always,
// KIVI when a 128-key tile spans at most 3 key groups and every head at most 2 value
// channel groups.
bool sym_path(int64_t codec, int64_t group_size, int64_t kv_heads, int64_t rows) {
  if (rows > 4 * origami::attn::kSymNQ) return false;
  if (codec == 1) return true;
  if (group_size < 64) return false;
  for (int64_t h = 0; h < kv_heads; ++h)
    if ((h * 128 + 127) / group_size - (h * 128) / group_size + 1 > origami::attn::kSymMaxC) return false;
  return true;
}

// Workspace for whichever kernel a call with these shapes takes: the larger plan.
// The shape checks of the workspace query (the launch repeats them with its own messages).
int32_t check_plan_args(int64_t query_tokens, int64_t query_heads, int64_t kv_heads, int64_t query_start_position,
                        int64_t sequence_length) {
  if (query_tokens <= 0 || query_heads <= 0)
    return fail(ORIGAMI_ERR_INVALID, "query token and head counts must be positive");
  if (kv_heads <= 0 || query_heads % kv_heads != 0)
    return fail(ORIGAMI_ERR_INVALID, "query_heads must be divisible by kv_heads");
  if (sequence_length <= 0 || query_start_position < 0 || query_start_position + query_tokens > sequence_length)
    return fail(ORIGAMI_ERR_INVALID, "query range exceeds sequence length");
  return ORIGAMI_OK;
}

int32_t workspace_plan(int64_t query_tokens, int64_t query_heads, int64_t kv_heads, int64_t query_start,
                       int64_t sequence_length, int64_t& bytes, int64_t& counters) {
  AttnPlan p;
  int32_t rc = make_plan(query_tokens, query_heads, kv_heads, query_start, sequence_length, false, p);
  if (rc) return rc;
  bytes = p.ws_bytes;
  counters = p.counters_bytes;
  if (query_tokens * (query_heads / kv_heads) <= 4 * origami::attn::kSymNQ) {
    AttnPlan q;
    if ((rc = make_plan(query_tokens, query_heads, kv_heads, query_start, sequence_length, true, q))) return rc;
    bytes = std::max(bytes, q.ws_bytes);
    counters = std::max(counters, q.counters_bytes);
  }
  return ORIGAMI_OK;
}

template <typename QT, int CODEC, int SLOT>
int32_t launch_sym_slot(const origami::AttnArgs& a, int64_t ctas, cudaStream_t st) {
  const void* fn = reinterpret_cast<const void*>(&origami::prefix_attention_sym<QT, CODEC, SLOT>);
  constexpr int smem = origami::AttnSymSmem::bytes(SLOT);
  int resident = 0;
  int32_t rc = persistent_slots(fn, smem, resident);  // raises the kernel's shared-memory limit
  if (rc) return rc;
  // programmatic dependent launch: the kernel's setup may overlap the previous kernel's tail
  // (it waits for that kernel before its first global access)
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(ctas));
  cfg.blockDim = dim3(origami::attn::kThreadsA);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, origami::prefix_attention_sym<QT, CODEC, SLOT>, a);
  if (e != cudaSuccess) return cuda_fail(e, "prefix_attention_sym launch");
  return after_launch("prefix_attention_sym launch");
}

template <typename QT, int CODEC>
int32_t launch_sym(const origami::AttnArgs& a, int64_t ctas, cudaStream_t st) {
  switch (a.slot_bits) {
    case 2: return launch_sym_slot<QT, CODEC, 2>(a, ctas, st);
    case 4: return launch_sym_slot<QT, CODEC, 4>(a, ctas, st);
    default: return launch_sym_slot<QT, CODEC, 8>(a, ctas, st);
  }
}

int64_t packed_symbol_bytes(int64_t bits, int64_t symbols) {
  return bits == 3 ? (symbols + 1) / 2 : (symbols * bits + 7) / 8;
}

}  // namespace

extern "C" {

int32_t origami_fused_prefix_attention_workspace(int64_t query_tokens, int64_t query_heads, int64_t kv_heads,
                                                 int64_t query_start_position, int64_t sequence_length,
                                                 int64_t* workspace_bytes) {
  if (workspace_bytes == nullptr) return fail(ORIGAMI_ERR_INVALID, "workspace_bytes is null");
  int32_t rc0 = check_plan_args(query_tokens, query_heads, kv_heads, query_start_position, sequence_length);
  if (rc0) return rc0;
  int64_t bytes = 0, counters = 0;
  const int32_t rc = workspace_plan(query_tokens, query_heads, kv_heads, query_start_position, sequence_length,
                                    bytes, counters);
  if (rc) return rc;
  *workspace_bytes = bytes;
  return ORIGAMI_OK;
}

int32_t origami_fused_prefix_attention(
    const uint8_t* d_bytestream, int64_t bytestream_bytes, int64_t key_offset, int64_t key_bytes,
    int64_t value_offset, int64_t value_bytes, int64_t codec, int64_t bits, int64_t group_size, int64_t sink_tokens,
    const void* d_key_scale, const void* d_key_zero, const void* d_value_scale, const void* d_value_zero,
    const void* d_key_sink, const void* d_value_sink, const int64_t* meta_numel, int32_t meta_dtype,
    const void* d_query, int32_t query_dtype, int64_t query_tokens, int64_t query_heads, int64_t head_dim,
    const origami_paged_kv* cache, int32_t cache_dtype, const int32_t* d_block_table, int64_t block_table_len,
    int64_t prefix_tokens, int64_t query_start_position, int64_t sequence_length, double softmax_scale,
    void* d_output, void* d_workspace, int64_t workspace_bytes, uint32_t* d_error_flags, origami_stream_t stream) {
  if (codec != 0 && codec != 1) return fail(ORIGAMI_ERR_INVALID, "codec must be 0 (KIVI) or 1 (KVQuant)");
  if (bits != 2 && bits != 3 && bits != 4 && bits != 8)
    return fail(ORIGAMI_ERR_INVALID, "fused attention supports 2, 3, 4, or 8 bits");
  if (group_size <= 0) return fail(ORIGAMI_ERR_INVALID, "group_size must be positive");
  if (prefix_tokens <= 0) return fail(ORIGAMI_ERR_INVALID, "prefix_tokens must be positive");
  if (sink_tokens < 0 || sink_tokens > prefix_tokens)
    return fail(ORIGAMI_ERR_INVALID, "sink_tokens must be in [0, prefix_tokens]");
  if (key_offset < 0 || key_bytes < 0 || value_offset < 0 || value_bytes < 0)
    return fail(ORIGAMI_ERR_INVALID, "invalid compressed stream offsets");
  if (key_offset + key_bytes > bytestream_bytes || value_offset + value_bytes > bytestream_bytes)
    return fail(ORIGAMI_ERR_INVALID, "compressed stream ranges exceed bytestream length");
  if (query_dtype != ORIGAMI_DTYPE_F16 && query_dtype != ORIGAMI_DTYPE_BF16)
    return fail(ORIGAMI_ERR_INVALID, "query must be float16 or bfloat16");
  if (cache_dtype != ORIGAMI_DTYPE_F16 && cache_dtype != ORIGAMI_DTYPE_BF16)
    return fail(ORIGAMI_ERR_INVALID, "kv_cache must be float16 or bfloat16");
  if (meta_dtype != ORIGAMI_DTYPE_F16) return fail(ORIGAMI_ERR_INVALID, "compressed metadata tensors must be float16");
  if (query_tokens <= 0 || query_heads <= 0)
    return fail(ORIGAMI_ERR_INVALID, "query token and head counts must be positive");
  if (head_dim != 128) return fail(ORIGAMI_ERR_INVALID, "the first Origami fused kernel supports head_dim 128 only");
  if (cache == nullptr || cache->d_data == nullptr) return fail(ORIGAMI_ERR_INVALID, "kv cache is null");
  if (cache->layout != ORIGAMI_KV_FIRST && cache->layout != ORIGAMI_BLOCKS_FIRST)
    return fail(ORIGAMI_ERR_INVALID,
                "kv_cache must be [num_blocks,2,block,heads,dim] or [2,num_blocks,block,heads,dim]");
  if (cache->elem_bytes != 2) return fail(ORIGAMI_ERR_INVALID, "kv_cache must be float16 or bfloat16");
  if (cache->head_dim != head_dim) return fail(ORIGAMI_ERR_INVALID, "kv_cache head_dim does not match query");
  const int64_t kv_heads = cache->num_heads;
  if (kv_heads <= 0 || query_heads % kv_heads != 0)
    return fail(ORIGAMI_ERR_INVALID, "query_heads must be divisible by kv_heads");
  if (cache->block_size <= 0 || cache->num_blocks <= 0)
    return fail(ORIGAMI_ERR_INVALID, "kv_cache block dimensions must be positive");
  if (query_start_position < prefix_tokens)
    return fail(ORIGAMI_ERR_INVALID, "query must start at or after the compressed prefix");
  if (sequence_length <= 0 || query_start_position + query_tokens > sequence_length)
    return fail(ORIGAMI_ERR_INVALID, "query range exceeds sequence length");
  const int64_t logical_blocks = (sequence_length + cache->block_size - 1) / cache->block_size;
  if (block_table_len < logical_blocks || d_block_table == nullptr)
    return fail(ORIGAMI_ERR_INVALID, "block_table is too short for sequence_length");
  const int64_t channels = kv_heads * head_dim;
  const int64_t body = prefix_tokens - sink_tokens;
  const int64_t stream_tokens = codec == 0 ? body : prefix_tokens;
  if (key_bytes < packed_symbol_bytes(bits, stream_tokens * channels) ||
      value_bytes < packed_symbol_bytes(bits, stream_tokens * channels))
    return fail(ORIGAMI_ERR_INVALID, "compressed K/V streams are smaller than their declared shape");
  if (meta_numel == nullptr) return fail(ORIGAMI_ERR_INVALID, "meta_numel is null");
  if (codec == 0) {
    const int64_t key_groups = (body + group_size - 1) / group_size;
    const int64_t value_groups = (channels + group_size - 1) / group_size;
    if (meta_numel[0] < key_groups * channels || meta_numel[1] < key_groups * channels)
      return fail(ORIGAMI_ERR_INVALID, "KIVI key metadata is too small");
    if (meta_numel[2] < body * value_groups || meta_numel[3] < body * value_groups)
      return fail(ORIGAMI_ERR_INVALID, "KIVI value metadata is too small");
    if (meta_numel[4] < sink_tokens * channels || meta_numel[5] < sink_tokens * channels)
      return fail(ORIGAMI_ERR_INVALID, "KIVI sink tensors are too small");
  } else {
    if (meta_numel[0] < channels || meta_numel[1] < channels)
      return fail(ORIGAMI_ERR_INVALID, "KVQuant key metadata is too small");
    if (meta_numel[2] < prefix_tokens || meta_numel[3] < prefix_tokens)
      return fail(ORIGAMI_ERR_INVALID, "KVQuant value metadata is too small");
  }
  if (d_bytestream == nullptr || d_query == nullptr || d_output == nullptr)
    return fail(ORIGAMI_ERR_INVALID, "null device pointer");
  if (!aligned(d_query, 2) || !aligned(d_output, 2) || !aligned(cache->d_data, 2))
    return fail(ORIGAMI_ERR_INVALID, "query, output and kv_cache must be 2-byte aligned");
  for (const void* m : {d_key_scale, d_key_zero, d_value_scale, d_value_zero})
    if (m == nullptr || !aligned(m, 2)) return fail(ORIGAMI_ERR_INVALID, "compressed metadata tensors must be float16");
  if (codec == 0 && sink_tokens > 0 && (d_key_sink == nullptr || d_value_sink == nullptr))
    return fail(ORIGAMI_ERR_INVALID, "KIVI sink tensors are too small");

  const bool sym = sym_path(codec, group_size, kv_heads, query_tokens * (query_heads / kv_heads));
  AttnPlan p;
  int32_t rc = make_plan(query_tokens, query_heads, kv_heads, query_start_position, sequence_length, sym, p);
  if (rc) return rc;
  if (p.ws_bytes > 0 && (d_workspace == nullptr || workspace_bytes < p.ws_bytes || !aligned(d_workspace, 16)))
    return fail(ORIGAMI_ERR_INVALID, "workspace must be 16-byte aligned and hold %lld bytes (zeroed before first use)",
                static_cast<long long>(p.ws_bytes));

  origami::AttnArgs a{};
  a.stream[0] = d_bytestream + key_offset;
  a.stream[1] = d_bytestream + value_offset;
  a.bytes_end = d_bytestream + bytestream_bytes;
  a.stream_end[0] = a.stream[0] + key_bytes;
  a.stream_end[1] = a.stream[1] + value_bytes;
  a.slot_bits = bits == 3 ? 4 : static_cast<int32_t>(bits);
  a.sym_mask = static_cast<int32_t>((1 << bits) - 1);
  a.group_size = group_size;
  a.sink = codec == 0 ? sink_tokens : 0;
  a.prefix = prefix_tokens;
  a.body = stream_tokens;
  a.scale[0] = static_cast<const __half*>(d_key_scale);
  a.zero[0] = static_cast<const __half*>(d_key_zero);
  a.scale[1] = static_cast<const __half*>(d_value_scale);
  a.zero[1] = static_cast<const __half*>(d_value_zero);
  a.sink_kv[0] = static_cast<const __half*>(d_key_sink);
  a.sink_kv[1] = static_cast<const __half*>(d_value_sink);
  a.query = static_cast<const uint16_t*>(d_query);
  a.output = static_cast<uint16_t*>(d_output);
  a.cache = static_cast<const uint16_t*>(cache->d_data);
  const int64_t slab = cache->block_size * channels;
  a.kv_stride = cache->layout == ORIGAMI_KV_FIRST ? cache->num_blocks * slab : slab;
  a.block_stride = cache->layout == ORIGAMI_KV_FIRST ? slab : 2 * slab;
  a.token_stride = channels;
  a.num_blocks = cache->num_blocks;
  a.block_size = cache->block_size;
  a.block_table = d_block_table;
  a.q_start = query_start_position;
  a.seq_len = sequence_length;
  a.q_tokens = static_cast<int32_t>(query_tokens);
  a.q_heads = static_cast<int32_t>(query_heads);
  a.kv_heads = static_cast<int32_t>(kv_heads);
  a.group = static_cast<int32_t>(query_heads / kv_heads);
  a.rows = p.rows;
  a.row_blocks = p.row_blocks;
  a.splits = p.splits;
  a.cache_bf16 = cache_dtype == ORIGAMI_DTYPE_BF16 ? 1 : 0;
  a.cache_vec = aligned(cache->d_data, 16) ? 1 : 0;
  a.meta_vec = (aligned(d_key_scale, 16) && aligned(d_key_zero, 16) && aligned(d_value_scale, 16) &&
                aligned(d_value_zero, 16)) ? 1 : 0;
  a.sym_len = bits == 3 ? 3 : static_cast<int32_t>(bits);
  a.scale_log2 = static_cast<float>(softmax_scale * 1.4426950408889634);
  if (p.splits > 1) {
    uint8_t* ws = static_cast<uint8_t*>(d_workspace);
    a.counters = reinterpret_cast<uint32_t*>(ws);
    a.ws_o = reinterpret_cast<float*>(ws + p.counters_bytes);
    a.ws_ml = reinterpret_cast<float*>(ws + p.counters_bytes + p.o_bytes);
  }
  a.err = d_error_flags;
  const int64_t ctas = kv_heads * p.row_blocks * p.splits;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (sym) {
    if (query_dtype == ORIGAMI_DTYPE_BF16)
      return codec == 0 ? launch_sym<__nv_bfloat16, 0>(a, ctas, st) : launch_sym<__nv_bfloat16, 1>(a, ctas, st);
    return codec == 0 ? launch_sym<__half, 0>(a, ctas, st) : launch_sym<__half, 1>(a, ctas, st);
  }
  if (query_dtype == ORIGAMI_DTYPE_BF16)
    return codec == 0 ? launch_nq<__nv_bfloat16, 0>(p.nq, a, ctas, st) : launch_nq<__nv_bfloat16, 1>(p.nq, a, ctas, st);
  return codec == 0 ? launch_nq<__half, 0>(p.nq, a, ctas, st) : launch_nq<__half, 1>(p.nq, a, ctas, st);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Allocation-free variant: the split workspace lives in a file-scope device array.
// ---------------------------------------------------------------------------------------
namespace {

constexpr int64_t kStaticScratchBytes = 8ll << 20;  // 8 MiB per device
__device__ __align__(256) uint8_t g_attention_scratch[kStaticScratchBytes];

// The array's device address on the current device, looked up once per device.
int32_t static_scratch(void** out) {
  static std::mutex mu;
  static std::vector<std::pair<int, void*>> cache;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& x : cache)
    if (x.first == dev) {
      *out = x.second;
      return ORIGAMI_OK;
    }
  void* p = nullptr;
  if ((e = cudaGetSymbolAddress(&p, g_attention_scratch)) != cudaSuccess)
    return cuda_fail(e, "cudaGetSymbolAddress(g_attention_scratch)");
  cache.push_back({dev, p});
  *out = p;
  return ORIGAMI_OK;
}

}  // namespace

extern "C" int32_t origami_fused_prefix_attention_noalloc(
    const uint8_t* d_bytestream, int64_t bytestream_bytes, int64_t key_offset, int64_t key_bytes,
    int64_t value_offset, int64_t value_bytes, int64_t codec, int64_t bits, int64_t group_size, int64_t sink_tokens,
    const void* d_key_scale, const void* d_key_zero, const void* d_value_scale, const void* d_value_zero,
    const void* d_key_sink, const void* d_value_sink, const int64_t* meta_numel, int32_t meta_dtype,
    const void* d_query, int32_t query_dtype, int64_t query_tokens, int64_t query_heads, int64_t head_dim,
    const origami_paged_kv* cache, int32_t cache_dtype, const int32_t* d_block_table, int64_t block_table_len,
    int64_t prefix_tokens, int64_t query_start_position, int64_t sequence_length, double softmax_scale,
    void* d_output, uint32_t* d_error_flags, origami_stream_t stream) {
  if (cache == nullptr) return fail(ORIGAMI_ERR_INVALID, "kv cache is null");
  int32_t rc = check_plan_args(query_tokens, query_heads, cache->num_heads, query_start_position, sequence_length);
  if (rc) return rc;
  int64_t need = 0, counters = 0;  // one plan gives both the workspace and its counters
  if ((rc = workspace_plan(query_tokens, query_heads, cache->num_heads, query_start_position, sequence_length, need,
                           counters)))
    return rc;
  if (need > kStaticScratchBytes)
    return fail(ORIGAMI_ERR_UNSUPPORTED,
                "these shapes need %lld bytes of split workspace; the static scratch holds %lld "
                "(use origami_fused_prefix_attention with a caller-provided workspace)",
                static_cast<long long>(need), static_cast<long long>(kStaticScratchBytes));
  void* scratch = nullptr;
  if ((rc = static_scratch(&scratch))) return rc;
  if (need > 0) {
    // the arrival counters lead the workspace and must read zero at launch
    const cudaError_t e =
        cudaMemsetAsync(scratch, 0, static_cast<size_t>(counters), reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(scratch counters)");
  }
  return origami_fused_prefix_attention(
      d_bytestream, bytestream_bytes, key_offset, key_bytes, value_offset, value_bytes, codec, bits, group_size,
      sink_tokens, d_key_scale, d_key_zero, d_value_scale, d_value_zero, d_key_sink, d_value_sink, meta_numel,
      meta_dtype, d_query, query_dtype, query_tokens, query_heads, head_dim, cache, cache_dtype, d_block_table,
      block_table_len, prefix_tokens, query_start_position, sequence_length, softmax_scale, d_output, scratch,
      kStaticScratchBytes, d_error_flags, stream);
}
