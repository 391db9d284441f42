/*
 * origami_b200 — C ABI of the B200 (sm_100a) KV layout hot path.
 *
 * The library moves one layer of a vLLM paged KV cache between the cache and the
 * "codec-friendly" chunked layout that Origami hands to its host lossless codec:
 *
 *   save    : gather a request's blocks -> split every 16-bit element into planes
 *             -> canonical head > channel > token order -> dense LSB-first bitpack
 *             into chunks sized by the head/channel chunk planner;
 *   restore : the exact inverse, scattering straight into the paged cache through
 *             the block table.
 *
 * The canonical chunk format is the one defined by Origami's CUDA unpack kernel
 * (csrc/origami/bitpack_layout_cuda.cu:70-128): a chunk spec row
 * [head_start, head_end, channel_start, channel_end, token_start, token_end]
 * covers symbols in head > channel > token order; symbol i of a chunk with
 * `bits` bits per symbol occupies stream bits [i*bits, (i+1)*bits), bit k of the
 * stream being bit (k % 8) of byte (k / 8); a chunk holds ceil(n*bits/8) bytes
 * (bitpack_layout_cuda.cpp:183-185).
 *
 * Conventions (all entry points):
 *   - plain pointers and sizes only; `d_` pointers are device memory, `h_` host;
 *   - every launch goes to the caller's stream; nothing synchronises the device;
 *   - the entry points allocate no device memory and are safe to call from
 *     several host threads at once (the only shared state, a per-kernel cache of the
 *     shared-memory attribute and occupancy, is behind a mutex);
 *   - return ORIGAMI_OK (0) or a negative ORIGAMI_ERR_*; origami_last_error()
 *     returns a message for the calling thread's last failure;
 *   - `d_error_count` (nullable) is a device uint32 that kernels increment for
 *     every row they had to skip (block id outside the cache); the caller owns it.
 */
#ifndef ORIGAMI_B200_H
#define ORIGAMI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* origami_stream_t; /* identical to cudaStream_t */

enum {
  ORIGAMI_OK = 0,
  ORIGAMI_ERR_INVALID = -1,     /* argument / table validation failed       */
  ORIGAMI_ERR_UNSUPPORTED = -2, /* valid request outside what this build does */
  ORIGAMI_ERR_CUDA = -3         /* a CUDA runtime call failed                */
};

/* Paged-cache layouts accepted for one layer's cache tensor. */
enum {
  ORIGAMI_KV_FIRST = 0,    /* [2, num_blocks, block_size, num_heads, head_dim] (FlashAttention NHD) */
  ORIGAMI_BLOCKS_FIRST = 1 /* [num_blocks, 2, block_size, num_heads, head_dim]                     */
};

/* One layer of a paged KV cache (device memory, contiguous in the layout above). */
typedef struct origami_paged_kv {
  void* d_data;
  int32_t layout;     /* ORIGAMI_KV_FIRST or ORIGAMI_BLOCKS_FIRST */
  int32_t elem_bytes; /* 2 (bf16 / fp16); the plane split works on the raw 16 bits */
  int64_t num_blocks;
  int64_t block_size;
  int64_t num_heads;
  int64_t head_dim;
} origami_paged_kv;

/* Plane split of a 16-bit element: plane p holds (x >> shift[p]) & ((1 << bits[p]) - 1).
 * The planes must cover bits 0..15 exactly once; every plane has 1..8 bits. */
#define ORIGAMI_MAX_PLANES 8
typedef struct origami_planes {
  int32_t num_planes;
  int32_t shift[ORIGAMI_MAX_PLANES];
  int32_t bits[ORIGAMI_MAX_PLANES];
} origami_planes;

/* Chunk table of one layer in the plane format.
 * The same `num_specs` specs (rows of 6 int64, the planner's output) apply to every
 * component; component q = kv * num_planes + p (K planes first, then V planes) and
 * chunk k = q * num_specs + s. offsets[k] is the byte offset of chunk k inside the
 * layer's packed buffer, offsets[2 * num_planes * num_specs] the total byte count.
 * Device copies feed the kernels; host copies are validated and size the launch. */
typedef struct origami_chunk_table {
  const int64_t* d_specs;
  const int64_t* d_offsets;
  const int64_t* h_specs;
  const int64_t* h_offsets;
  int64_t num_specs;
} origami_chunk_table;

/* ---------------------------------------------------------------------------------
 * Library
 * ------------------------------------------------------------------------------- */
int32_t origami_b200_version(void);
const char* origami_last_error(void);
/* Packed bytes of a chunk of `symbols` symbols at `bits` bits
 * (replaces packed_bytes_for_symbols, bitpack_layout_cuda.cpp:183-185). */
int64_t origami_packed_bytes(int64_t symbols, int32_t bits);

/* ---------------------------------------------------------------------------------
 * Canonical chunk ops on uint8 symbol tensors
 * ------------------------------------------------------------------------------- */

/* Drop-in for unpack_canonical_storage_chunks_cuda (bitpack_layout_cuda.cpp:316-400,
 * bound at cpp:894-903, called by lossless/native_gpu.py:113-146).
 * Same arguments and checks: flat_chunks holds every chunk back to back; offsets has
 * num_chunks + 1 entries; bits_per_chunk 1..8; chunk_specs [num_chunks][6]; source
 * shape of rank 3 or 4; axis_positions = {token, head, head_dim, layer or -1}.
 * Writes the symbols into d_output (prod(shape) bytes, source layout); positions no
 * chunk covers are zero, as in the reference. Tables are passed both on the device
 * (read by the kernels) and on the host (validated, no device->host copies). */
int32_t origami_unpack_canonical_storage_chunks(
    const uint8_t* d_flat_chunks, int64_t flat_bytes,
    const int64_t* d_chunk_offsets, const int64_t* d_bits_per_chunk,
    const int64_t* d_chunk_specs, const int64_t* h_chunk_offsets,
    const int64_t* h_bits_per_chunk, const int64_t* h_chunk_specs,
    int64_t num_chunks, const int64_t* h_source_shape, int32_t source_rank,
    const int64_t* h_axis_positions, int64_t token_count, int64_t num_heads,
    int64_t head_dim, uint8_t* d_output, int64_t output_bytes,
    origami_stream_t stream);

/* Inverse of the above, replacing the stub pack_canonical_storage_chunks
 * (lossless/native_cpu.py:144-151; called by worker.py:2010-2016). Symbols are
 * masked to `bits`; pad bits of a chunk's last byte are zero. d_flat_chunks must be
 * 16-byte aligned and hold offsets[num_chunks] bytes; chunks must not overlap. */
int32_t origami_pack_canonical_storage_chunks(
    const uint8_t* d_symbols, int64_t symbol_bytes,
    const int64_t* d_chunk_offsets, const int64_t* d_bits_per_chunk,
    const int64_t* d_chunk_specs, const int64_t* h_chunk_offsets,
    const int64_t* h_bits_per_chunk, const int64_t* h_chunk_specs,
    int64_t num_chunks, const int64_t* h_source_shape, int32_t source_rank,
    const int64_t* h_axis_positions, int64_t token_count, int64_t num_heads,
    int64_t head_dim, uint8_t* d_flat_chunks, int64_t flat_bytes,
    origami_stream_t stream);

/* ---------------------------------------------------------------------------------
 * Fused layer ops on the paged cache (plane format)
 * ------------------------------------------------------------------------------- */

/* Save side of one layer: gather the first num_tokens tokens of a request through
 * d_block_ids[ceil(num_tokens / block_size)] (int64), split K and V into planes and
 * pack every component in canonical order into d_packed (16-byte aligned,
 * h_offsets[last] bytes). Replaces _select_blocks + quantize + _pack_quantized_symbols
 * (worker.py:1887-1897, 1899-2040). The chunk specs must have token range
 * [0, num_tokens) and partition (head, channel) of the cache's heads. */
int32_t origami_pack_layer_from_paged(
    const origami_paged_kv* cache, const int64_t* d_block_ids,
    int64_t num_block_ids, int64_t num_tokens, const origami_planes* planes,
    const origami_chunk_table* table, uint8_t* d_packed, int64_t packed_bytes,
    uint32_t* d_error_count, origami_stream_t stream);

/* Restore side of one layer: unpack every component, merge the planes and scatter
 * tokens [0, num_tokens) into the paged cache through d_block_ids. Slots of the last
 * block past num_tokens are left untouched. Replaces the GPU bit-unpack + dequantize +
 * copy_kv_to_hbm of worker.py:1087-1248 (native_gpu.py:113-146,
 * benchmark_utils.py:434-532). */
int32_t origami_restore_layer_to_paged(
    const uint8_t* d_packed, int64_t packed_bytes, const origami_planes* planes,
    const origami_chunk_table* table, const origami_paged_kv* cache,
    const int64_t* d_block_ids, int64_t num_block_ids, int64_t num_tokens,
    uint32_t* d_error_count, origami_stream_t stream);

/* Prefix restore: the first restore_tokens (1..num_tokens) tokens of a num_tokens-token
 * packed layer go to the cache; the other token rows are left as they are, and only the
 * first ceil(restore_tokens / block_size) block ids are read. Replaces the reference's
 * partial restore, which narrows the dequantized layer to the request's token count and
 * copies that many tokens' blocks (worker.py:116-130, 1133-1139, 1165). */
int32_t origami_restore_layer_prefix_to_paged(
    const uint8_t* d_packed, int64_t packed_bytes, const origami_planes* planes,
    const origami_chunk_table* table, const origami_paged_kv* cache,
    const int64_t* d_block_ids, int64_t num_block_ids, int64_t num_tokens, int64_t restore_tokens,
    uint32_t* d_error_count, origami_stream_t stream);

/* One job of a batched layer op: a layer (or a request) whose packed bytes start at
 * d_packed + j * job_stride and whose rows live in d_kv_cache (the shared geometry). */
typedef struct origami_layer_job {
  void* d_kv_cache;
  const int64_t* d_block_ids; /* int64, device */
  int64_t num_block_ids;
} origami_layer_job;

/* Batched restore of num_jobs layers / requests that share one chunk table (same token
 * count, heads, head_dim, planes and chunk sizes) and cache geometry (`cache`; its d_data
 * is not used), in as few launches as possible. job_stride is a multiple of 16 bytes and
 * at least h_offsets[last]; d_packed holds packed_bytes bytes. Same results as one
 * origami_restore_layer_to_paged per job. No counterpart in the reference, which restores
 * one layer of one request per call (worker.py:1087-1248): batching amortises the launch
 * tail over a whole step. */
int32_t origami_restore_layers_to_paged(
    const uint8_t* d_packed, int64_t packed_bytes, int64_t job_stride, const origami_planes* planes,
    const origami_chunk_table* table, const origami_paged_kv* cache, const origami_layer_job* jobs,
    int32_t num_jobs, int64_t num_tokens, uint32_t* d_error_count, origami_stream_t stream);

/* Batched save: the inverse of origami_restore_layers_to_paged (same job conventions);
 * job j's chunks are written at d_packed + j * job_stride. */
int32_t origami_pack_layers_from_paged(
    const origami_paged_kv* cache, const origami_layer_job* jobs, int32_t num_jobs, int64_t num_tokens,
    const origami_planes* planes, const origami_chunk_table* table, uint8_t* d_packed, int64_t packed_bytes,
    int64_t job_stride, uint32_t* d_error_count, origami_stream_t stream);

/* ---------------------------------------------------------------------------------
 * Raw-bytes path (the reference's lossless RawBytesTensorAdapter layout)
 * ------------------------------------------------------------------------------- */

/* index_select of d_block_ids[num_block_ids] along the cache's block dimension into
 * d_out ([2, n, bs, H, D] for KV_FIRST, [n, 2, bs, H, D] for BLOCKS_FIRST); the bytes
 * of d_out are the reference's raw-bytes symbols, i.e. the concatenation of its
 * 1 MiB chunks (worker.py:1881-1897, quantization/raw_tensor.py:100-122). */
int32_t origami_gather_blocks(const origami_paged_kv* cache,
                              const int64_t* d_block_ids, int64_t num_block_ids,
                              void* d_out, int64_t out_bytes,
                              uint32_t* d_error_count, origami_stream_t stream);

/* index_copy_ of d_in (layout as above) into the cache's blocks
 * (benchmark_utils.py:434-444). */
int32_t origami_scatter_blocks(const void* d_in, int64_t in_bytes,
                               const origami_paged_kv* cache,
                               const int64_t* d_block_ids, int64_t num_block_ids,
                               uint32_t* d_error_count, origami_stream_t stream);

/* ---------------------------------------------------------------------------------
 * Quantized (lossy) restore paths: fused dequantize into the paged cache
 * ------------------------------------------------------------------------------- */

/* Element types of the tensors below. */
enum {
  ORIGAMI_DTYPE_F16 = 1,
  ORIGAMI_DTYPE_BF16 = 2,
  ORIGAMI_DTYPE_F32 = 3
};

/* Drop-in for cachegen_unpack_dequantize_to_kv_cache_cuda (bitpack_layout_cuda.cpp:475-580,
 * kernel bitpack_layout_cuda.cu:348-423; called by quantization/cachegen_adapter.py:770).
 * Key / value symbol streams (token > head > head_dim order, dense LSB-first, bits 1..8)
 * live at d_bytestream + key_offset / value_offset; each element becomes
 * ((s - c) / c) * max[token] with c = bins / 2 - 1, written as cache_dtype (F16 or BF16)
 * into cache rows d_block_ids[token / block_size]. max_dtype is F16 or F32 (both tensors).
 * Same checks and messages as the reference; out-of-range block ids are skipped and, when
 * d_error_count is given, counted once per (kv, token, head) row. */
int32_t origami_cachegen_unpack_dequantize_to_kv_cache(
    const uint8_t* d_bytestream, int64_t bytestream_bytes, int64_t key_offset, int64_t key_bytes,
    int64_t value_offset, int64_t value_bytes, int64_t key_bits, int64_t value_bits, int64_t key_bins,
    int64_t value_bins, const void* d_max_key, int64_t max_key_numel, const void* d_max_value,
    int64_t max_value_numel, int32_t max_dtype, const origami_paged_kv* cache, int32_t cache_dtype,
    const int64_t* d_block_ids, int64_t num_block_ids, int64_t tokens, uint32_t* d_error_count,
    origami_stream_t stream);

/* Drop-in for cachegen_unpack_dequantize_cuda (bitpack_layout_cuda.cpp:402-473, kernel
 * bitpack_layout_cuda.cu:141-185): 2 * layers streams (all key layers, then all value
 * layers) at d_bytestream + offsets[i], bits_per_layer[i] bits each, dequantized into
 * d_output = fp16 [layers, 2, heads, tokens, head_dim] (output_bytes bytes). Offsets and
 * bits are given on the device (read by the kernel) and on the host (validated). */
int32_t origami_cachegen_unpack_dequantize(
    const uint8_t* d_bytestream, int64_t bytestream_bytes, const int64_t* d_offsets, const int64_t* h_offsets,
    int64_t num_offsets, const int64_t* d_bits_per_layer, const int64_t* h_bits_per_layer, int64_t num_bits,
    const int64_t* d_key_bins, int64_t num_key_bins, const int64_t* d_value_bins, int64_t num_value_bins,
    const void* d_max_key, int64_t max_key_numel, const void* d_max_value, int64_t max_value_numel,
    int32_t max_dtype, int64_t tokens, int64_t heads, int64_t head_dim, void* d_output, int64_t output_bytes,
    origami_stream_t stream);

/* Drop-in for kivi_dequantize_to_kv_cache_cuda (bitpack_layout_cuda.cpp:583-700, kernel
 * bitpack_layout_cuda.cu:577-683; called by quantization/kivi_adapter.py:643). Tokens
 * [0, sink_tokens) are copied from the sink tensors ([sink_tokens, heads * head_dim]);
 * body token bt of channel ch = head * head_dim + dim is fma(s, scale, zero) with s at
 * stream index (head * head_dim + dim) * body + bt (value) or (dim * heads + head) * body +
 * bt (key), value scale/zero [body, ceil(channels / group_size)] by (bt, ch / group_size),
 * key scale/zero [ceil(body / group_size), channels] by (bt / group_size, ch).
 * meta_numel = element counts of {key_scale, key_zero, value_scale, value_zero, key_sink,
 * value_sink}; meta_dtype F16 or F32 (all six). */
int32_t origami_kivi_dequantize_to_kv_cache(
    const uint8_t* d_bytestream, int64_t bytestream_bytes, int64_t key_offset, int64_t key_bytes,
    int64_t value_offset, int64_t value_bytes, int64_t bits, int64_t group_size, int64_t sink_tokens,
    const void* d_key_scale, const void* d_key_zero, const void* d_value_scale, const void* d_value_zero,
    const void* d_key_sink, const void* d_value_sink, const int64_t* meta_numel, int32_t meta_dtype,
    const origami_paged_kv* cache, int32_t cache_dtype, const int64_t* d_block_ids, int64_t num_block_ids,
    int64_t tokens, uint32_t* d_error_count, origami_stream_t stream);

/* Drop-in for fused_prefix_attention_cuda (bitpack_layout_cuda.cpp:716-890, kernel
 * bitpack_layout_cuda.cu:873-1091; called through native_gpu.py:279-420). Attention of
 * query [query_tokens, query_heads, 128] (query_dtype F16 or BF16; d_output the same) over
 * keys [0, min(sequence_length - 1, query_start_position + q)] for query token q: keys
 * below prefix_tokens from the KIVI (codec 0) or KVQuant (codec 1) symbol streams and fp16
 * metadata (meta_numel = element counts of key_scale, key_zero, value_scale, value_zero,
 * key_sink, value_sink), the others from the paged cache through the int32 block table
 * (an out-of-range block reads as zero K and V). 3-bit symbols are nibble-packed; 2, 4 and
 * 8 bits are dense. Same checks and messages as the reference.
 * d_workspace: origami_fused_prefix_attention_workspace() bytes, 16-byte aligned and zero
 * before its first use (the kernel leaves it zero again); calls sharing a workspace must
 * not overlap. d_error_flags (nullable) gets bit 31 if a bounded wait inside the kernel
 * ran out. */
int32_t origami_fused_prefix_attention(
    const uint8_t* d_bytestream, int64_t bytestream_bytes, int64_t key_offset, int64_t key_bytes,
    int64_t value_offset, int64_t value_bytes, int64_t codec, int64_t bits, int64_t group_size, int64_t sink_tokens,
    const void* d_key_scale, const void* d_key_zero, const void* d_value_scale, const void* d_value_zero,
    const void* d_key_sink, const void* d_value_sink, const int64_t* meta_numel, int32_t meta_dtype,
    const void* d_query, int32_t query_dtype, int64_t query_tokens, int64_t query_heads, int64_t head_dim,
    const origami_paged_kv* cache, int32_t cache_dtype, const int32_t* d_block_table, int64_t block_table_len,
    int64_t prefix_tokens, int64_t query_start_position, int64_t sequence_length, double softmax_scale,
    void* d_output, void* d_workspace, int64_t workspace_bytes, uint32_t* d_error_flags, origami_stream_t stream);

/* Workspace bytes origami_fused_prefix_attention needs for these shapes on the current
 * device (0 when the key range is not split). No counterpart in the reference, whose
 * kernel needs no workspace (one CTA per query token and head). */
int32_t origami_fused_prefix_attention_workspace(int64_t query_tokens, int64_t query_heads, int64_t kv_heads,
                                                 int64_t query_start_position, int64_t sequence_length,
                                                 int64_t* workspace_bytes);

/* origami_fused_prefix_attention without a caller-provided workspace: the split
 * workspace is a file-scope device array of 8 MiB per device inside the library, so the
 * call allocates nothing. It serves hosts with no device allocator of their own (plain C
 * or FFI bindings) and serving loops that must not call cudaMalloc, which can synchronise
 * the whole device. No counterpart in the reference, whose kernel needs no workspace.
 * - Shapes whose split plan needs more than 8 MiB are rejected (ORIGAMI_ERR_UNSUPPORTED,
 *   message with both sizes); use the workspace entry point for those.
 * - The first call on a device looks the array's address up (cudaGetSymbolAddress, with
 *   that device current); make that first call before any stream capture.
 * - Each call clears the arrival counters at the head of the array (cudaMemsetAsync on
 *   `stream`) before the launch; nothing else has to start at zero.
 * - All calls on a device share the one array: calls that overlap in time (other streams,
 *   other threads) race and must be serialised by the caller. */
int32_t origami_fused_prefix_attention_noalloc(
    const uint8_t* d_bytestream, int64_t bytestream_bytes, int64_t key_offset, int64_t key_bytes,
    int64_t value_offset, int64_t value_bytes, int64_t codec, int64_t bits, int64_t group_size, int64_t sink_tokens,
    const void* d_key_scale, const void* d_key_zero, const void* d_value_scale, const void* d_value_zero,
    const void* d_key_sink, const void* d_value_sink, const int64_t* meta_numel, int32_t meta_dtype,
    const void* d_query, int32_t query_dtype, int64_t query_tokens, int64_t query_heads, int64_t head_dim,
    const origami_paged_kv* cache, int32_t cache_dtype, const int32_t* d_block_table, int64_t block_table_len,
    int64_t prefix_tokens, int64_t query_start_position, int64_t sequence_length, double softmax_scale,
    void* d_output, uint32_t* d_error_flags, origami_stream_t stream);

/* ---------------------------------------------------------------------------------
 * Host codec boundary (CPU only; no CUDA calls): the ORIGQZ1 chunk bundle and raw-deflate
 * chunk coding between caller-owned host buffers (pinned staging on the restore path)
 * ------------------------------------------------------------------------------- */

/* One chunk of an ORIGQZ1 bundle: lengths from its record, the byte offset of its
 * compressed data in the bundle and of its decoded bytes in the bundle's raw output. */
typedef struct origami_dz_record {
  uint32_t raw_len;
  uint32_t comp_len;
  int64_t comp_offset;
  int64_t output_offset;
} origami_dz_record;

/* Parses the header of an ORIGQZ1 bundle (the reference's qat_bundle.dz, written at
 * store.py:694-705) with the checks and messages of qat_deflate_prepare_bundle_dp
 * (qat_deflate.cpp:1804-1860). records may be null to query the counts only; otherwise
 * it holds max_records entries. Outputs (nullable): record count, chunk_bytes, total raw
 * bytes, byte offset of the first compressed chunk. */
int32_t origami_origqz1_parse(const uint8_t* bundle, int64_t bundle_bytes, origami_dz_record* records,
                              int64_t max_records, int64_t* num_records, int64_t* chunk_bytes, int64_t* raw_bytes,
                              int64_t* payload_offset);

/* Upper bound of the raw-deflate size of raw_bytes bytes (zlib compressBound). */
int64_t origami_deflate_bound(int64_t raw_bytes);

/* Raw deflate (zlib, window bits -15, memory level 8, default strategy; the reference CPU
 * codec, lossless/cpu_qat.py:64-74) of num_chunks chunks src[src_offsets[i], +src_lengths[i])
 * into dst at dst_offsets[i], each slot at least origami_deflate_bound(src_lengths[i])
 * bytes; writes the compressed lengths. `threads` <= 0: all hardware threads. */
int32_t origami_deflate_chunks(const uint8_t* src, const int64_t* src_offsets, const int64_t* src_lengths,
                               int64_t num_chunks, int32_t level, uint8_t* dst, int64_t dst_capacity,
                               const int64_t* dst_offsets, int64_t* dst_lengths, int32_t threads);

/* Raw inflate of num_chunks chunks src[src_offsets[i], +src_lengths[i]) into
 * dst[dst_offsets[i], +dst_lengths[i]); every chunk must decode to exactly dst_lengths[i]
 * bytes (lossless/cpu_qat.py:76-84). Replaces the reference's decompress-window + torch.cat
 * + pageable copy (worker.py:796-1049): dst is the pinned staging the H2D copy reads. */
int32_t origami_inflate_chunks(const uint8_t* src, const int64_t* src_offsets, const int64_t* src_lengths,
                               int64_t num_chunks, uint8_t* dst, int64_t dst_capacity, const int64_t* dst_offsets,
                               const int64_t* dst_lengths, int32_t threads);

#ifdef __cplusplus
/* ---------------------------------------------------------------------------------
 * Self-test
 * ------------------------------------------------------------------------------- */

/* Runs the bounded-wait bail-out that every TMA / bulk-copy layer kernel takes when a copy
 * does not land in time, on a wait that cannot complete (an mbarrier expecting 16 bytes that
 * no copy delivers, nothing in flight): the kernel gives up after `polls` (1..2^22) polls,
 * sets bit 31 of *d_error_count and returns, leaving the context usable. No counterpart in
 * the reference, whose kernels have no waits. */
int32_t origami_selftest_wait_timeout(uint32_t* d_error_count, int32_t polls, origami_stream_t stream);

} /* extern "C" */
#endif

#endif /* ORIGAMI_B200_H */
