// Host side of the save / restore path: the ORIGQZ1 chunk bundle and raw-deflate chunk
// coding straight between caller-owned (pinned) host buffers, spread over threads.
//
// * ORIGQZ1 is the reference's qat_bundle.dz (written by store.py:694-705, parsed by
//   qat_deflate_prepare_bundle_dp, qat_deflate.cpp:1804-1860): "ORIGQZ1\0", u32 chunk
//   bytes, u32 chunk count, u64 raw bytes, one (u32 raw length, u32 compressed length)
//   record per chunk, then the compressed chunks back to back. The checks and messages
//   are the reference parser's.
// * The codec is the reference CPU codec's (lossless/cpu_qat.py:64-84): zlib raw deflate
//   (window bits -15), level 1, default strategy, memory level 8. With the same zlib the
//   streams are byte-identical; decoding checks each chunk's length like cpu_qat.py:79-84.
// * Decoding writes every chunk of a window at its own offset of one output buffer (the
//   restore path's pinned staging slot), so the host->device copy reads it with no
//   concatenation or pageable bounce (the reference copies decoded chunks with torch.cat
//   and a pageable .to(device), worker.py:796-1049, benchmark_utils.py:438).
#include <zlib.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <thread>
#include <vector>

#include "host_common.h"

namespace {

using namespace origami_host;

constexpr uint8_t kMagic[8] = {'O', 'R', 'I', 'G', 'Q', 'Z', '1', '\0'};
constexpr uint32_t kMaxCompressedChunk = 64u * 1024u * 1024u;  // qat_deflate.cpp:48

uint32_t load_u32(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) | (static_cast<uint32_t>(p[2]) << 16) |
         (static_cast<uint32_t>(p[3]) << 24);
}

uint64_t load_u64(const uint8_t* p) { return static_cast<uint64_t>(load_u32(p)) | (static_cast<uint64_t>(load_u32(p + 4)) << 32); }

int worker_count(int32_t threads, int64_t items) {
  int n = threads > 0 ? threads : static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(n, items)));
}

// Runs fn(i) for i in [0, n) on `workers` threads (the calling thread is one of them);
// returns the first nonzero status.
template <typename Fn>
int32_t parallel_for(int64_t n, int workers, Fn fn) {
  std::atomic<int64_t> next{0};
  std::atomic<int32_t> status{ORIGAMI_OK};
  auto body = [&]() {
    for (;;) {
      if (status.load(std::memory_order_relaxed) != ORIGAMI_OK) return;
      const int64_t i = next.fetch_add(1);
      if (i >= n) return;
      const int32_t rc = fn(i);
      if (rc != ORIGAMI_OK) {
        int32_t ok = ORIGAMI_OK;
        status.compare_exchange_strong(ok, rc);
      }
    }
  };
  std::vector<std::thread> pool;
  pool.reserve(static_cast<size_t>(workers > 0 ? workers - 1 : 0));
  for (int w = 1; w < workers; ++w) pool.emplace_back(body);
  body();
  for (std::thread& t : pool) t.join();
  return status.load();
}

struct ChunkError {
  int64_t index = -1;
  int64_t got = 0;
  int code = Z_OK;
};

}  // namespace

extern "C" {

int32_t origami_origqz1_parse(const uint8_t* bundle, int64_t bundle_bytes, origami_dz_record* records,
                              int64_t max_records, int64_t* num_records, int64_t* chunk_bytes, int64_t* raw_bytes,
                              int64_t* payload_offset) {
  if (bundle == nullptr || bundle_bytes < 24) return fail(ORIGAMI_ERR_INVALID, "ORIGQZ1 bundle is too small");
  if (std::memcmp(bundle, kMagic, sizeof(kMagic)) != 0) return fail(ORIGAMI_ERR_INVALID, "invalid ORIGQZ1 bundle magic");
  const uint32_t cb = load_u32(bundle + 8);
  const uint32_t count = load_u32(bundle + 12);
  const uint64_t raw = load_u64(bundle + 16);
  if (cb == 0) return fail(ORIGAMI_ERR_INVALID, "ORIGQZ1 chunk_bytes must be positive");
  if (count == 0) return fail(ORIGAMI_ERR_INVALID, "ORIGQZ1 chunk_count must be positive");
  const uint64_t header = 24ull + 8ull * count;
  if (header > static_cast<uint64_t>(bundle_bytes))
    return fail(ORIGAMI_ERR_INVALID, "ORIGQZ1 record table exceeds bundle size");
  if (num_records) *num_records = count;
  if (chunk_bytes) *chunk_bytes = cb;
  if (raw_bytes) *raw_bytes = static_cast<int64_t>(raw);
  if (payload_offset) *payload_offset = static_cast<int64_t>(header);
  if (records != nullptr && max_records < static_cast<int64_t>(count))
    return fail(ORIGAMI_ERR_INVALID, "record buffer holds %lld records, the bundle has %u", (long long)max_records,
                count);
  uint64_t raw_sum = 0, comp_sum = 0;
  for (uint32_t i = 0; i < count; ++i) {
    const uint8_t* p = bundle + 24 + 8ull * i;
    const uint32_t rl = load_u32(p), cl = load_u32(p + 4);
    if (rl == 0 || rl > cb) return fail(ORIGAMI_ERR_INVALID, "invalid ORIGQZ1 raw chunk length");
    if (cl == 0) return fail(ORIGAMI_ERR_INVALID, "invalid ORIGQZ1 compressed chunk length");
    if (cl >= kMaxCompressedChunk)
      return fail(ORIGAMI_ERR_INVALID, "ORIGQZ1 prepared restore only supports compressed chunks below 64 MiB");
    if (records != nullptr) records[i] = origami_dz_record{rl, cl, static_cast<int64_t>(header + comp_sum),
                                                           static_cast<int64_t>(raw_sum)};
    raw_sum += rl;
    comp_sum += cl;
  }
  if (raw_sum != raw) return fail(ORIGAMI_ERR_INVALID, "ORIGQZ1 raw size mismatch");
  if (header + comp_sum != static_cast<uint64_t>(bundle_bytes))
    return fail(ORIGAMI_ERR_INVALID, "ORIGQZ1 compressed payload size mismatch");
  return ORIGAMI_OK;
}

int64_t origami_deflate_bound(int64_t raw_bytes) {
  return raw_bytes < 0 ? -1 : static_cast<int64_t>(compressBound(static_cast<uLong>(raw_bytes)));
}

int32_t origami_deflate_chunks(const uint8_t* src, const int64_t* src_offsets, const int64_t* src_lengths,
                               int64_t num_chunks, int32_t level, uint8_t* dst, int64_t dst_capacity,
                               const int64_t* dst_offsets, int64_t* dst_lengths, int32_t threads) {
  if (num_chunks < 0) return fail(ORIGAMI_ERR_INVALID, "num_chunks must be non-negative");
  if (num_chunks == 0) return ORIGAMI_OK;
  if (src == nullptr || dst == nullptr || src_offsets == nullptr || src_lengths == nullptr || dst_offsets == nullptr ||
      dst_lengths == nullptr)
    return fail(ORIGAMI_ERR_INVALID, "null buffer or table");
  if (level < 0 || level > 9) return fail(ORIGAMI_ERR_INVALID, "deflate level must be 0..9");
  for (int64_t i = 0; i < num_chunks; ++i) {
    if (src_lengths[i] < 0 || src_offsets[i] < 0 || src_lengths[i] > 0xFFFFFFFFll)
      return fail(ORIGAMI_ERR_INVALID, "chunk %lld: bad source range", (long long)i);
    const int64_t bound = origami_deflate_bound(src_lengths[i]);
    if (dst_offsets[i] < 0 || dst_offsets[i] + bound > dst_capacity)
      return fail(ORIGAMI_ERR_INVALID, "chunk %lld: output slot [%lld, +%lld) exceeds %lld bytes", (long long)i,
                  (long long)dst_offsets[i], (long long)bound, (long long)dst_capacity);
  }
  ChunkError err;
  std::atomic<bool> err_set{false};
  const int32_t rc = parallel_for(num_chunks, worker_count(threads, num_chunks), [&](int64_t i) -> int32_t {
    z_stream zs{};
    int code = deflateInit2(&zs, level, Z_DEFLATED, -15, 8, Z_DEFAULT_STRATEGY);
    if (code == Z_OK) {
      zs.next_in = const_cast<Bytef*>(src + src_offsets[i]);
      zs.avail_in = static_cast<uInt>(src_lengths[i]);
      zs.next_out = dst + dst_offsets[i];
      zs.avail_out = static_cast<uInt>(origami_deflate_bound(src_lengths[i]));
      code = deflate(&zs, Z_FINISH);
      dst_lengths[i] = static_cast<int64_t>(zs.total_out);
      deflateEnd(&zs);
      if (code == Z_STREAM_END) return ORIGAMI_OK;
    }
    if (!err_set.exchange(true)) err = ChunkError{i, 0, code};
    return ORIGAMI_ERR_INVALID;
  });
  if (rc != ORIGAMI_OK)
    return fail(ORIGAMI_ERR_INVALID, "deflate of chunk %lld failed (zlib status %d)", (long long)err.index, err.code);
  return ORIGAMI_OK;
}

int32_t origami_inflate_chunks(const uint8_t* src, const int64_t* src_offsets, const int64_t* src_lengths,
                               int64_t num_chunks, uint8_t* dst, int64_t dst_capacity, const int64_t* dst_offsets,
                               const int64_t* dst_lengths, int32_t threads) {
  if (num_chunks < 0) return fail(ORIGAMI_ERR_INVALID, "num_chunks must be non-negative");
  if (num_chunks == 0) return ORIGAMI_OK;
  if (src == nullptr || dst == nullptr || src_offsets == nullptr || src_lengths == nullptr || dst_offsets == nullptr ||
      dst_lengths == nullptr)
    return fail(ORIGAMI_ERR_INVALID, "null buffer or table");
  for (int64_t i = 0; i < num_chunks; ++i) {
    if (src_offsets[i] < 0 || src_lengths[i] < 0 || src_lengths[i] > 0xFFFFFFFFll)
      return fail(ORIGAMI_ERR_INVALID, "chunk %lld: bad compressed range", (long long)i);
    if (dst_offsets[i] < 0 || dst_lengths[i] < 0 || dst_lengths[i] > 0xFFFFFFFFll ||
        dst_offsets[i] + dst_lengths[i] > dst_capacity)
      return fail(ORIGAMI_ERR_INVALID, "chunk %lld: output range [%lld, +%lld) exceeds %lld bytes", (long long)i,
                  (long long)dst_offsets[i], (long long)dst_lengths[i], (long long)dst_capacity);
  }
  ChunkError err;
  std::atomic<bool> err_set{false};
  const int32_t rc = parallel_for(num_chunks, worker_count(threads, num_chunks), [&](int64_t i) -> int32_t {
    z_stream zs{};
    int code = inflateInit2(&zs, -15);
    int64_t got = 0;
    if (code == Z_OK) {
      zs.next_in = const_cast<Bytef*>(src + src_offsets[i]);
      zs.avail_in = static_cast<uInt>(src_lengths[i]);
      zs.next_out = dst + dst_offsets[i];
      zs.avail_out = static_cast<uInt>(dst_lengths[i]);
      code = inflate(&zs, Z_FINISH);
      got = static_cast<int64_t>(zs.total_out);
      // a stream longer than its slot stops with Z_BUF_ERROR / Z_OK and output left over
      if (code == Z_STREAM_END && got == dst_lengths[i]) {
        inflateEnd(&zs);
        return ORIGAMI_OK;
      }
      if (code != Z_STREAM_END) {
        uint8_t spill[256];
        while (code == Z_OK || code == Z_BUF_ERROR) {  // count what did not fit
          zs.next_out = spill;
          zs.avail_out = sizeof(spill);
          const uLong before = zs.total_out;
          code = inflate(&zs, Z_FINISH);
          if (zs.total_out == before) break;
        }
        got = static_cast<int64_t>(zs.total_out);
      }
      inflateEnd(&zs);
    }
    if (!err_set.exchange(true)) err = ChunkError{i, got, code};
    return ORIGAMI_ERR_INVALID;
  });
  if (rc != ORIGAMI_OK) {
    if (err.code == Z_STREAM_END || err.code == Z_OK || err.code == Z_BUF_ERROR)
      return fail(ORIGAMI_ERR_INVALID, "Origami CPU lossless decoded %lld bytes, expected %lld (chunk %lld)",
                  (long long)err.got, (long long)dst_lengths[err.index], (long long)err.index);
    return fail(ORIGAMI_ERR_INVALID, "inflate of chunk %lld failed (zlib status %d)", (long long)err.index, err.code);
  }
  return ORIGAMI_OK;
}

}  // extern "C"
