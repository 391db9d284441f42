// C ABI of liborigami_b200.so: argument validation (host tables only, no device->host
// copies), kernel selection and launches. Declarations: include/origami_b200.h.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <string>
#include <utility>
#include <vector>

#include "../../include/origami_b200.h"
#include <cudaTypedefs.h>

#include <mutex>

#include "linear_kernels.cuh"
#include "tile_kernels.cuh"
#include "tma_kernels.cuh"
#include "bulk_kernels.cuh"
#include "row_kernels.cuh"
#include "host_common.h"

namespace origami_host {

thread_local std::string g_last_error;

int32_t fail(int32_t code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int32_t cuda_fail(cudaError_t e, const char* what) {
  return fail(ORIGAMI_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int32_t after_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return ORIGAMI_OK;
}


int32_t validate_cache(const origami_paged_kv* kv, PagedGeom& g) {
  if (kv == nullptr || kv->d_data == nullptr) return fail(ORIGAMI_ERR_INVALID, "kv cache is null");
  if (kv->layout != ORIGAMI_KV_FIRST && kv->layout != ORIGAMI_BLOCKS_FIRST)
    return fail(ORIGAMI_ERR_INVALID, "unknown kv cache layout %d", kv->layout);
  if (kv->elem_bytes != 2) return fail(ORIGAMI_ERR_UNSUPPORTED, "kv cache elements must be 2 bytes (bf16/fp16)");
  if (kv->num_blocks <= 0 || kv->block_size <= 0 || kv->num_heads <= 0 || kv->head_dim <= 0)
    return fail(ORIGAMI_ERR_INVALID, "kv cache dimensions must be positive");
  if (!aligned(kv->d_data, 16)) return fail(ORIGAMI_ERR_INVALID, "kv cache must be 16-byte aligned");
  const int64_t HD = kv->num_heads * kv->head_dim;
  const int64_t slab = kv->block_size * HD;
  g.token_stride = HD;
  g.head_stride = kv->head_dim;
  if (kv->layout == ORIGAMI_KV_FIRST) {
    g.kv_stride = kv->num_blocks * slab;
    g.block_stride = slab;
  } else {
    g.kv_stride = slab;
    g.block_stride = 2 * slab;
  }
  return ORIGAMI_OK;
}

// Dynamic shared memory is raised per (kernel, device) to the largest size ever launched
// (the attribute is a maximum, so it never has to go down); resident CTAs for a
// persistent launch (SMs x blocks per SM) are cached per (kernel, device, size).
int32_t persistent_slots(const void* fn, int smem, int& resident) {
  struct Attr {
    const void* fn;
    int dev, smem_max;
  };
  struct Occ {
    const void* fn;
    int dev, smem, slots;
  };
  static std::mutex mu;
  static std::vector<Attr> attrs;
  static std::vector<Occ> occ;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  Attr* a = nullptr;
  for (Attr& x : attrs)
    if (x.fn == fn && x.dev == dev) a = &x;
  if (a == nullptr || a->smem_max < smem) {
    if ((e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess)
      return cuda_fail(e, "cudaFuncSetAttribute");
    if (a == nullptr) attrs.push_back({fn, dev, smem});
    else a->smem_max = smem;
  }
  for (const Occ& x : occ)
    if (x.fn == fn && x.dev == dev && x.smem == smem) {
      resident = x.slots;
      return ORIGAMI_OK;
    }
  int sms = 0, per_sm = 0;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
    return cuda_fail(e, "cudaDeviceGetAttribute");
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, smem)) != cudaSuccess)
    return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  resident = sms * std::max(per_sm, 1);
  occ.push_back({fn, dev, smem, resident});
  return ORIGAMI_OK;
}

}  // namespace origami_host


namespace {

using namespace origami_host;
using origami::CanonStrides;
using origami::TileArgs;

constexpr int32_t kVersion = 1;

int64_t packed_bytes_for(int64_t symbols, int64_t bits) { return (symbols * bits + 7) / 8; }

struct Spec {
  int64_t h0, h1, c0, c1, t0, t1;
  int64_t symbols() const { return (h1 - h0) * (c1 - c0) * (t1 - t0); }
};

// Mirrors read_chunk_specs (bitpack_layout_cuda.cpp:149-175).
int32_t read_specs(const int64_t* h_specs, int64_t n, int64_t T, int64_t H, int64_t D,
                   std::vector<Spec>& out) {
  if (n < 0) return fail(ORIGAMI_ERR_INVALID, "chunk count must be non-negative");
  if (n > 0 && h_specs == nullptr) return fail(ORIGAMI_ERR_INVALID, "chunk_specs host copy is null");
  out.resize(static_cast<size_t>(n));
  for (int64_t i = 0; i < n; ++i) {
    const int64_t* r = h_specs + 6 * i;
    Spec s{r[0], r[1], r[2], r[3], r[4], r[5]};
    if (!(0 <= s.h0 && s.h0 < s.h1 && s.h1 <= H))
      return fail(ORIGAMI_ERR_INVALID, "invalid head range in Origami chunk spec %lld", (long long)i);
    if (!(0 <= s.c0 && s.c0 < s.c1 && s.c1 <= D))
      return fail(ORIGAMI_ERR_INVALID, "invalid channel range in Origami chunk spec %lld", (long long)i);
    if (!(0 <= s.t0 && s.t0 < s.t1 && s.t1 <= T))
      return fail(ORIGAMI_ERR_INVALID, "invalid token range in Origami chunk spec %lld", (long long)i);
    out[static_cast<size_t>(i)] = s;
  }
  return ORIGAMI_OK;
}

// Mirrors read_source_layout (bitpack_layout_cuda.cpp:84-147); returns strides.
int32_t read_layout(const int64_t* shape, int32_t rank, const int64_t* axes, int64_t T, int64_t H,
                    int64_t D, CanonStrides& ls, int64_t& numel) {
  if (shape == nullptr || axes == nullptr) return fail(ORIGAMI_ERR_INVALID, "source layout is null");
  if (rank != 3 && rank != 4) return fail(ORIGAMI_ERR_INVALID, "Origami source layout supports rank 3 or rank 4");
  int64_t stride[4] = {1, 1, 1, 1};
  numel = 1;
  for (int i = 0; i < rank; ++i) {
    if (shape[i] <= 0) return fail(ORIGAMI_ERR_INVALID, "source_shape dimensions must be positive");
    numel *= shape[i];
  }
  for (int i = rank - 2; i >= 0; --i) stride[i] = stride[i + 1] * shape[i + 1];
  const int64_t ta = axes[0], ha = axes[1], ca = axes[2], la = axes[3];
  if (!(0 <= ta && ta < rank)) return fail(ORIGAMI_ERR_INVALID, "token axis must be present in source layout");
  if (!(0 <= ha && ha < rank)) return fail(ORIGAMI_ERR_INVALID, "head axis must be present in source layout");
  if (!(0 <= ca && ca < rank)) return fail(ORIGAMI_ERR_INVALID, "head_dim axis must be present in source layout");
  if (!(la == -1 || (0 <= la && la < rank)))
    return fail(ORIGAMI_ERR_INVALID, "layer axis must be -1 or present in source layout");
  if (shape[ta] != T) return fail(ORIGAMI_ERR_INVALID, "source token axis size must match token_count");
  if (shape[ha] != H) return fail(ORIGAMI_ERR_INVALID, "source head axis size must match num_heads");
  if (shape[ca] != D) return fail(ORIGAMI_ERR_INVALID, "source head_dim axis size must match head_dim");
  if (la != -1 && shape[la] != 1)
    return fail(ORIGAMI_ERR_INVALID, "per-layer Origami native layout requires layer axis size 1");
  if (ta == ha || ta == ca || ha == ca || la == ta || la == ha || la == ca)
    return fail(ORIGAMI_ERR_INVALID, "source layout axes must be distinct");
  ls.st = stride[ta];
  ls.sh = stride[ha];
  ls.sc = stride[ca];
  return ORIGAMI_OK;
}

// True when every (head, channel) pair is covered exactly once by full-token specs.
bool covers_head_channel_exactly(const std::vector<Spec>& specs, int64_t H, int64_t D) {
  std::vector<std::pair<int64_t, int64_t>> iv;
  for (const Spec& s : specs) {
    for (int64_t h = s.h0; h < s.h1; ++h) iv.emplace_back(h * D + s.c0, h * D + s.c1);
    if (iv.size() > (size_t)(1 << 22)) return false;
  }
  std::sort(iv.begin(), iv.end());
  int64_t at = 0;
  for (const auto& x : iv) {
    if (x.first != at) return false;
    at = x.second;
  }
  return at == H * D;
}

int tile_tokens(int64_t D) { return origami::tile_tokens_for(static_cast<int>(D)); }

// Shared-memory layout of a tile launch (must match the kernels' plane_stride /
// plane_base). Returns the dynamic smem byte count.
size_t layout_tile_smem(TileArgs& a, int elem, bool restore, const int* plane_bits) {
  const int D = a.D, TT = a.TT, P = a.P;
  size_t off = static_cast<size_t>((2 * D + 15) & ~15);
  a.rowoff_off = static_cast<int32_t>(off);
  off += static_cast<size_t>(8) * TT;
  a.meta_off = static_cast<int32_t>(off);
  off += static_cast<size_t>(16) * P * D;
  off = (off + 127) & ~static_cast<size_t>(127);
  a.data_off = static_cast<int32_t>(off);
  size_t planes_bytes = 0;
  for (int p = 0; p < P; ++p) planes_bytes += static_cast<size_t>(D) * origami::run_stride(TT, plane_bits[p], restore);
  const size_t rows_bytes = static_cast<size_t>(TT) * D * elem;
  return off + std::max(planes_bytes, rows_bytes) + 32;  // + slack for window64 / words5 over-reads
}

int classify_planes(const origami_planes& pl) {
  auto is = [&](int P, const int* sh, const int* bi) {
    if (pl.num_planes != P) return false;
    for (int p = 0; p < P; ++p)
      if (pl.shift[p] != sh[p] || pl.bits[p] != bi[p]) return false;
    return true;
  };
  const int s2[] = {8, 0}, b2[] = {8, 8};
  const int sbf[] = {7, 15, 0}, bbf[] = {8, 1, 7};
  const int sfp[] = {10, 8, 0}, bfp[] = {6, 2, 8};
  if (is(2, s2, b2)) return origami::kModeByte2;
  if (is(3, sbf, bbf)) return origami::kModeBf16Bits;
  if (is(3, sfp, bfp)) return origami::kModeFp16Bits;
  return origami::kModeGeneric;
}

int32_t validate_planes(const origami_planes* pl) {
  if (pl == nullptr) return fail(ORIGAMI_ERR_INVALID, "planes descriptor is null");
  if (pl->num_planes < 1 || pl->num_planes > ORIGAMI_MAX_PLANES)
    return fail(ORIGAMI_ERR_INVALID, "num_planes must be 1..%d", ORIGAMI_MAX_PLANES);
  uint32_t seen = 0;
  for (int p = 0; p < pl->num_planes; ++p) {
    const int s = pl->shift[p], b = pl->bits[p];
    if (b < 1 || b > 8) return fail(ORIGAMI_ERR_INVALID, "plane %d: bits must be 1..8", p);
    if (s < 0 || s + b > 16) return fail(ORIGAMI_ERR_INVALID, "plane %d: shift + bits must fit 16 bits", p);
    const uint32_t m = ((1u << b) - 1u) << s;
    if (seen & m) return fail(ORIGAMI_ERR_INVALID, "plane %d overlaps another plane", p);
    seen |= m;
  }
  if (seen != 0xFFFFu) return fail(ORIGAMI_ERR_INVALID, "planes must cover all 16 element bits");
  return ORIGAMI_OK;
}



template <int ELEM, int MODE, int DT>
int32_t launch_tiles(bool restore, TileArgs& a, size_t smem, cudaStream_t st) {
  const void* fn = restore ? reinterpret_cast<const void*>(&origami::restore_tiles<ELEM, MODE, DT>)
                           : reinterpret_cast<const void*>(&origami::pack_tiles<ELEM, MODE, DT>);
  if (smem > 48 * 1024) {
    int resident = 0;  // sets the shared-memory attribute once per (kernel, device, size)
    const int32_t rc = persistent_slots(fn, static_cast<int>(smem), resident);
    if (rc) return rc;
  }
  const int64_t tiles = static_cast<int64_t>(a.num_kv) * a.H * a.tiles_per_head;
  if (tiles <= 0) return ORIGAMI_OK;
  if (tiles > 0x7FFFFFFF) return fail(ORIGAMI_ERR_UNSUPPORTED, "too many tiles");
  const dim3 grid(static_cast<unsigned>(tiles));
  if (restore) origami::restore_tiles<ELEM, MODE, DT><<<grid, kThreads, smem, st>>>(a);
  else origami::pack_tiles<ELEM, MODE, DT><<<grid, kThreads, smem, st>>>(a);
  return after_launch(restore ? "restore_tiles launch" : "pack_tiles launch");
}

template <int ELEM, int MODE>
int32_t launch_by_dim(bool restore, TileArgs& a, size_t smem, cudaStream_t st) {
  switch (a.D) {
    case 64: return launch_tiles<ELEM, MODE, 64>(restore, a, smem, st);
    case 128: return launch_tiles<ELEM, MODE, 128>(restore, a, smem, st);
    case 256: return launch_tiles<ELEM, MODE, 256>(restore, a, smem, st);
    default: return launch_tiles<ELEM, MODE, 0>(restore, a, smem, st);
  }
}

int32_t dispatch_tiles(bool restore, int elem, int mode, TileArgs& a, size_t smem, cudaStream_t st) {
  if (elem == 1) return launch_by_dim<1, origami::kModeGeneric>(restore, a, smem, st);
  switch (mode) {
    case origami::kModeByte2: return launch_by_dim<2, origami::kModeByte2>(restore, a, smem, st);
    case origami::kModeBf16Bits: return launch_by_dim<2, origami::kModeBf16Bits>(restore, a, smem, st);
    case origami::kModeFp16Bits: return launch_by_dim<2, origami::kModeFp16Bits>(restore, a, smem, st);
    default: return launch_tiles<2, origami::kModeGeneric, 0>(restore, a, smem, st);
  }
}

// Shared by the canonical pack and unpack entry points.
int32_t canonical_common(bool restore, const uint8_t* d_packed, int64_t packed_bytes,
                         const int64_t* d_offsets, const int64_t* d_bits, const int64_t* d_specs,
                         const int64_t* h_offsets, const int64_t* h_bits, const int64_t* h_specs,
                         int64_t n, const int64_t* shape, int32_t rank, const int64_t* axes, int64_t T,
                         int64_t H, int64_t D, uint8_t* d_symbols, int64_t symbol_bytes, cudaStream_t st) {
  if (T <= 0 || H <= 0 || D <= 0) return fail(ORIGAMI_ERR_INVALID, "canonical symbol shape must be positive");
  if (T > 0x7FFFFFFF) return fail(ORIGAMI_ERR_UNSUPPORTED, "token_count must be below 2^31");
  CanonStrides ls{};
  int64_t numel = 0;
  int32_t rc = read_layout(shape, rank, axes, T, H, D, ls, numel);
  if (rc) return rc;
  if (symbol_bytes != numel)
    return fail(ORIGAMI_ERR_INVALID, "symbol tensor holds %lld bytes, layout needs %lld", (long long)symbol_bytes,
                (long long)numel);
  std::vector<Spec> specs;
  rc = read_specs(h_specs, n, T, H, D, specs);
  if (rc) return rc;
  if (n > 0 && (h_offsets == nullptr || h_bits == nullptr || d_offsets == nullptr || d_bits == nullptr ||
                d_specs == nullptr))
    return fail(ORIGAMI_ERR_INVALID, "chunk tables must be given on host and device");
  int max_bits = 1;
  int64_t max_symbols = 0;
  for (int64_t i = 0; i < n; ++i) {
    if (h_bits[i] < 1 || h_bits[i] > 8)
      return fail(ORIGAMI_ERR_INVALID, "Origami CUDA bitpack supports only 1..8 bit symbols");
    const int64_t expect = packed_bytes_for(specs[i].symbols(), h_bits[i]);
    if (h_offsets[i + 1] - h_offsets[i] != expect)
      return fail(ORIGAMI_ERR_INVALID, "Origami CUDA packed chunk byte size mismatch");
    if (h_offsets[i] < 0) return fail(ORIGAMI_ERR_INVALID, "chunk offsets must be non-negative");
    max_bits = std::max<int>(max_bits, static_cast<int>(h_bits[i]));
    max_symbols = std::max(max_symbols, specs[i].symbols());
  }
  if (n > 0 && h_offsets[n] > packed_bytes)
    return fail(ORIGAMI_ERR_INVALID, "chunk offsets exceed the flat chunk buffer (%lld > %lld)",
                (long long)h_offsets[n], (long long)packed_bytes);
  if (numel > 0 && d_symbols == nullptr) return fail(ORIGAMI_ERR_INVALID, "symbol tensor is null");
  if (n == 0 || max_symbols == 0) {
    if (restore && numel > 0) {
      const cudaError_t e = cudaMemsetAsync(d_symbols, 0, static_cast<size_t>(numel), st);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
    }
    return ORIGAMI_OK;
  }
  if (d_packed == nullptr) return fail(ORIGAMI_ERR_INVALID, "flat chunk buffer is null");

  bool full_tokens = true;
  for (const Spec& s : specs) full_tokens = full_tokens && s.t0 == 0 && s.t1 == T;
  const bool tile_ok = full_tokens && ls.sc == 1 && D % 8 == 0 && D <= 1024 && aligned(d_packed, 16) &&
                       aligned(d_symbols, 16);
  if (tile_ok) {
    TileArgs a{};
    a.rows = d_symbols;
    a.kv_stride = 0;
    a.block_stride = 0;
    a.token_stride = ls.st;
    a.head_stride = ls.sh;
    a.block_size = T;
    a.num_blocks = 1;
    a.block_ids = nullptr;
    a.packed = const_cast<uint8_t*>(d_packed);
    a.packed_bytes = packed_bytes;
    a.specs = d_specs;
    a.offsets = d_offsets;
    a.chunk_bits = d_bits;
    if (n > 32767) return fail(ORIGAMI_ERR_UNSUPPORTED, "more than 32767 chunks in one call");
    a.S = static_cast<int32_t>(n);
    a.num_kv = 1;
    a.H = static_cast<int32_t>(H);
    a.D = static_cast<int32_t>(D);
    a.T = T;
    a.write_tokens = T;  // canonical symbols: every token
    a.TT = tile_tokens(D);
    a.tiles_per_head = static_cast<int32_t>((T + a.TT - 1) / a.TT);
    a.P = 1;
    a.shift[0] = 0;
    a.bits[0] = max_bits;
    a.err = nullptr;
    const int pb[1] = {max_bits};
    const size_t smem = layout_tile_smem(a, 1, restore, pb);
    return dispatch_tiles(restore, 1, origami::kModeGeneric, a, smem, st);
  }

  // Linear path.
  if (restore) {
    bool complete = full_tokens && covers_head_channel_exactly(specs, H, D);
    if (!complete) {
      const cudaError_t e = cudaMemsetAsync(d_symbols, 0, static_cast<size_t>(numel), st);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
    }
  }
  const int64_t per_block = static_cast<int64_t>(kThreads) * 16;
  const int64_t gx = std::min<int64_t>((max_symbols + per_block - 1) / per_block, 65535);
  if (n > 65535) return fail(ORIGAMI_ERR_UNSUPPORTED, "more than 65535 chunks in one linear call");
  const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(n));
  if (restore) {
    origami::canon_unpack_linear<<<grid, kThreads, 0, st>>>(d_packed, d_offsets, d_bits, d_specs, ls, d_symbols);
    return after_launch("canon_unpack_linear launch");
  }
  origami::canon_pack_linear<<<grid, kThreads, 0, st>>>(d_symbols, d_offsets, d_bits, d_specs, ls,
                                                         const_cast<uint8_t*>(d_packed));
  return after_launch("canon_pack_linear launch");
}

// ---------------------------------------------------------------------------------------
// TMA path for the aligned plane format (see tma_kernels.cuh).
// ---------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// True when every (kv, plane) component is a dense [H*D runs][T*bits/8] byte array in
// canonical order with 16-byte aligned rows, and the tile boxes are 16-byte multiples.
bool tma_eligible(int mode, const std::vector<Spec>& specs, const int64_t* off, const origami_planes* pl,
                  int64_t T, int64_t H, int64_t D, const uint8_t* packed) {
  if (mode == origami::kModeGeneric) return false;
  if (D != 64 && D != 128 && D != 256) return false;
  if (!aligned(packed, 16)) return false;
  const int TT = tile_tokens(D);
  const int64_t S = static_cast<int64_t>(specs.size());
  const int P = pl->num_planes;
  for (int q = 0; q < 2 * P; ++q) {
    const int b = pl->bits[q % P];
    if ((T * b) % 128 != 0 || (TT * b) % 128 != 0 || TT * b / 8 > 256) return false;
    const int64_t run = T * b / 8;
    const int64_t base = off[q * S];
    if (base % 16 != 0) return false;
    for (int64_t s = 0; s < S; ++s) {
      if (off[q * S + s] != base + (specs[s].h0 * D + specs[s].c0) * run) return false;
    }
  }
  return H * D <= 0x7FFFFFFF && T * 8 <= 0x7FFFFFFF;
}

struct Job {
  void* rows;
  const int64_t* ids;
  int64_t num_ids;
};

template <int MODE, int D>
int32_t launch_tma(bool restore, const origami_paged_kv* cache, const PagedGeom& g, const Job* jobs, int num_jobs,
                   int64_t T, int64_t write_tokens, const int64_t* off, int64_t S, uint8_t* packed, int64_t job_stride, uint32_t* d_err,
                   cudaStream_t st) {
  using G = origami::TmaGeo<MODE, D>;
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return fail(ORIGAMI_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const void* fn = restore ? reinterpret_cast<const void*>(&origami::restore_tma<MODE, D>)
                           : reinterpret_cast<const void*>(&origami::pack_tma<MODE, D>);
  const int smem = restore ? G::smem_bytes : origami::PackGeo<MODE, D>::smem_bytes;
  int resident = 0;
  int32_t rc = persistent_slots(fn, smem, resident);
  if (rc) return rc;
  const int P = G::P;
  const int32_t tiles_per_head = static_cast<int32_t>((T + G::TT - 1) / G::TT);
  const int64_t tiles_per_job = 2 * cache->num_heads * tiles_per_head;
  for (int j0 = 0; j0 < num_jobs; j0 += origami::kMaxJobs) {
    const int nj = std::min(num_jobs - j0, origami::kMaxJobs);
    origami::TmaArgs a{};
    uint8_t* base = packed + static_cast<int64_t>(j0) * job_stride;
    for (int q = 0; q < 2 * P; ++q) {
      const int b = G::bits(q % P);
      const cuuint64_t dims[3] = {static_cast<cuuint64_t>(T * b / 8), static_cast<cuuint64_t>(cache->num_heads * D),
                                  static_cast<cuuint64_t>(nj)};
      const cuuint64_t strides[2] = {static_cast<cuuint64_t>(T * b / 8), static_cast<cuuint64_t>(job_stride)};
      const cuuint32_t box[3] = {static_cast<cuuint32_t>(G::TT * b / 8), static_cast<cuuint32_t>(D), 1};
      const cuuint32_t estr[3] = {1, 1, 1};
      const CUresult r = encode(&a.maps[q], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base + off[q * S], dims, strides, box,
                                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) return fail(ORIGAMI_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    }
    for (int j = 0; j < nj; ++j) {
      a.rows[j] = jobs[j0 + j].rows;
      a.block_ids[j] = jobs[j0 + j].ids;
    }
    a.kv_stride = g.kv_stride;
    a.block_stride = g.block_stride;
    a.token_stride = g.token_stride;
    a.head_stride = g.head_stride;
    a.block_size = cache->block_size;
    a.num_blocks = cache->num_blocks;
    a.T = T;
    a.write_tokens = write_tokens;
    a.H = static_cast<int32_t>(cache->num_heads);
    a.tiles_per_head = tiles_per_head;
    const int64_t tiles = tiles_per_job * nj;
    if (tiles > 0x7FFFFFFF) return fail(ORIGAMI_ERR_UNSUPPORTED, "too many tiles");
    a.tiles_per_job = static_cast<int32_t>(tiles_per_job);
    a.num_tiles = static_cast<int32_t>(tiles);
    a.err = d_err;
    const int grid = static_cast<int>(std::min<int64_t>(tiles, resident));
    if (restore) origami::restore_tma<MODE, D><<<grid, kThreads, smem, st>>>(a);
    else origami::pack_tma<MODE, D><<<grid, kThreads, smem, st>>>(a);
    rc = after_launch(restore ? "restore_tma launch" : "pack_tma launch");
    if (rc) return rc;
  }
  return ORIGAMI_OK;
}

template <int MODE>
int32_t launch_tma_by_dim(bool restore, int64_t D, const origami_paged_kv* cache, const PagedGeom& g, const Job* jobs,
                          int num_jobs, int64_t T, int64_t write_tokens, const int64_t* off, int64_t S, uint8_t* packed, int64_t job_stride,
                          uint32_t* err, cudaStream_t st) {
  switch (D) {
    case 64: return launch_tma<MODE, 64>(restore, cache, g, jobs, num_jobs, T, write_tokens, off, S, packed, job_stride, err, st);
    case 128: return launch_tma<MODE, 128>(restore, cache, g, jobs, num_jobs, T, write_tokens, off, S, packed, job_stride, err, st);
    default: return launch_tma<MODE, 256>(restore, cache, g, jobs, num_jobs, T, write_tokens, off, S, packed, job_stride, err, st);
  }
}

// Contiguous canonical format (see bulk_kernels.cuh): runs at computable bit offsets,
// any token count with T * bits a multiple of 8.
bool bulk_eligible(int mode, const std::vector<Spec>& specs, const int64_t* off, const origami_planes* pl, int64_t T,
                   int64_t D, const uint8_t* packed, int num_jobs, int64_t job_stride) {
  if (mode == origami::kModeGeneric) return false;
  if (D != 64 && D != 128 && D != 256) return false;
  if (!aligned(packed, 16) || (num_jobs > 1 && job_stride % 16 != 0)) return false;
  const int64_t S = static_cast<int64_t>(specs.size());
  const int P = pl->num_planes;
  for (int q = 0; q < 2 * P; ++q) {
    const int b = pl->bits[q % P];
    if ((T * b) % 8 != 0) return false;
    const int64_t run = T * b / 8;
    for (int64_t s = 0; s < S; ++s)
      if (off[q * S + s] != off[q * S] + (specs[s].h0 * D + specs[s].c0) * run) return false;
  }
  return true;
}

template <int MODE, int D>
int32_t launch_bulk(bool restore, const origami_paged_kv* cache, const PagedGeom& g, const Job* jobs, int num_jobs,
                    int64_t T, int64_t write_tokens, const int64_t* off, int64_t S, uint8_t* packed, int64_t packed_bytes, int64_t job_stride,
                    uint32_t* d_err, cudaStream_t st) {
  using G = origami::TmaGeo<MODE, D>;
  const void* fn = restore ? reinterpret_cast<const void*>(&origami::restore_bulk<MODE, D>)
                           : reinterpret_cast<const void*>(&origami::pack_bulk<MODE, D>);
  const int smem = restore ? origami::BulkGeo<MODE, D>::smem_bytes : origami::PackBulkGeo<MODE, D>::smem_bytes;
  int resident = 0;
  int32_t rc = persistent_slots(fn, smem, resident);
  if (rc) return rc;
  const int32_t tiles_per_head = static_cast<int32_t>((T + G::TT - 1) / G::TT);
  const int64_t tiles_per_job = 2 * cache->num_heads * tiles_per_head;
  for (int j0 = 0; j0 < num_jobs; j0 += origami::kMaxJobs) {
    const int nj = std::min(num_jobs - j0, origami::kMaxJobs);
    origami::BulkArgs a{};
    a.packed = packed + static_cast<int64_t>(j0) * job_stride;
    a.job_stride = job_stride;
    a.packed_bytes = packed_bytes - static_cast<int64_t>(j0) * job_stride;
    for (int q = 0; q < 2 * G::P; ++q) a.comp_base[q] = off[q * S];
    for (int j = 0; j < nj; ++j) {
      a.rows[j] = jobs[j0 + j].rows;
      a.block_ids[j] = jobs[j0 + j].ids;
    }
    a.kv_stride = g.kv_stride;
    a.block_stride = g.block_stride;
    a.token_stride = g.token_stride;
    a.head_stride = g.head_stride;
    a.block_size = cache->block_size;
    a.num_blocks = cache->num_blocks;
    a.T = T;
    a.write_tokens = write_tokens;
    a.H = static_cast<int32_t>(cache->num_heads);
    a.tiles_per_head = tiles_per_head;
    const int64_t tiles = tiles_per_job * nj;
    if (tiles > 0x7FFFFFFF) return fail(ORIGAMI_ERR_UNSUPPORTED, "too many tiles");
    a.tiles_per_job = static_cast<int32_t>(tiles_per_job);
    a.num_tiles = static_cast<int32_t>(tiles);
    a.err = d_err;
    const int grid = static_cast<int>(std::min<int64_t>(tiles, resident));
    if (restore) origami::restore_bulk<MODE, D><<<grid, kThreads, smem, st>>>(a);
    else origami::pack_bulk<MODE, D><<<grid, kThreads, smem, st>>>(a);
    rc = after_launch(restore ? "restore_bulk launch" : "pack_bulk launch");
    if (rc) return rc;
  }
  return ORIGAMI_OK;
}

template <int MODE>
int32_t launch_bulk_by_dim(bool restore, int64_t D, const origami_paged_kv* cache, const PagedGeom& g, const Job* jobs,
                           int num_jobs, int64_t T, int64_t write_tokens, const int64_t* off, int64_t S, uint8_t* packed,
                           int64_t packed_bytes, int64_t job_stride, uint32_t* err, cudaStream_t st) {
  switch (D) {
    case 64:
      return launch_bulk<MODE, 64>(restore, cache, g, jobs, num_jobs, T, write_tokens, off, S, packed, packed_bytes, job_stride, err, st);
    case 128:
      return launch_bulk<MODE, 128>(restore, cache, g, jobs, num_jobs, T, write_tokens, off, S, packed, packed_bytes, job_stride, err,
                                    st);
    default:
      return launch_bulk<MODE, 256>(restore, cache, g, jobs, num_jobs, T, write_tokens, off, S, packed, packed_bytes, job_stride, err,
                                    st);
  }
}

// Row kernels (row_kernels.cuh) for head_dim 128 and 256: restore for every plane preset,
// aligned (TMA) or ragged (bulk copies) runs; pack for byte planes.
template <int MODE, int D>
int32_t launch_rows(bool restore, bool ragged, const origami_paged_kv* cache, const PagedGeom& g, const Job* jobs,
                    int num_jobs, int64_t T, int64_t write_tokens, const int64_t* off, int64_t S, uint8_t* packed, int64_t packed_bytes,
                    int64_t job_stride, uint32_t* d_err, cudaStream_t st) {
  using G = origami::TmaGeo<MODE, D>;
  const void* fn;
  int smem;
  if (restore && ragged) {
    fn = reinterpret_cast<const void*>(&origami::restore_rows<MODE, D, true>);
    smem = origami::RestoreRowsGeo<MODE, D, true>::smem_bytes;
  } else if (restore) {
    fn = reinterpret_cast<const void*>(&origami::restore_rows<MODE, D, false>);
    smem = origami::RestoreRowsGeo<MODE, D, false>::smem_bytes;
  } else {
    fn = reinterpret_cast<const void*>(&origami::pack_rows<D>);
    smem = origami::PackRowsGeo<D>::smem_bytes;
  }
  const bool maps = restore && !ragged;
  auto encode = maps ? tensor_map_encoder() : nullptr;
  if (maps && encode == nullptr) return fail(ORIGAMI_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  int resident = 0;
  int32_t rc = persistent_slots(fn, smem, resident);
  if (rc) return rc;
  const int P = G::P;
  // pack tiles own PackRowsGeo::STEP tokens each (their windows overlap by LOOK tokens)
  const int64_t tile_step = restore ? G::TT : origami::PackRowsGeo<D>::STEP;
  const int32_t tiles_per_head = static_cast<int32_t>((T + tile_step - 1) / tile_step);
  const int64_t tiles_per_job = 2 * cache->num_heads * tiles_per_head;
  for (int j0 = 0; j0 < num_jobs; j0 += origami::kMaxJobs) {
    const int nj = std::min(num_jobs - j0, origami::kMaxJobs);
    origami::RowArgs a{};
    a.packed = packed + static_cast<int64_t>(j0) * job_stride;
    a.job_stride = job_stride;
    a.packed_bytes = packed_bytes - static_cast<int64_t>(j0) * job_stride;
    for (int q = 0; q < 2 * P; ++q) a.comp_base[q] = off[q * S];
    for (int p = 0; p < P; ++p) a.run_bytes[p] = T * G::bits(p) / 8;
    if (maps) {
      for (int q = 0; q < 2 * P; ++q) {
        const int b = G::bits(q % P);
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(T * b / 8), static_cast<cuuint64_t>(cache->num_heads * D),
                                    static_cast<cuuint64_t>(nj)};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(T * b / 8), static_cast<cuuint64_t>(job_stride)};
        const cuuint32_t box[3] = {static_cast<cuuint32_t>(G::TT * b / 8), static_cast<cuuint32_t>(D), 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        const CUresult r = encode(&a.maps[q], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a.packed + off[q * S], dims, strides,
                                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(ORIGAMI_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
      }
    }
    for (int j = 0; j < nj; ++j) {
      a.rows[j] = jobs[j0 + j].rows;
      a.block_ids[j] = jobs[j0 + j].ids;
    }
    a.kv_stride = g.kv_stride;
    a.block_stride = g.block_stride;
    a.token_stride = g.token_stride;
    a.head_stride = g.head_stride;
    a.block_size = cache->block_size;
    a.num_blocks = cache->num_blocks;
    a.T = T;
    a.write_tokens = write_tokens;
    a.H = static_cast<int32_t>(cache->num_heads);
    a.tiles_per_head = tiles_per_head;
    const int64_t tiles = tiles_per_job * nj;
    if (tiles > 0x7FFFFFFF) return fail(ORIGAMI_ERR_UNSUPPORTED, "too many tiles");
    a.tiles_per_job = static_cast<int32_t>(tiles_per_job);
    a.num_tiles = static_cast<int32_t>(tiles);
    a.err = d_err;
    const int grid = static_cast<int>(std::min<int64_t>(tiles, resident));
    if (restore && ragged) origami::restore_rows<MODE, D, true><<<grid, kThreads, smem, st>>>(a);
    else if (restore) origami::restore_rows<MODE, D, false><<<grid, kThreads, smem, st>>>(a);
    else origami::pack_rows<D><<<grid, kThreads, smem, st>>>(a);
    rc = after_launch(restore ? "restore_rows launch" : "pack_rows launch");
    if (rc) return rc;
  }
  return ORIGAMI_OK;
}

template <int MODE>
int32_t launch_rows_by_dim(bool restore, bool ragged, int64_t D, const origami_paged_kv* cache, const PagedGeom& g,
                           const Job* jobs, int num_jobs, int64_t T, int64_t write_tokens, const int64_t* off, int64_t S, uint8_t* packed,
                           int64_t packed_bytes, int64_t job_stride, uint32_t* err, cudaStream_t st) {
  if (D == 128)
    return launch_rows<MODE, 128>(restore, ragged, cache, g, jobs, num_jobs, T, write_tokens, off, S, packed, packed_bytes, job_stride,
                                  err, st);
  return launch_rows<MODE, 256>(restore, ragged, cache, g, jobs, num_jobs, T, write_tokens, off, S, packed, packed_bytes, job_stride,
                                err, st);
}

int32_t launch_rows_by_mode(int mode, bool restore, bool ragged, int64_t D, const origami_paged_kv* cache,
                            const PagedGeom& g, const Job* jobs, int num_jobs, int64_t T, int64_t write_tokens,
                            const int64_t* off, int64_t S,
                            uint8_t* packed, int64_t packed_bytes, int64_t job_stride, uint32_t* err, cudaStream_t st) {
  switch (mode) {
    case origami::kModeByte2:
      return launch_rows_by_dim<origami::kModeByte2>(restore, ragged, D, cache, g, jobs, num_jobs, T, write_tokens, off, S, packed,
                                                     packed_bytes, job_stride, err, st);
    case origami::kModeBf16Bits:
      return launch_rows_by_dim<origami::kModeBf16Bits>(restore, ragged, D, cache, g, jobs, num_jobs, T, write_tokens, off, S,
                                                        packed, packed_bytes, job_stride, err, st);
    default:
      return launch_rows_by_dim<origami::kModeFp16Bits>(restore, ragged, D, cache, g, jobs, num_jobs, T, write_tokens, off, S,
                                                        packed, packed_bytes, job_stride, err, st);
  }
}

// Fused layer ops over `num_jobs` jobs sharing one chunk table and cache geometry; job j's
// packed bytes start at d_packed + j * job_stride.
int32_t layer_common(bool restore, const origami_paged_kv* cache, const Job* jobs, int num_jobs, int64_t T,
                     int64_t write_tokens, const origami_planes* planes, const origami_chunk_table* table, uint8_t* d_packed,
                     int64_t packed_bytes, int64_t job_stride, uint32_t* d_err, cudaStream_t st) {
  if (cache == nullptr) return fail(ORIGAMI_ERR_INVALID, "kv cache descriptor is null");
  if (num_jobs <= 0 || jobs == nullptr) return fail(ORIGAMI_ERR_INVALID, "at least one job is required");
  origami_paged_kv geom = *cache;
  geom.d_data = jobs[0].rows;
  PagedGeom g{};
  int32_t rc = validate_cache(&geom, g);
  if (rc) return rc;
  rc = validate_planes(planes);
  if (rc) return rc;
  if (table == nullptr) return fail(ORIGAMI_ERR_INVALID, "chunk table is null");
  const int64_t H = cache->num_heads, D = cache->head_dim;
  if (D % 8 != 0 || D > 1024) return fail(ORIGAMI_ERR_UNSUPPORTED, "head_dim must be a multiple of 8, at most 1024");
  if (planes->num_planes * D > 2048) return fail(ORIGAMI_ERR_UNSUPPORTED, "num_planes * head_dim must be <= 2048");
  if (T <= 0) return fail(ORIGAMI_ERR_INVALID, "num_tokens must be positive");
  if (T > 0x7FFFFFFF || cache->block_size > 0x7FFFFFFF)
    return fail(ORIGAMI_ERR_UNSUPPORTED, "num_tokens and block_size must be below 2^31");
  if (write_tokens <= 0 || write_tokens > T)
    return fail(ORIGAMI_ERR_INVALID, "restore_tokens must be in [1, num_tokens]");
  const int64_t need_blocks = (write_tokens + cache->block_size - 1) / cache->block_size;
  for (int j = 0; j < num_jobs; ++j) {
    if (jobs[j].rows == nullptr || !aligned(jobs[j].rows, 16))
      return fail(ORIGAMI_ERR_INVALID, "job %d: kv cache must be non-null and 16-byte aligned", j);
    if (jobs[j].ids == nullptr || jobs[j].num_ids < need_blocks)
      return fail(ORIGAMI_ERR_INVALID, "block table of job %d has %lld ids, %lld tokens need %lld", j,
                  (long long)jobs[j].num_ids, (long long)T, (long long)need_blocks);
  }
  const int64_t S = table->num_specs;
  if (S <= 0 || S > 32767) return fail(ORIGAMI_ERR_INVALID, "num_specs must be 1..32767");
  if (table->d_specs == nullptr || table->d_offsets == nullptr || table->h_offsets == nullptr)
    return fail(ORIGAMI_ERR_INVALID, "chunk table pointers are null");
  std::vector<Spec> specs;
  rc = read_specs(table->h_specs, S, T, H, D, specs);
  if (rc) return rc;
  for (const Spec& s : specs)
    if (s.t0 != 0 || s.t1 != T) return fail(ORIGAMI_ERR_INVALID, "layer chunk specs must span tokens [0, num_tokens)");
  if (!covers_head_channel_exactly(specs, H, D))
    return fail(ORIGAMI_ERR_INVALID, "layer chunk specs must cover every (head, channel) exactly once");
  const int P = planes->num_planes;
  const int64_t nchunks = 2 * P * S;
  const int64_t* off = table->h_offsets;
  for (int64_t k = 0; k < nchunks; ++k) {
    const int p = static_cast<int>((k / S) % P);
    const int64_t expect = packed_bytes_for(specs[static_cast<size_t>(k % S)].symbols(), planes->bits[p]);
    if (off[k] < 0 || off[k + 1] - off[k] != expect)
      return fail(ORIGAMI_ERR_INVALID, "chunk %lld: offsets give %lld bytes, expected %lld", (long long)k,
                  (long long)(off[k + 1] - off[k]), (long long)expect);
  }
  if (num_jobs > 1 && (job_stride < off[nchunks] || job_stride % 16 != 0))
    return fail(ORIGAMI_ERR_INVALID, "job stride %lld must be a multiple of 16 holding %lld bytes",
                (long long)job_stride, (long long)off[nchunks]);
  const int64_t extent = static_cast<int64_t>(num_jobs - 1) * job_stride + off[nchunks];
  if (extent > packed_bytes)
    return fail(ORIGAMI_ERR_INVALID, "packed buffer holds %lld bytes, the chunk table needs %lld",
                (long long)packed_bytes, (long long)extent);
  if (d_packed == nullptr || !aligned(d_packed, 16)) return fail(ORIGAMI_ERR_INVALID, "packed buffer must be 16-byte aligned");
  if (num_jobs == 1) job_stride = (off[nchunks] + 15) & ~static_cast<int64_t>(15);

  const int mode = classify_planes(*planes);
  // restore_rows for every preset at head_dim 128 / 256; pack_rows for ragged byte planes
  // there (aligned byte planes pack faster through pack_tma's staged TMA stores)
  const bool aligned_runs = tma_eligible(mode, specs, off, planes, T, H, D, d_packed);
  const bool rows = (D == 128 || D == 256) && (restore || (mode == origami::kModeByte2 && !aligned_runs));
  if (rows && (aligned_runs || bulk_eligible(mode, specs, off, planes, T, D, d_packed, num_jobs, job_stride)))
    return launch_rows_by_mode(mode, restore, !aligned_runs, D, &geom, g, jobs, num_jobs, T, write_tokens, off, S, d_packed,
                               packed_bytes, job_stride, d_err, st);
  if (aligned_runs) {
    switch (mode) {
      case origami::kModeByte2:
        return launch_tma_by_dim<origami::kModeByte2>(restore, D, &geom, g, jobs, num_jobs, T, write_tokens, off, S, d_packed,
                                                      job_stride, d_err, st);
      case origami::kModeBf16Bits:
        return launch_tma_by_dim<origami::kModeBf16Bits>(restore, D, &geom, g, jobs, num_jobs, T, write_tokens, off, S, d_packed,
                                                         job_stride, d_err, st);
      default:
        return launch_tma_by_dim<origami::kModeFp16Bits>(restore, D, &geom, g, jobs, num_jobs, T, write_tokens, off, S, d_packed,
                                                         job_stride, d_err, st);
    }
  }
  if (bulk_eligible(mode, specs, off, planes, T, D, d_packed, num_jobs, job_stride)) {
    switch (mode) {
      case origami::kModeByte2:
        return launch_bulk_by_dim<origami::kModeByte2>(restore, D, &geom, g, jobs, num_jobs, T, write_tokens, off, S, d_packed,
                                                       packed_bytes, job_stride, d_err, st);
      case origami::kModeBf16Bits:
        return launch_bulk_by_dim<origami::kModeBf16Bits>(restore, D, &geom, g, jobs, num_jobs, T, write_tokens, off, S, d_packed,
                                                          packed_bytes, job_stride, d_err, st);
      default:
        return launch_bulk_by_dim<origami::kModeFp16Bits>(restore, D, &geom, g, jobs, num_jobs, T, write_tokens, off, S, d_packed,
                                                          packed_bytes, job_stride, d_err, st);
    }
  }

  TileArgs a{};
  a.kv_stride = g.kv_stride;
  a.block_stride = g.block_stride;
  a.token_stride = g.token_stride;
  a.head_stride = g.head_stride;
  a.block_size = cache->block_size;
  a.num_blocks = cache->num_blocks;
  a.specs = table->d_specs;
  a.offsets = table->d_offsets;
  a.chunk_bits = nullptr;
  a.S = static_cast<int32_t>(S);
  a.num_kv = 2;
  a.H = static_cast<int32_t>(H);
  a.D = static_cast<int32_t>(D);
  a.T = T;
  a.write_tokens = write_tokens;
  a.TT = tile_tokens(D);
  a.tiles_per_head = static_cast<int32_t>((T + a.TT - 1) / a.TT);
  a.P = P;
  for (int p = 0; p < P; ++p) {
    a.shift[p] = planes->shift[p];
    a.bits[p] = planes->bits[p];
  }
  a.err = d_err;
  const size_t smem = layout_tile_smem(a, 2, restore, planes->bits);
  if (smem > 227 * 1024) return fail(ORIGAMI_ERR_UNSUPPORTED, "tile needs %zu bytes of shared memory", smem);
  for (int j = 0; j < num_jobs; ++j) {
    a.rows = jobs[j].rows;
    a.block_ids = jobs[j].ids;
    a.packed = d_packed + static_cast<int64_t>(j) * job_stride;
    a.packed_bytes = packed_bytes - static_cast<int64_t>(j) * job_stride;
    rc = dispatch_tiles(restore, 2, mode, a, smem, st);
    if (rc) return rc;
  }
  return ORIGAMI_OK;
}

int32_t slab_geometry(const origami_paged_kv* cache, int64_t num_block_ids, int64_t bytes, int64_t& slab,
                      int64_t& per_id) {
  PagedGeom g{};
  int32_t rc = validate_cache(cache, g);
  if (rc) return rc;
  const int64_t slab_elems = cache->block_size * cache->num_heads * cache->head_dim;
  if (cache->layout == ORIGAMI_KV_FIRST) {
    slab = slab_elems * cache->elem_bytes;
    per_id = 2;
  } else {
    slab = 2 * slab_elems * cache->elem_bytes;
    per_id = 1;
  }
  if (slab % 16 != 0) return fail(ORIGAMI_ERR_UNSUPPORTED, "block slab must be a multiple of 16 bytes");
  if (num_block_ids < 0) return fail(ORIGAMI_ERR_INVALID, "num_block_ids must be non-negative");
  if (bytes != per_id * slab * num_block_ids)
    return fail(ORIGAMI_ERR_INVALID, "buffer holds %lld bytes, %lld blocks need %lld", (long long)bytes,
                (long long)num_block_ids, (long long)(per_id * slab * num_block_ids));
  return ORIGAMI_OK;
}

int slab_grid(int64_t slabs) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(slabs, static_cast<int64_t>(sms) * 8)));
}

}  // namespace

namespace origami {

// Self-test of the bounded-wait bail-out the layer kernels share (stage_wait_or_bail):
// the mbarrier expects 16 bytes that no copy will deliver, so the CTA's wait runs out with
// nothing in flight, and the CTA flags kWaitTimeoutFlag and leaves exactly as a layer
// kernel whose copy never landed would.
__global__ void selftest_wait_timeout(uint32_t* err, uint32_t polls) {
  __shared__ __align__(8) uint64_t bar[2];
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_expect_tx(&bar[0], 16);  // a transaction no copy completes
  if (stage_wait_or_bail(&bar[0], 0, &bar[1], 0, false, err, polls)) return;
  if (threadIdx.x == 0) atomicAdd(err, 1u);  // reached only if the phase completed
}

}  // namespace origami

extern "C" {

int32_t origami_b200_version(void) { return kVersion; }

const char* origami_last_error(void) { return origami_host::g_last_error.c_str(); }

int64_t origami_packed_bytes(int64_t symbols, int32_t bits) { return packed_bytes_for(symbols, bits); }

int32_t origami_unpack_canonical_storage_chunks(
    const uint8_t* d_flat_chunks, int64_t flat_bytes, const int64_t* d_chunk_offsets,
    const int64_t* d_bits_per_chunk, const int64_t* d_chunk_specs, const int64_t* h_chunk_offsets,
    const int64_t* h_bits_per_chunk, const int64_t* h_chunk_specs, int64_t num_chunks,
    const int64_t* h_source_shape, int32_t source_rank, const int64_t* h_axis_positions, int64_t token_count,
    int64_t num_heads, int64_t head_dim, uint8_t* d_output, int64_t output_bytes, origami_stream_t stream) {
  return canonical_common(true, d_flat_chunks, flat_bytes, d_chunk_offsets, d_bits_per_chunk, d_chunk_specs,
                          h_chunk_offsets, h_bits_per_chunk, h_chunk_specs, num_chunks, h_source_shape,
                          source_rank, h_axis_positions, token_count, num_heads, head_dim, d_output, output_bytes,
                          reinterpret_cast<cudaStream_t>(stream));
}

int32_t origami_pack_canonical_storage_chunks(
    const uint8_t* d_symbols, int64_t symbol_bytes, const int64_t* d_chunk_offsets,
    const int64_t* d_bits_per_chunk, const int64_t* d_chunk_specs, const int64_t* h_chunk_offsets,
    const int64_t* h_bits_per_chunk, const int64_t* h_chunk_specs, int64_t num_chunks,
    const int64_t* h_source_shape, int32_t source_rank, const int64_t* h_axis_positions, int64_t token_count,
    int64_t num_heads, int64_t head_dim, uint8_t* d_flat_chunks, int64_t flat_bytes, origami_stream_t stream) {
  return canonical_common(false, d_flat_chunks, flat_bytes, d_chunk_offsets, d_bits_per_chunk, d_chunk_specs,
                          h_chunk_offsets, h_bits_per_chunk, h_chunk_specs, num_chunks, h_source_shape,
                          source_rank, h_axis_positions, token_count, num_heads, head_dim,
                          const_cast<uint8_t*>(d_symbols), symbol_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int32_t origami_pack_layer_from_paged(const origami_paged_kv* cache, const int64_t* d_block_ids,
                                      int64_t num_block_ids, int64_t num_tokens, const origami_planes* planes,
                                      const origami_chunk_table* table, uint8_t* d_packed, int64_t packed_bytes,
                                      uint32_t* d_error_count, origami_stream_t stream) {
  if (cache == nullptr) return fail(ORIGAMI_ERR_INVALID, "kv cache is null");
  const Job job{cache->d_data, d_block_ids, num_block_ids};
  return layer_common(false, cache, &job, 1, num_tokens, num_tokens, planes, table, d_packed, packed_bytes, 0,
                      d_error_count, reinterpret_cast<cudaStream_t>(stream));
}

int32_t origami_restore_layer_to_paged(const uint8_t* d_packed, int64_t packed_bytes, const origami_planes* planes,
                                       const origami_chunk_table* table, const origami_paged_kv* cache,
                                       const int64_t* d_block_ids, int64_t num_block_ids, int64_t num_tokens,
                                       uint32_t* d_error_count, origami_stream_t stream) {
  if (cache == nullptr) return fail(ORIGAMI_ERR_INVALID, "kv cache is null");
  const Job job{cache->d_data, d_block_ids, num_block_ids};
  return layer_common(true, cache, &job, 1, num_tokens, num_tokens, planes, table, const_cast<uint8_t*>(d_packed),
                      packed_bytes, 0, d_error_count, reinterpret_cast<cudaStream_t>(stream));
}

int32_t origami_restore_layer_prefix_to_paged(const uint8_t* d_packed, int64_t packed_bytes,
                                              const origami_planes* planes, const origami_chunk_table* table,
                                              const origami_paged_kv* cache, const int64_t* d_block_ids,
                                              int64_t num_block_ids, int64_t num_tokens, int64_t restore_tokens,
                                              uint32_t* d_error_count, origami_stream_t stream) {
  if (cache == nullptr) return fail(ORIGAMI_ERR_INVALID, "kv cache is null");
  const Job job{cache->d_data, d_block_ids, num_block_ids};
  return layer_common(true, cache, &job, 1, num_tokens, restore_tokens, planes, table, const_cast<uint8_t*>(d_packed),
                      packed_bytes, 0, d_error_count, reinterpret_cast<cudaStream_t>(stream));
}

static int32_t jobs_from(const origami_layer_job* jobs, int32_t n, std::vector<Job>& out) {
  if (jobs == nullptr || n <= 0) return fail(ORIGAMI_ERR_INVALID, "at least one job is required");
  out.resize(static_cast<size_t>(n));
  for (int32_t j = 0; j < n; ++j) out[j] = Job{jobs[j].d_kv_cache, jobs[j].d_block_ids, jobs[j].num_block_ids};
  return ORIGAMI_OK;
}

int32_t origami_pack_layers_from_paged(const origami_paged_kv* cache, const origami_layer_job* jobs, int32_t num_jobs,
                                       int64_t num_tokens, const origami_planes* planes,
                                       const origami_chunk_table* table, uint8_t* d_packed, int64_t packed_bytes,
                                       int64_t job_stride, uint32_t* d_error_count, origami_stream_t stream) {
  std::vector<Job> js;
  const int32_t rc = jobs_from(jobs, num_jobs, js);
  if (rc) return rc;
  return layer_common(false, cache, js.data(), num_jobs, num_tokens, num_tokens, planes, table, d_packed, packed_bytes,
                      job_stride, d_error_count, reinterpret_cast<cudaStream_t>(stream));
}

int32_t origami_restore_layers_to_paged(const uint8_t* d_packed, int64_t packed_bytes, int64_t job_stride,
                                        const origami_planes* planes, const origami_chunk_table* table,
                                        const origami_paged_kv* cache, const origami_layer_job* jobs,
                                        int32_t num_jobs, int64_t num_tokens, uint32_t* d_error_count,
                                        origami_stream_t stream) {
  std::vector<Job> js;
  const int32_t rc = jobs_from(jobs, num_jobs, js);
  if (rc) return rc;
  return layer_common(true, cache, js.data(), num_jobs, num_tokens, num_tokens, planes, table,
                      const_cast<uint8_t*>(d_packed), packed_bytes, job_stride, d_error_count,
                      reinterpret_cast<cudaStream_t>(stream));
}

int32_t origami_gather_blocks(const origami_paged_kv* cache, const int64_t* d_block_ids, int64_t num_block_ids,
                              void* d_out, int64_t out_bytes, uint32_t* d_error_count, origami_stream_t stream) {
  int64_t slab = 0, per_id = 0;
  int32_t rc = slab_geometry(cache, num_block_ids, out_bytes, slab, per_id);
  if (rc) return rc;
  if (num_block_ids == 0) return ORIGAMI_OK;
  if (d_block_ids == nullptr || d_out == nullptr || !aligned(d_out, 16))
    return fail(ORIGAMI_ERR_INVALID, "block ids / output must be non-null, output 16-byte aligned");
  const int grid = slab_grid(per_id * num_block_ids);
  origami::gather_slabs<<<grid, kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(cache->d_data), slab, per_id, cache->num_blocks, d_block_ids, num_block_ids,
      static_cast<uint8_t*>(d_out), d_error_count);
  return after_launch("gather_slabs launch");
}

int32_t origami_scatter_blocks(const void* d_in, int64_t in_bytes, const origami_paged_kv* cache,
                               const int64_t* d_block_ids, int64_t num_block_ids, uint32_t* d_error_count,
                               origami_stream_t stream) {
  int64_t slab = 0, per_id = 0;
  int32_t rc = slab_geometry(cache, num_block_ids, in_bytes, slab, per_id);
  if (rc) return rc;
  if (num_block_ids == 0) return ORIGAMI_OK;
  if (d_block_ids == nullptr || d_in == nullptr || !aligned(d_in, 16))
    return fail(ORIGAMI_ERR_INVALID, "block ids / input must be non-null, input 16-byte aligned");
  const int grid = slab_grid(per_id * num_block_ids);
  origami::scatter_slabs<<<grid, kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(d_in), slab, per_id, cache->num_blocks, d_block_ids, num_block_ids,
      static_cast<uint8_t*>(cache->d_data), d_error_count);
  return after_launch("scatter_slabs launch");
}

int32_t origami_selftest_wait_timeout(uint32_t* d_error_count, int32_t polls, origami_stream_t stream) {
  if (d_error_count == nullptr) return fail(ORIGAMI_ERR_INVALID, "error word is null");
  if (polls <= 0 || polls > static_cast<int32_t>(origami::kWaitPolls))
    return fail(ORIGAMI_ERR_INVALID, "polls must be 1..%u", origami::kWaitPolls);
  origami::selftest_wait_timeout<<<1, kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      d_error_count, static_cast<uint32_t>(polls));
  return after_launch("selftest_wait_timeout launch");
}

}  // extern "C"
