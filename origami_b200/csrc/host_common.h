// Host helpers shared by the translation units of liborigami_b200.so: the per-thread
// error message, CUDA error mapping, paged-cache validation and the persistent-grid
// occupancy cache.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

#include "../../include/origami_b200.h"

namespace origami_host {

constexpr int kThreads = 256;

// Records a printf-style message for origami_last_error() and returns `code`.
int32_t fail(int32_t code, const char* fmt, ...);
int32_t cuda_fail(cudaError_t e, const char* what);
// cudaGetLastError() after a launch, as an ORIGAMI_ERR_CUDA status.
int32_t after_launch(const char* what);

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Element strides of one layer's paged cache.
struct PagedGeom {
  int64_t kv_stride, block_stride, token_stride, head_stride;
};
int32_t validate_cache(const origami_paged_kv* kv, PagedGeom& g);

// Raises the kernel's dynamic shared-memory limit to `smem` (once per kernel and device)
// and returns the CTAs of kThreads threads resident on the whole device.
int32_t persistent_slots(const void* fn, int smem, int& resident);

}  // namespace origami_host
