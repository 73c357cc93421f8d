// In-kernel bounds checks for debug builds: `FYB_BOUNDS_CHECK=1 python setup.py build_ext --inplace` compiles every
// FYB_IN_BOUNDS(i, n, site) into a check of 0 <= i < n; a failing index records (kBounds << 16 | site) in the device
// status word (the first failure wins; word[1] keeps the index's low 32 bits) and the caller skips the access, so the
// kernel finishes and the host reads the failure (utils/faults.py DeviceStatus) instead of the GPU faulting. Used
// where an index comes from data or from a table the host built: token ids, cross-entropy targets, exchange piece
// tables, owner-map results. Release builds compile the checks to `true`.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"

namespace fyb {

#ifdef FYB_BOUNDS_CHECK
// this translation unit's pointer to the status word; set per device by its binder (FYB_BOUNDS_BINDER) when
// status_ptr() allocates the word
static __device__ int* g_bounds_status = nullptr;

__host__ __device__ __forceinline__ bool bounds_ok(int64_t i, int64_t n, int site) {
  if (i >= 0 && i < n) return true;
#ifdef __CUDA_ARCH__
  int* s = g_bounds_status;
  if (s != nullptr && atomicCAS(s, 0, (kBounds << 16) | (site & 0xffff)) == 0) s[1] = static_cast<int>(i);
#endif
  return false;
}

#define FYB_IN_BOUNDS(i, n, site) ::fyb::bounds_ok(static_cast<int64_t>(i), static_cast<int64_t>(n), (site))
#define FYB_BOUNDS_BINDER(fn) \
  void fn(int* p) { FYB_CUDA(cudaMemcpyToSymbol(g_bounds_status, &p, sizeof(p))); }
#else
#define FYB_IN_BOUNDS(i, n, site) true
#define FYB_BOUNDS_BINDER(fn) \
  void fn(int*) {}
#endif

}  // namespace fyb
