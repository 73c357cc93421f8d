// Host-side helpers: tensor-map encoding through the driver entry point, launch checks, device properties.
#pragma once

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <nvtx3/nvToolsExt.h>

#include <cstdint>
#include <cstdlib>
#include <stdexcept>
#include <string>

namespace fyb {

#define FYB_CHECK(cond, msg)                                                         \
  do {                                                                               \
    if (!(cond)) throw std::runtime_error(std::string("faster_yoco_b200: ") + (msg)); \
  } while (0)

#define FYB_CUDA(call)                                                                               \
  do {                                                                                               \
    cudaError_t e_ = (call);                                                                         \
    if (e_ != cudaSuccess)                                                                           \
      throw std::runtime_error(std::string("faster_yoco_b200 CUDA error: ") + cudaGetErrorString(e_) + \
                               " at " + __FILE__ + ":" + std::to_string(__LINE__));                  \
  } while (0)

// Driver-API calls need the primary context current on the calling thread. Threads that only ever called
// cudaGetDevice (autograd's device threads, for instance) may have none, so bind it once per thread.
inline void ensure_context() {
  thread_local bool bound = false;
  if (!bound) {
    int d;
    FYB_CUDA(cudaGetDevice(&d));
    FYB_CUDA(cudaSetDevice(d));
    bound = true;
  }
}

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  ensure_context();
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    FYB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    FYB_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major matrix [rows, cols] with row stride ld (elements), 128-byte swizzle,
// box {64 columns, box_rows rows}. Out-of-range elements of a box read as zero.
inline CUtensorMap make_tmap_2d(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  FYB_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  FYB_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  FYB_CHECK(box_rows >= 1 && box_rows <= 256, "TMA box rows out of range");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FYB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (2d) code " + std::to_string(static_cast<int>(r)));
  return m;
}

// 3-D bf16 tensor map: dims {d0 (contiguous), d1, d2} with strides (elements) s1, s2; box {64, 1, box2}.
// Used for per-head tiles of [tokens, heads, head_dim] activations: d0 = head_dim, d1 = heads, d2 = tokens.
inline CUtensorMap make_tmap_3d(const void* base, int64_t d0, int64_t d1, int64_t d2, int64_t s1, int64_t s2,
                                int box2) {
  FYB_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  FYB_CHECK((s1 * 2) % 16 == 0 && (s2 * 2) % 16 == 0, "TMA strides must be multiples of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(s1 * 2), static_cast<cuuint64_t>(s2 * 2)};
  cuuint32_t box[3] = {64u, 1u, static_cast<cuuint32_t>(box2)};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FYB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (3d) code " + std::to_string(static_cast<int>(r)));
  return m;
}

// 3-D fp32 tensor map: dims {d0 (contiguous), d1, d2}, strides (elements) s1, s2, box {32, 1, box2}, 128-byte
// swizzle (a box row is 32 floats = 128 bytes). Used by bulk tensor reductions of fp32 accumulators.
inline CUtensorMap make_tmap_3d_f32(const void* base, int64_t d0, int64_t d1, int64_t d2, int64_t s1, int64_t s2,
                                    int box2) {
  FYB_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  FYB_CHECK((s1 * 4) % 16 == 0 && (s2 * 4) % 16 == 0, "TMA strides must be multiples of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(s1 * 4), static_cast<cuuint64_t>(s2 * 4)};
  cuuint32_t box[3] = {32u, 1u, static_cast<cuuint32_t>(box2)};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FYB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (3d f32) code " + std::to_string(static_cast<int>(r)));
  return m;
}

inline int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    FYB_CUDA(cudaGetDevice(&dev));
    FYB_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

// Device status word shared by all kernels with bounded waits (one int per device, zero = ok).
int* status_ptr();

// Debug builds (FYB_BOUNDS_CHECK): hand the status word to the bounds checks of each translation unit that has them
// (no-ops in release builds).
void bind_bounds_gemm(int* status);
void bind_bounds_elementwise(int* status);
void bind_bounds_comm(int* status);

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// Scoped NVTX range around a native op's host call (header-only NVTX 3: visible to an attached profiler such as
// Nsight Systems, a few nanoseconds otherwise; host-side only, so legal during CUDA graph capture).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};
#define FYB_RANGE(name) ::fyb::NvtxRange fyb_nvtx_range_(name)

// FYB_DEBUG_SYNC=1: synchronise the stream after every native launch (outside graph capture), so that an
// asynchronous kernel error is reported by the op that caused it instead of a later, unrelated call.
inline bool debug_sync() {
  static const bool on = [] {
    const char* e = std::getenv("FYB_DEBUG_SYNC");
    return e != nullptr && e[0] == '1';
  }();
  return on;
}

inline void check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && debug_sync()) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(cur_stream(), &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone)
      e = cudaStreamSynchronize(cur_stream());
  }
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace fyb
