// Allocation-free C entry point of the RMSNorm backward.
//
// This entry point has no counterpart in the reference: it is an addition of this library for callers that cannot
// allocate device memory themselves, for example a plugin or custom-call interface of another runtime that owns all
// device memory and hands the kernel only its input and output buffers, or a latency-critical path where
// cudaMalloc / cudaFree (which can synchronize the device) are not allowed.
//
// fyb_rms_norm_bwd_noalloc computes the same result as the library's regular RMSNorm backward
// (dx = rstd * (dy*w - n * mean(dy*w * n)), dw = sum over rows of dy * bf16(x * rstd)), with every buffer passed
// in by the caller. Its only scratch memory -- the per-block fp32 partial sums of the weight gradient -- is one
// file-scope `static __device__` array of 64 x 8192 floats (2 MiB), which every GPU that loads the library keeps
// until the process exits. Hence the limits:
//   * N (the normalised width) must be a multiple of 8 and at most 8192; larger N is rejected (return code 1).
//   * All calls share that array, and each call leaves its partials in it. The kernel writes every slot it reads
//     in the same call, so nothing needs clearing, but calls that overlap on the GPU (unordered streams, several
//     host threads) race on the array: order them, e.g. by using one stream.
//   * The first call on a device, with that device current, looks up the array's device address
//     (cudaGetSymbolAddress) and caches it; make that first call before any stream capture.
//   * It calls no cudaMalloc, cudaFree or other allocating routine.
//   * A CUDA error that earlier work left pending is not consumed: the call returns code 7 without launching.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// dy, x: bf16 [M, N] row-major; w: bf16 [N] or NULL (then dw must be NULL); rstd: fp32 [M] from the forward;
// dx: bf16 [M, N] output; dw: bf16 [N] output. All pointers 16-byte aligned. Returns 0 on success, else a code
// that fyb_noalloc_strerror describes.
__attribute__((visibility("default"))) int fyb_rms_norm_bwd_noalloc(const void* dy, const void* x, const void* w,
                                                                    const float* rstd, void* dx, void* dw, int64_t M,
                                                                    int64_t N, cudaStream_t stream);

__attribute__((visibility("default"))) const char* fyb_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif
