// NVLink peer-memory collectives for ZeRO data parallelism (one process per GPU, buffers shared with CUDA IPC).
//
// Reference: the copy-engine reduce-to-owner (yoco/models/decoder/ce_reduce.py: IPC peer mappings,
// cudaMemcpyAsync pushes into per-owner staging slots, a 1-element NCCL all-reduce as barrier, then the Triton
// _sum_slots FP32 rank-order sum x 1/world -> bf16) and the in-place BF16 parameter all-gather
// (yoco/tasks/zero1_fast.py:224-226). Here the SMs do the transfers themselves from inside the kernels that consume
// them, with no staging copy:
//
//  * flag_barrier     : epoch-tagged all-to-all flags (st.release.sys to every peer, bounded ld.acquire.sys spin)
//  * reduce_owner     : the owner reads every rank's bf16 gradient slice over NVLink in rank order, sums in FP32,
//                       scales by 1/world, writes bf16 in place and emits per-CTA partial sums of squares (the
//                       grad-norm partial) -- the reduce-scatter fused with the norm
//  * gather_segments  : pulls a list of (offset, length, owner) ranges of the flat parameter buffer from their
//                       owners (the all-gather, per layer so it can run ahead of the forward pass)
//  * allreduce_small  : a few fp32 values summed in rank order through peer slots (loss, sample size, norm)
//
// Every spin is bounded (FYB_WAIT_NS); a timeout records a status word and the kernel returns.
#include <ATen/ATen.h>

#include <cstring>
#include <vector>

#include "common/host.h"
#include "common/ptx.cuh"
#include "common/zero_map.cuh"

namespace fyb {
namespace {

constexpr int kMaxWorld = 8;

struct PeerPtrs {
  const void* p[kMaxWorld];
};

__device__ __forceinline__ void st_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// flags layout on every rank: [slots][kMaxWorld] uint32; rank r writes epoch into flags_q[slot][r] on every peer q.
// The epoch of a slot is a per-rank device counter incremented by the barrier itself, so a captured CUDA graph
// replays with fresh epochs (every rank runs the same barrier sequence, so the counters agree).
__global__ void flag_barrier_kernel(PeerPtrs peer_flags, uint32_t* my_flags, uint32_t* counters, int rank, int world,
                                    int slot, int* status) {
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) {
    s_epoch = counters[slot] + 1u;
    counters[slot] = s_epoch;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  if (threadIdx.x < world) {
    __threadfence_system();
    uint32_t* f = reinterpret_cast<uint32_t*>(const_cast<void*>(peer_flags.p[threadIdx.x])) + slot * kMaxWorld + rank;
    st_release_sys(f, epoch);
  }
  __syncthreads();
  if (threadIdx.x < world) {
    const uint32_t* f = my_flags + slot * kMaxWorld + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    uint32_t it = 0;
    while (static_cast<int32_t>(ld_acquire_sys(f) - epoch) < 0) {
      if ((++it & 255u) == 0u && globaltimer_ns() - t0 > FYB_WAIT_NS) {
        record_status(status, kPeerTimeout, 200 + slot);
        break;
      }
    }
  }
  __syncthreads();
  __threadfence_system();
}

// owner-side reduction of its n owned elements: out = bf16(sum_r g_r / world) in rank order; per-CTA partial sums of
// squares of the bf16 result in part[blockIdx.x]. Local element i is flat element base + zero_flat(z, i) (the segment
// [base, base + n) in the contiguous layout).
__global__ void reduce_owner_kernel(PeerPtrs grads, __nv_bfloat16* out, int64_t base, int64_t n, int world,
                                    float inv_world, float* part, const ZeroMap z) {
  float ss = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 8;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < n; i += stride) {
    if (i + 8 <= n) {
      const int64_t x = base + zero_flat(z, i);
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      uint4 u[kMaxWorld];
#pragma unroll
      for (int r = 0; r < kMaxWorld; ++r)
        if (r < world) u[r] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(grads.p[r]) + x);
#pragma unroll
      for (int r = 0; r < kMaxWorld; ++r) {
        if (r < world) {
          const uint32_t w[4] = {u[r].x, u[r].y, u[r].z, u[r].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = unpack_bf16(w[k]);
            acc[2 * k] += f.x;
            acc[2 * k + 1] += f.y;
          }
        }
      }
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float a = bf16_round(acc[2 * k] * inv_world), b = bf16_round(acc[2 * k + 1] * inv_world);
        ss += a * a + b * b;
        o[k] = pack_bf16(a, b);
      }
      *reinterpret_cast<uint4*>(out + x) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
      for (int64_t j = i; j < n; ++j) {
        const int64_t xj = base + zero_flat(z, j);
        float acc = 0.f;
        for (int r = 0; r < world; ++r) acc += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(grads.p[r])[xj]);
        const float a = bf16_round(acc * inv_world);
        ss += a * a;
        out[xj] = __float2bfloat16_rn(a);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    part[blockIdx.x] = t;
  }
}

__global__ void sum_partials_kernel(const float* __restrict__ part, int P, float* __restrict__ out) {
  __shared__ float red[1024];
  float s = 0.f;
  for (int i = threadIdx.x; i < P; i += blockDim.x) s += part[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[0] = red[0];
}

// segments: [nseg][3] int64 = (element offset, element count, owner rank); each CTA walks segments in 16-byte
// vectors (offsets and counts are multiples of 8 elements by construction of the flat layout)
__global__ void gather_segments_kernel(PeerPtrs src, __nv_bfloat16* dst, const int64_t* __restrict__ segs, int nseg,
                                       int rank) {
  for (int s = 0; s < nseg; ++s) {
    const int64_t off = segs[3 * s], cnt = segs[3 * s + 1];
    const int owner = static_cast<int>(segs[3 * s + 2]);
    if (owner == rank) continue;
    const uint4* sp = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(src.p[owner]) + off);
    uint4* dp = reinterpret_cast<uint4*>(dst + off);
    const int64_t nv = cnt / 8;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    // 4 independent 16-byte NVLink loads in flight per thread (remote latency is ~microseconds)
    int64_t i = tid;
    for (; i + 3 * nthr < nv; i += 4 * nthr) {
      const uint4 a = sp[i], b = sp[i + nthr], c = sp[i + 2 * nthr], d = sp[i + 3 * nthr];
      dp[i] = a;
      dp[i + nthr] = b;
      dp[i + 2 * nthr] = c;
      dp[i + 3 * nthr] = d;
    }
    for (; i < nv; i += nthr) dp[i] = sp[i];
    const int64_t tail0 = nv * 8;
    if (blockIdx.x == 0)
      for (int64_t j = tail0 + threadIdx.x; j < cnt; j += blockDim.x)
        dst[off + j] = reinterpret_cast<const __nv_bfloat16*>(src.p[owner])[off + j];
  }
}

// push form of the all-gather: this rank's range [off, off+n) of its flat buffer is stored into the same range of
// every peer's buffer (remote stores are posted writes: no round trip per access, unlike remote loads)
// (n owned elements; local element c is flat element off + zero_flat(z, c))
__global__ void push_range_kernel(const __nv_bfloat16* __restrict__ src, PeerPtrs dst, int64_t off, int64_t n,
                                  int world, int rank, int64_t chunk) {
  const ZeroMap z{chunk, world, rank};
  const int64_t nv = n / 8;
  const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nv; i += nthr) {
    const int64_t x = off + zero_flat(z, i * 8);
    const uint4 v = *reinterpret_cast<const uint4*>(src + x);
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < world && q != rank)
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(dst.p[q])) + x) = v;
  }
  if (blockIdx.x == 0)
    for (int64_t j = nv * 8 + threadIdx.x; j < n; j += blockDim.x) {
      const int64_t x = off + zero_flat(z, j);
      for (int q = 0; q < world; ++q)
        if (q != rank) reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(dst.p[q]))[x] = src[x];
    }
  __threadfence_system();   // the barrier that follows publishes these remote stores
}

// Push this rank's pieces of one bucket (ranges [n][2] = (offset, count)) into every peer's flat buffer, then each CTA
// makes its stores visible system-wide and adds 1 to the bucket's arrival counter on every peer.
__global__ void push_bucket_kernel(const __nv_bfloat16* __restrict__ src, PeerPtrs dst, PeerPtrs arrive,
                                   const int64_t* __restrict__ ranges, int nranges, int bucket, int world, int rank) {
  const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int rg = 0; rg < nranges; ++rg) {
    const int64_t off = ranges[2 * rg], n = ranges[2 * rg + 1];
    const uint4* sp = reinterpret_cast<const uint4*>(src + off);
    const int64_t nv = n / 8;
    for (int64_t i = tid; i < nv; i += nthr) {
      const uint4 v = sp[i];
#pragma unroll
      for (int q = 0; q < kMaxWorld; ++q)
        if (q < world && q != rank)
          reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(dst.p[q])) + off)[i] = v;
    }
    for (int64_t j = nv * 8 + tid; j < n; j += nthr)
      for (int q = 0; q < world; ++q)
        if (q != rank) reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(dst.p[q]))[off + j] = src[off + j];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world && threadIdx.x != rank) {
    uint32_t* c = reinterpret_cast<uint32_t*>(const_cast<void*>(arrive.p[threadIdx.x])) + bucket;
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(c), "r"(1u) : "memory");
  }
}

// Gradient push for the owner-side reduction: for every piece (offset, count, owner q != rank) of this bucket, this
// rank's gradient values are stored into owner q's staging buffer, slot `rank` (staging_q[rank * seg + offset -
// q * seg]); then each CTA fences and adds 1 to the bucket's arrival counter on every peer.
__global__ void push_grads_kernel(const __nv_bfloat16* __restrict__ grad, PeerPtrs staging, PeerPtrs arrive,
                                  const int64_t* __restrict__ pieces, int npieces, int bucket, int world, int rank,
                                  int64_t seg, int64_t chunk) {
  const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int pc = 0; pc < npieces; ++pc) {
    const int64_t off = pieces[3 * pc], n = pieces[3 * pc + 1];
    const int q = static_cast<int>(pieces[3 * pc + 2]);
    if (!FYB_IN_BOUNDS(q, world, 510) || !FYB_IN_BOUNDS(off + n - 1, static_cast<int64_t>(world) * seg, 511)) continue;
    // a piece lies inside one chunk (one owner segment in the contiguous layout): its local positions are contiguous
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(staging.p[q])) +
                         static_cast<int64_t>(rank) * seg + zero_local(chunk, world, seg, off);
    const uint4* sp = reinterpret_cast<const uint4*>(grad + off);
    const int64_t nv = n / 8;
    for (int64_t i = tid; i < nv; i += nthr) reinterpret_cast<uint4*>(dst)[i] = sp[i];
    for (int64_t j = nv * 8 + tid; j < n; j += nthr) dst[j] = grad[off + j];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world && threadIdx.x != rank) {
    uint32_t* c = reinterpret_cast<uint32_t*>(const_cast<void*>(arrive.p[threadIdx.x])) + bucket;
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(c), "r"(1u) : "memory");
  }
}

// Owner-side sum from local memory: for each owned range, out = bf16(sum over ranks in rank order / world), where
// rank `rank`'s own values come from its gradient buffer and the others' from the staging slots. Per-CTA partial
// sums of squares of the result in part[blockIdx.x].
// W: the largest world this instance serves (2, 4 or 8). Each thread handles 8 / W groups of 8 elements per step
// and issues all sources' 16-byte loads of them before the first add, so 8 loads (128 bytes) are in flight per thread
// whatever the world (one group per step with 4 ranks measured 0.39 of HBM: latency-bound), in registers sized for W
// sources rather than the maximum of 8; three CTAs of 256 threads fit on an SM.
template <int W>
__global__ void __launch_bounds__(256, 3) reduce_staged_kernel(__nv_bfloat16* __restrict__ grad, const __nv_bfloat16* __restrict__ staging,
                                     const int64_t* __restrict__ ranges, int nranges, int world, int rank,
                                     int64_t seg, float inv_world, float* __restrict__ part, int64_t chunk) {
  constexpr int kStagedGroups = 8 / W;
  float ss = 0.f;
  const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int rg = 0; rg < nranges; ++rg) {
    const int64_t off = ranges[2 * rg], n = ranges[2 * rg + 1];
    if (!FYB_IN_BOUNDS(off, static_cast<int64_t>(world) * seg, 512) ||
        !FYB_IN_BOUNDS(off + n - 1, static_cast<int64_t>(world) * seg, 512))
      continue;
    const int64_t loc = zero_local(chunk, world, seg, off);        // position inside the owner's segment
    for (int64_t i = tid * 8; i < n; i += nthr * 8 * kStagedGroups) {
      uint4 u[kStagedGroups][W];
#pragma unroll
      for (int q = 0; q < kStagedGroups; ++q) {
        const int64_t j = i + q * nthr * 8;
        if (j + 8 <= n) {
#pragma unroll
          for (int r = 0; r < W; ++r) {
            if (r < world) {
              const __nv_bfloat16* src = r == rank ? grad + off : staging + static_cast<int64_t>(r) * seg + loc;
              u[q][r] = *reinterpret_cast<const uint4*>(src + j);
            }
          }
        }
      }
#pragma unroll
      for (int q = 0; q < kStagedGroups; ++q) {
        const int64_t j = i + q * nthr * 8;
        if (j + 8 <= n) {
          float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
          for (int r = 0; r < W; ++r) {
            if (r < world) {
              const uint32_t w[4] = {u[q][r].x, u[q][r].y, u[q][r].z, u[q][r].w};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float2 f = unpack_bf16(w[k]);
                acc[2 * k] += f.x;
                acc[2 * k + 1] += f.y;
              }
            }
          }
          uint32_t o[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float a = bf16_round(acc[2 * k] * inv_world), b = bf16_round(acc[2 * k + 1] * inv_world);
            ss += a * a + b * b;
            o[k] = pack_bf16(a, b);
          }
          *reinterpret_cast<uint4*>(grad + off + j) = make_uint4(o[0], o[1], o[2], o[3]);
        } else if (j < n) {
          for (int64_t e = j; e < n; ++e) {
            float acc = 0.f;
            for (int r = 0; r < world; ++r)
              acc += __bfloat162float(r == rank ? grad[off + e] : staging[static_cast<int64_t>(r) * seg + loc + e]);
            const float a = bf16_round(acc * inv_world);
            ss += a * a;
            grad[off + e] = __float2bfloat16_rn(a);
          }
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    part[blockIdx.x] = t;
  }
}

// Owner-side sum of a whole owned segment from local memory (GEMM-fused reduce-scatter): local element c in [0, n)
// is flat element base + zero_flat(z, c); this rank's own value is read from its gradient buffer there, rank r's from
// staging slot r (staging[r * seg + c]); out = bf16(sum in rank order / world) is written back to the gradient
// buffer. Same arithmetic as reduce_owner_kernel. Per-CTA partial sums of squares in part[blockIdx.x].
__global__ void reduce_compact_kernel(__nv_bfloat16* __restrict__ grad, const __nv_bfloat16* __restrict__ staging,
                                      int64_t base, int64_t n, int64_t seg, float inv_world, float* __restrict__ part,
                                      const ZeroMap z) {
  float ss = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 8;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < n; i += stride) {
    if (i + 8 <= n) {
      const int64_t x = base + zero_flat(z, i);
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int r = 0; r < kMaxWorld; ++r) {
        if (r < z.world) {
          const __nv_bfloat16* src = r == z.rank ? grad + x : staging + static_cast<int64_t>(r) * seg + i;
          const uint4 u = *reinterpret_cast<const uint4*>(src);
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = unpack_bf16(w[k]);
            acc[2 * k] += f.x;
            acc[2 * k + 1] += f.y;
          }
        }
      }
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float a = bf16_round(acc[2 * k] * inv_world), b = bf16_round(acc[2 * k + 1] * inv_world);
        ss += a * a + b * b;
        o[k] = pack_bf16(a, b);
      }
      *reinterpret_cast<uint4*>(grad + x) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
      for (int64_t j = i; j < n; ++j) {
        const int64_t xj = base + zero_flat(z, j);
        float acc = 0.f;
        for (int r = 0; r < z.world; ++r)
          acc += __bfloat162float(r == z.rank ? grad[xj] : staging[static_cast<int64_t>(r) * seg + j]);
        const float a = bf16_round(acc * inv_world);
        ss += a * a;
        grad[xj] = __float2bfloat16_rn(a);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    part[blockIdx.x] = t;
  }
}

// Clear the staging slots of every other rank over the listed local ranges ([n][2] = (local offset, count)) of this
// owner's segment: the regions peers fill sparsely (the embedding rows of the tokens in their batch) must read zero
// where nothing was stored.
__global__ void zero_staged_kernel(__nv_bfloat16* __restrict__ staging, const int64_t* __restrict__ ranges,
                                   int nranges, int world, int rank, int64_t seg) {
  const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int rg = 0; rg < nranges; ++rg) {
    const int64_t lo = ranges[2 * rg], n = ranges[2 * rg + 1];
    if (!FYB_IN_BOUNDS(lo, seg, 513) || !FYB_IN_BOUNDS(lo + n - 1, seg, 513)) continue;
    for (int r = 0; r < world; ++r) {
      if (r == rank) continue;
      __nv_bfloat16* p = staging + static_cast<int64_t>(r) * seg + lo;
      const int64_t nv = n / 8;
      for (int64_t i = tid; i < nv; i += nthr) reinterpret_cast<uint4*>(p)[i] = make_uint4(0, 0, 0, 0);
      for (int64_t j = nv * 8 + tid; j < n; j += nthr) p[j] = __float2bfloat16_rn(0.f);
    }
  }
}

// Compute-stream wait until bucket b's pushes of the current update have all arrived: expected[b] += increment, then
// spin (bounded) until arrive[b] >= expected[b]. The expectation is device-resident, so graph replays stay correct.
__global__ void wait_arrivals_kernel(const uint32_t* __restrict__ arrive, uint32_t* __restrict__ expected, int bucket,
                                     uint32_t increment, int* status) {
  if (threadIdx.x != 0) return;
  const uint32_t want = expected[bucket] + increment;
  expected[bucket] = want;
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (static_cast<int32_t>(ld_acquire_sys(arrive + bucket) - want) < 0) {
    if ((++it & 255u) == 0u && globaltimer_ns() - t0 > FYB_WAIT_NS) {
      record_status(status, kPeerTimeout, 300 + bucket);
      break;
    }
  }
  __threadfence_system();
}

// Copy-engine transport: after the stream's peer copies (cudaMemcpyAsync, executed by the copy engines, so no SM
// time is taken from the compute stream), one thread publishes their completion by adding 1 to a counter in the
// destination GPU's memory. Stream order makes the copies complete before this kernel starts; the release add
// orders them before the counter update for a reader that acquires the counter.
__global__ void signal_peer_kernel(uint32_t* counter) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(counter), "r"(1u) : "memory");
  }
}

// each rank writes its k values into slot [rank] of every peer's mailbox, then (after a flag barrier) sums the
// world slots of its own mailbox in rank order
__global__ void mailbox_put_kernel(PeerPtrs boxes, const float* __restrict__ vals, int k, int rank, int world,
                                   const uint32_t* __restrict__ counter) {
  const int slot_base = static_cast<int>(counter[0] & 1u) * kMaxWorld * 32;
  for (int q = 0; q < world; ++q) {
    float* box = reinterpret_cast<float*>(const_cast<void*>(boxes.p[q])) + slot_base + rank * 32;
    for (int i = threadIdx.x; i < k; i += blockDim.x) box[i] = vals[i];
  }
}

__global__ void mailbox_sum_kernel(const float* __restrict__ box, float* __restrict__ out, int k, int world,
                                   uint32_t* __restrict__ counter) {
  const int slot_base = static_cast<int>(counter[0] & 1u) * kMaxWorld * 32;
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < world; ++r) s += box[slot_base + r * 32 + i];
    out[i] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) counter[0] += 1u;
}

PeerPtrs to_ptrs(const std::vector<int64_t>& v) {
  FYB_CHECK(static_cast<int>(v.size()) <= kMaxWorld, "at most 8 ranks");
  PeerPtrs p{};
  for (size_t i = 0; i < v.size(); ++i) p.p[i] = reinterpret_cast<const void*>(v[i]);
  return p;
}

}  // namespace

// ---------------------------------------------------------------------------------------------------- IPC buffers

// cudaMalloc'd buffer (its own allocation, so its IPC handle maps exactly this range) + the handle bytes
std::vector<at::Tensor> ipc_alloc(int64_t nbytes) {
  ensure_context();
  void* p = nullptr;
  FYB_CUDA(cudaMalloc(&p, static_cast<size_t>(nbytes)));
  FYB_CUDA(cudaMemset(p, 0, static_cast<size_t>(nbytes)));
  cudaIpcMemHandle_t h;
  FYB_CUDA(cudaIpcGetMemHandle(&h, p));
  int dev;
  FYB_CUDA(cudaGetDevice(&dev));
  auto t = at::from_blob(
      p, {nbytes}, [](void* q) { cudaFree(q); }, at::TensorOptions().dtype(at::kByte).device(at::kCUDA, dev));
  auto hb = at::empty({static_cast<int64_t>(sizeof(h))}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(hb.data_ptr(), &h, sizeof(h));
  return {t, hb};
}

int64_t ipc_open(const at::Tensor& handle_bytes) {
  ensure_context();
  FYB_CHECK(handle_bytes.numel() == static_cast<int64_t>(sizeof(cudaIpcMemHandle_t)), "ipc_open: bad handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle_bytes.data_ptr(), sizeof(h));
  void* p = nullptr;
  FYB_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) { FYB_CUDA(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

// ------------------------------------------------------------------------------------------------------- kernels

void flag_barrier(const std::vector<int64_t>& peer_flags, const at::Tensor& my_flags, const at::Tensor& counters,
                  int64_t rank, int64_t slot) {
  FYB_RANGE("fyb::flag_barrier");
  const int world = static_cast<int>(peer_flags.size());
  FYB_CHECK(counters.is_cuda() && counters.numel() > slot, "flag_barrier: counters");
  flag_barrier_kernel<<<1, 32, 0, cur_stream()>>>(to_ptrs(peer_flags), reinterpret_cast<uint32_t*>(my_flags.data_ptr()),
                                                  reinterpret_cast<uint32_t*>(counters.data_ptr()),
                                                  static_cast<int>(rank), world, static_cast<int>(slot), status_ptr());
  check_launch("flag_barrier");
}

int reduce_ctas() { return std::min(num_sms() * 2, 1024); }

// reduce [base, base+n) of the flat gradient buffers into out (this rank's buffer) and sq[0] = sum of squares
// (chunk > 0: block-cyclic layout, base must be 0 and local element c is flat element zero_flat(c))
void reduce_owner(const std::vector<int64_t>& peer_grads, at::Tensor& out, int64_t base, int64_t n, at::Tensor& part,
                  at::Tensor& sq, int64_t chunk, int64_t rank) {
  FYB_RANGE("fyb::reduce_owner");
  const int world = static_cast<int>(peer_grads.size());
  FYB_CHECK(base % 8 == 0, "reduce_owner: segment base must be a multiple of 8 elements");
  FYB_CHECK(chunk == 0 || (chunk % 8 == 0 && base == 0 && rank >= 0 && rank < world),
            "reduce_owner: block-cyclic layout needs chunk % 8 == 0, base 0 and this rank");
  const int P = static_cast<int>(part.numel());
  FYB_CHECK(P >= 1 && P <= 1024, "reduce_owner: 1..1024 partials");
  reduce_owner_kernel<<<P, 256, 0, cur_stream()>>>(to_ptrs(peer_grads),
                                                   reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), base, n, world,
                                                   1.0f / static_cast<float>(world), part.data_ptr<float>(),
                                                   ZeroMap{chunk, world, static_cast<int>(rank)});
  check_launch("reduce_owner");
  sum_partials_kernel<<<1, 1024, 0, cur_stream()>>>(part.data_ptr<float>(), P, sq.data_ptr<float>());
  check_launch("reduce_owner_sum");
}

// reduce the listed owned ranges; part (>= ctas floats) receives the per-CTA sums of squares
void sum_partials(const at::Tensor& part, at::Tensor& out) {
  sum_partials_kernel<<<1, 1024, 0, cur_stream()>>>(part.data_ptr<float>(), static_cast<int>(part.numel()),
                                                   out.data_ptr<float>());
  check_launch("sum_partials");
}

void gather_segments(const std::vector<int64_t>& peer_params, at::Tensor& dst, const at::Tensor& segs, int64_t rank,
                     int64_t ctas) {
  FYB_RANGE("fyb::gather_segments");
  FYB_CHECK(segs.is_cuda() && segs.scalar_type() == at::kLong && segs.dim() == 2 && segs.size(1) == 3,
            "gather_segments: segs must be a device int64 [n, 3]");
  if (segs.size(0) == 0) return;
  gather_segments_kernel<<<static_cast<int>(ctas), 512, 0, cur_stream()>>>(
      to_ptrs(peer_params), reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()), segs.data_ptr<int64_t>(),
      static_cast<int>(segs.size(0)), static_cast<int>(rank));
  check_launch("gather_segments");
}

void push_range(const at::Tensor& src, const std::vector<int64_t>& peer_dst, int64_t off, int64_t n, int64_t rank,
                int64_t ctas, int64_t chunk) {
  FYB_RANGE("fyb::push_range");
  const int world = static_cast<int>(peer_dst.size());
  FYB_CHECK(off % 8 == 0, "push_range: offset must be a multiple of 8 elements");
  FYB_CHECK(chunk == 0 || (chunk % 8 == 0 && off == 0), "push_range: block-cyclic layout needs chunk % 8 == 0, off 0");
  if (n <= 0) return;
  push_range_kernel<<<static_cast<int>(ctas), 512, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), to_ptrs(peer_dst), off, n, world,
      static_cast<int>(rank), chunk);
  check_launch("push_range");
}

void push_bucket(const at::Tensor& src, const std::vector<int64_t>& peer_dst, const std::vector<int64_t>& peer_arrive,
                 const at::Tensor& ranges, int64_t bucket, int64_t rank, int64_t ctas) {
  FYB_RANGE("fyb::push_bucket");
  const int world = static_cast<int>(peer_dst.size());
  FYB_CHECK(ranges.is_cuda() && ranges.scalar_type() == at::kLong && ranges.dim() == 2 && ranges.size(1) == 2,
            "push_bucket: ranges must be a device int64 [n, 2]");
  push_bucket_kernel<<<static_cast<int>(ctas), 512, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), to_ptrs(peer_dst), to_ptrs(peer_arrive),
      ranges.data_ptr<int64_t>(), static_cast<int>(ranges.size(0)), static_cast<int>(bucket), world,
      static_cast<int>(rank));
  check_launch("push_bucket");
}

void push_grads(const at::Tensor& grad, const std::vector<int64_t>& peer_staging,
                const std::vector<int64_t>& peer_arrive, const at::Tensor& pieces, int64_t bucket, int64_t rank,
                int64_t seg, int64_t ctas, int64_t chunk) {
  FYB_RANGE("fyb::push_grads");
  const int world = static_cast<int>(peer_staging.size());
  FYB_CHECK(pieces.is_cuda() && pieces.scalar_type() == at::kLong && pieces.dim() == 2 && pieces.size(1) == 3,
            "push_grads: pieces must be a device int64 [n, 3]");
  push_grads_kernel<<<static_cast<int>(ctas), 512, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(grad.data_ptr()), to_ptrs(peer_staging), to_ptrs(peer_arrive),
      pieces.data_ptr<int64_t>(), static_cast<int>(pieces.size(0)), static_cast<int>(bucket), world,
      static_cast<int>(rank), seg, chunk);
  check_launch("push_grads");
}

void reduce_staged(at::Tensor& grad, const at::Tensor& staging, const at::Tensor& ranges, int64_t world, int64_t rank,
                   int64_t seg, at::Tensor& part, int64_t ctas, int64_t chunk) {
  FYB_RANGE("fyb::reduce_staged");
  // ranges: flat (offset, count) pieces of this owner's elements, offsets multiples of 8 elements (16-byte loads);
  // every range of the ZeRO bucket tables is (parameters start 64-element aligned, owner cuts are multiples of 64)
  FYB_CHECK(ranges.is_cuda() && ranges.scalar_type() == at::kLong && ranges.dim() == 2 && ranges.size(1) == 2,
            "reduce_staged: ranges must be a device int64 [n, 2]");
  FYB_CHECK(grad.scalar_type() == at::kBFloat16 && staging.scalar_type() == at::kBFloat16 &&
                grad.numel() == world * seg && staging.numel() == world * seg && seg % 8 == 0,
            "reduce_staged: bf16 gradient buffer and staging of world x seg elements");
  FYB_CHECK(reinterpret_cast<uintptr_t>(grad.data_ptr()) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(staging.data_ptr()) % 16 == 0,
            "reduce_staged: 16-byte aligned buffers");
  FYB_CHECK(ctas >= 1 && part.numel() >= ctas, "reduce_staged: partials buffer too small");
  if (ranges.size(0) == 0) {
    part.zero_();
    return;
  }
  FYB_CHECK(world >= 1 && world <= kMaxWorld && rank >= 0 && rank < world, "reduce_staged: 1..8 ranks");
  auto kern = world <= 2 ? reduce_staged_kernel<2> : (world <= 4 ? reduce_staged_kernel<4> : reduce_staged_kernel<8>);
  kern<<<static_cast<int>(ctas), 256, 0, cur_stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(staging.data_ptr()),
      ranges.data_ptr<int64_t>(), static_cast<int>(ranges.size(0)), static_cast<int>(world), static_cast<int>(rank),
      seg, 1.0f / static_cast<float>(world), part.data_ptr<float>(), chunk);
  check_launch("reduce_staged");
}

void zero_staged(at::Tensor& staging, const at::Tensor& ranges, int64_t world, int64_t rank, int64_t seg,
                 int64_t ctas) {
  FYB_RANGE("fyb::zero_staged");
  FYB_CHECK(ranges.is_cuda() && ranges.scalar_type() == at::kLong && ranges.dim() == 2 && ranges.size(1) == 2,
            "zero_staged: ranges must be a device int64 [n, 2]");
  FYB_CHECK(staging.numel() == world * seg && seg % 8 == 0, "zero_staged: staging of world x seg elements");
  if (ranges.size(0) == 0) return;
  zero_staged_kernel<<<static_cast<int>(ctas), 256, 0, cur_stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(staging.data_ptr()), ranges.data_ptr<int64_t>(),
      static_cast<int>(ranges.size(0)), static_cast<int>(world), static_cast<int>(rank), seg);
  check_launch("zero_staged");
}

// The owner's n local elements summed from its gradient buffer (own values) and the staging slots (peers'), written
// back in place; part (>= ctas floats) receives the per-CTA sums of squares.
void reduce_compact(at::Tensor& grad, const at::Tensor& staging, int64_t n, int64_t world, int64_t rank, int64_t seg,
                    int64_t chunk, at::Tensor& part, int64_t ctas) {
  FYB_RANGE("fyb::reduce_compact");
  FYB_CHECK(world >= 1 && world <= kMaxWorld && rank >= 0 && rank < world, "reduce_compact: 1..8 ranks");
  FYB_CHECK(seg % 8 == 0 && chunk % 8 == 0 && n <= seg, "reduce_compact: seg / chunk multiples of 8, n <= seg");
  FYB_CHECK(grad.numel() == world * seg && staging.numel() == world * seg,
            "reduce_compact: gradient and staging buffers of world x seg elements");
  FYB_CHECK(part.numel() >= ctas && ctas >= 1, "reduce_compact: partials buffer too small");
  if (n == 0) {
    part.zero_();
    return;
  }
  const int64_t base = chunk == 0 ? rank * seg : 0;
  reduce_compact_kernel<<<static_cast<int>(ctas), 256, 0, cur_stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(staging.data_ptr()),
      base, n, seg, 1.0f / static_cast<float>(world), part.data_ptr<float>(),
      ZeroMap{chunk, static_cast<int>(world), static_cast<int>(rank)});
  check_launch("reduce_compact");
}

void peer_copy(int64_t dst, int64_t src, int64_t nbytes) {
  FYB_RANGE("fyb::peer_copy");
  // one copy-engine transfer per call (the batched copy entry points are not used)
  if (nbytes <= 0) return;
  FYB_CUDA(cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src),
                           static_cast<size_t>(nbytes), cudaMemcpyDeviceToDevice, cur_stream()));
}

void signal_peer(int64_t counter_base, int64_t index) {
  signal_peer_kernel<<<1, 32, 0, cur_stream()>>>(reinterpret_cast<uint32_t*>(counter_base) + index);
  check_launch("signal_peer");
}

void wait_arrivals(const at::Tensor& arrive, at::Tensor& expected, int64_t bucket, int64_t increment) {
  FYB_RANGE("fyb::wait_arrivals");
  wait_arrivals_kernel<<<1, 32, 0, cur_stream()>>>(reinterpret_cast<const uint32_t*>(arrive.data_ptr()),
                                                   reinterpret_cast<uint32_t*>(expected.data_ptr()),
                                                   static_cast<int>(bucket), static_cast<uint32_t>(increment),
                                                   status_ptr());
  check_launch("wait_arrivals");
}

void mailbox_put(const std::vector<int64_t>& peer_boxes, const at::Tensor& vals, int64_t rank,
                 const at::Tensor& counter) {
  FYB_RANGE("fyb::mailbox_put");
  const int world = static_cast<int>(peer_boxes.size());
  FYB_CHECK(vals.numel() <= 32 && vals.scalar_type() == at::kFloat, "mailbox_put: at most 32 fp32 values");
  mailbox_put_kernel<<<1, 32, 0, cur_stream()>>>(to_ptrs(peer_boxes), vals.data_ptr<float>(),
                                                 static_cast<int>(vals.numel()), static_cast<int>(rank), world,
                                                 reinterpret_cast<const uint32_t*>(counter.data_ptr()));
  check_launch("mailbox_put");
}

void mailbox_sum(const at::Tensor& box, at::Tensor& out, int64_t world, at::Tensor& counter) {
  FYB_RANGE("fyb::mailbox_sum");
  mailbox_sum_kernel<<<1, 32, 0, cur_stream()>>>(box.data_ptr<float>(), out.data_ptr<float>(),
                                                 static_cast<int>(out.numel()), static_cast<int>(world),
                                                 reinterpret_cast<uint32_t*>(counter.data_ptr()));
  check_launch("mailbox_sum");
}

FYB_BOUNDS_BINDER(bind_bounds_comm)

}  // namespace fyb
