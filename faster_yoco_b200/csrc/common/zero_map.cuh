// ZeRO owner map shared by the optimizer, exchange and owner-scatter GEMM kernels.
//
// The flat parameter / gradient buffer holds world * seg elements. Two layouts:
//   contiguous (chunk == 0): rank r owns the segment [r * seg, (r + 1) * seg);
//   block-cyclic (chunk > 0): the buffer is cut into chunks of `chunk` elements dealt to the ranks in turn, so rank r
//     owns chunks r, r + world, r + 2 world, ... and every large weight is spread over all owners (an exchange that
//     follows the backward pass layer by layer then loads every NVLink port at once instead of one owner's).
// An owner's optimizer state is compact: its c-th owned element has "local" index c in [0, seg).
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

#include "bounds.cuh"

namespace fyb {

struct ZeroMap {
  int64_t chunk;   // 0: contiguous segments
  int world, rank;
};

// Flat index of this owner's local element c, RELATIVE to the base the kernel was given: the segment base
// (contiguous layout) or the start of the flat buffer (block-cyclic).
__host__ __device__ __forceinline__ int64_t zero_flat(const ZeroMap& z, int64_t c) {
  if (z.chunk == 0) return c;
  const int64_t b = c / z.chunk;
  return (b * z.world + z.rank) * z.chunk + (c - b * z.chunk);
}

// Owner of flat element x.
__host__ __device__ __forceinline__ int zero_owner(int64_t chunk, int world, int64_t seg, int64_t x) {
  return chunk == 0 ? static_cast<int>(x / seg) : static_cast<int>((x / chunk) % world);
}

// Local (owned-state) index of flat element x inside its owner's segment.
__host__ __device__ __forceinline__ int64_t zero_local(int64_t chunk, int world, int64_t seg, int64_t x) {
  if (chunk == 0) return x - (x / seg) * seg;
  const int64_t span = chunk * world;
  return (x / span) * chunk + x % chunk;
}

// Owner scatter (a gradient producer fused with the ZeRO reduce-scatter): a weight's gradient slot starts at flat
// index x0 of the gradient buffer; instead of storing element x locally, the producer stores it where its owner o
// sums it: this rank's own buffer when o == rank, else owner o's staging buffer, slot `rank`, at the element's local
// index (bases[o] + rank * seg + local(x)), over NVLink. Every 8-element vector lies inside one segment / chunk
// (seg, chunk, x0 and the row length multiples of 8), so one owner lookup per vector.
struct OwnerScatter {
  const unsigned long long* bases;   // [world] staging buffer of every rank (peer pointers)
  __nv_bfloat16* own;                // this rank's flat gradient buffer
  int64_t x0, seg, chunk;
  int rank, world;
};

// (nullptr when a debug build's bounds check fails: the caller skips the store)
__host__ __device__ __forceinline__ __nv_bfloat16* owner_dst(const OwnerScatter& s, int64_t x) {
  if (!FYB_IN_BOUNDS(x, static_cast<int64_t>(s.world) * s.seg, 520)) return nullptr;
  const int o = zero_owner(s.chunk, s.world, s.seg, x);
  if (o == s.rank) return s.own + x;
  return reinterpret_cast<__nv_bfloat16*>(s.bases[o]) +
         (static_cast<int64_t>(s.rank) * s.seg + zero_local(s.chunk, s.world, s.seg, x));
}

}  // namespace fyb
