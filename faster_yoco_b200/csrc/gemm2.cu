// Two-CTA tcgen05 GEMM for sm_100a: C[M,N] = sum_k A(m,k) * B(n,k) (+ R), tiles of 256 x 256 computed by a CTA pair.
//
// The one-CTA kernel (gemm.cu) fills 48 KB of shared memory per 64-wide K slab for each 128 x 256 output tile: the
// whole 256-row B slab goes to every CTA. Here a cluster of two CTAs on one TPC issues tcgen05.mma.cta_group::2 with
// M = 256: CTA r holds rows [128 r, 128 r + 128) of the A tile and rows [128 r, 128 r + 128) of the B tile (its half),
// the tensor cores of the pair exchange the B halves, and each CTA's TMEM receives its 128 rows of the 256 x 256 fp32
// accumulator. Per SM that is 32 KB of operand fill per K slab for the same 128 x 256 output (one third less), which
// is what limited the one-CTA kernel (tensor pipe 63 % active, operand feed from L2).
//
// Roles (6 warps per CTA, both CTAs):
//   warp 0      : TMA producer (one lane): loads this CTA's A rows and B half; the bytes of BOTH CTAs complete on
//                 the leader CTA's (rank 0) full barrier, which only the leader's producer arms with the pair's total
//   warp 1      : TMEM allocation for the pair (cta_group::2, both CTAs); on the leader, one lane issues the MMAs and
//                 commits: stage release to both CTAs' empty barriers, accumulator ready to both CTAs' tfull barriers
//                 (one commit per CTA, addressed through mapa)
//   warps 2..5  : epilogue on each CTA's own TMEM rows; the peer's warps arrive on the leader's tempty barrier
// Loads are plain cp.async.bulk.tensor of this GPU's memory in the .cta_group::2 form; each CTA loads its own tiles.
// Every wait is bounded (2 s) and records a status word; both CTAs always reach the final cluster barrier.
#include <ATen/ATen.h>
#include <c10/util/Optional.h>

#include "common/host.h"
#include "common/ptx.cuh"

namespace fyb {
namespace {

constexpr int kBM = 128;        // rows of A (and of the output) per CTA
constexpr int kBK = 64;
constexpr int kThreads2 = 192;
constexpr int kThreadsG = 320;  // the gather form: + 4 warps that pull the weight rows from their ZeRO owners
constexpr int kGatherThreads = kThreadsG - kThreads2;

// The ZeRO parameter all-gather fused into a forward GEMM (the consumer of the gathered weight). B is a contiguous
// [N, K] weight inside this rank's flat parameter replica (element offset w_off); after the owners' optimizer
// step only the rows this rank owns are current here. Every tile (mb, nb) of the GEMM is computed by one CTA pair,
// and its two CTAs' gather warps pull shares 2 mb and 2 mb + 1 (of 2 num_m) of B's tile column nb -- the elements
// [w_off + 256 nb K, w_off + 256 (nb + 1) K) -- from the owners' replicas into this one, with plain 16-byte loads of
// peer memory, then count the share done on counters[nb] (release). Before loading tile column nb with TMA (from
// this replica only) the producer waits (acquire, bounded) for all 2 num_m shares. The gather warps never wait, so
// the column a producer waits for is always being copied; they run ahead of the MMAs through the CTA's tile list,
// so the NVLink transfer of the next tiles overlaps the math of the current ones.
// Owner of flat element x: (x / chunk) mod world (block-cyclic map) or x / seg (contiguous segments).
struct GatherArgs {
  const int64_t* peers;      // [world] base addresses of every rank's flat replica (this rank's entry unused)
  __nv_bfloat16* local;      // this rank's flat replica
  int64_t w_off;             // element offset of B[0, 0] in the flat buffer
  int64_t seg;               // owner segment length (elements)
  int64_t chunk;             // block-cyclic chunk (elements), 0: contiguous segments
  int* counters;             // [num_n] shares done per tile column, zero at launch
  int world, rank;
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// generic-proxy writes of this thread (or ordered before it) vs. async-proxy (TMA) accesses of global memory
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// bounded wait until *p >= target (status word + abort flag on timeout, like the mbarrier waits)
__device__ __forceinline__ bool wait_count(const int* p, int target, volatile int* abort, int* status, int site) {
  if (ld_acquire_gpu(p) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  for (uint32_t it = 1;; ++it) {
    __nanosleep(32);
    if (ld_acquire_gpu(p) >= target) return true;
    if ((it & 63u) == 0u) {
      if (abort != nullptr && *abort) return false;
      if (globaltimer_ns() - t0 > FYB_WAIT_NS) {
        record_status(status, kPeerTimeout, site);
        if (abort != nullptr) *abort = 1;
        return false;
      }
    }
  }
}

// copy the elements [lo, hi) of the flat buffer that other ranks own from their replicas into this one; called by
// the kGatherThreads gather threads (index gt), 8 loads of 16 bytes in flight per thread
__device__ __forceinline__ void gather_range(const GatherArgs& ga, int64_t lo, int64_t hi, int gt) {
  const int64_t step = ga.chunk ? ga.chunk : ga.seg;
  int64_t x = lo;
#pragma unroll 1
  while (x < hi) {
    const int64_t blk = x / step;
    const int64_t end = min(hi, (blk + 1) * step);
    const int owner = ga.chunk ? static_cast<int>(blk % ga.world) : static_cast<int>(blk);
    if (owner != ga.rank) {
      const uint4* src = reinterpret_cast<const uint4*>(ga.peers[owner] + x * 2);
      uint4* dst = reinterpret_cast<uint4*>(ga.local + x);
      const int64_t nv = (end - x) >> 3;
#pragma unroll 1
      for (int64_t i = gt; i < nv; i += 8 * kGatherThreads) {
        uint4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (i + j * kGatherThreads < nv) v[j] = src[i + j * kGatherThreads];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (i + j * kGatherThreads < nv) dst[i + j * kGatherThreads] = v[j];
      }
    }
    x = end;
  }
}

// kE2Bf16Sq / kE2Bf16ResSq: the bf16 store plus the sum of squares of the stored values, one fp32 partial per
// (tile, CTA of the pair, epilogue warp) -- the weight-gradient form behind the one-GPU clip norm.
// Fused elementwise epilogues (operands in EpiAux):
//   kE2Rope      : interleaved rotary embedding of the leading aux.i1 columns (the q / k blocks of a projection) at
//                  position row % aux.i0, cos / sin tables aux.t0 / aux.t1 [L, 64] (kernel/rotary.py:20-141)
//   kE2Swiglu    : the merged fc1 | gate projection: the pair's two B halves are rows [j0, j0 + 128) and
//                  [f + j0, f + j0 + 128) of B (f = aux.i0), so one tile holds both operands of silu(a) * b for 128
//                  columns; stores a and b (kept for the backward) and h = silu(a) * b into aux.out2
//                  (kernel/swiglu.py:4-17)
//   kE2SwigluBwd : the fc2 input gradient dh (N = f columns) is not stored: with a, b from aux.t0 (the saved
//                  fc1 | gate output, row stride aux.ld2) the epilogue stores da at C[:, col] and db at C[:, f + col]
// Every fused epilogue rounds the accumulator to bf16 first, as the separate kernels read it from memory.
enum Epi2 : int {
  kE2Bf16 = 0, kE2Bf16Res = 1, kE2F32 = 2, kE2Bf16Sq = 3, kE2Bf16ResSq = 4, kE2Rope = 5, kE2Swiglu = 6,
  kE2SwigluBwd = 7
};
__host__ __device__ constexpr bool e2_res(int e) { return e == kE2Bf16Res || e == kE2Bf16ResSq; }
__host__ __device__ constexpr bool e2_sq(int e) { return e == kE2Bf16Sq || e == kE2Bf16ResSq; }

// operands of the fused epilogues (unused fields zero)
struct EpiAux {
  const __nv_bfloat16* t0;   // kE2Rope: cos [L, 64]; kE2SwigluBwd: fc1 | gate output [M, 2f]
  const __nv_bfloat16* t1;   // kE2Rope: sin [L, 64]
  __nv_bfloat16* out2;       // kE2Swiglu: h [M, f]
  int64_t ld2;               // row stride of out2 (kE2Swiglu) / t0 (kE2SwigluBwd)
  int i0;                    // kE2Rope: L; kE2Swiglu / kE2SwigluBwd: f
  int i1;                    // kE2Rope: rotated leading columns (a multiple of 128)
};

// BN: output columns per tile (256; 192 or 128 for shapes whose 256-wide tiles leave a mostly empty last round);
// each CTA loads BN / 2 rows of B per K slab
template <int BN, int STAGES>
struct Smem2 {
  static constexpr int A_BYTES = kBM * kBK * 2;             // 16 KB
  // this CTA's half of the B slab, in whole 64-wide swizzle atoms (BN = 192: 96 rows / columns, 2 atoms reserved)
  static constexpr int B_ATOMS = (BN / 2 + 63) / 64;
  static constexpr int B_BYTES = B_ATOMS * 64 * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;
  static_assert(TOTAL <= 227 * 1024, "two-CTA GEMM shared memory above the per-CTA limit");
};
template <int BN>
struct PairCfg;
template <>
struct PairCfg<256> {
  static constexpr int STAGES = 6;
};
template <>
struct PairCfg<192> {
  static constexpr int STAGES = 6;
};
template <>
struct PairCfg<128> {
  static constexpr int STAGES = 8;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared-memory location in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t mapa_u32(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMA 2-D load into this CTA's shared memory whose completion bytes go to the mbarrier at cluster address bar
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// arrive (once) on the mbarrier at cluster address bar when the pair's previously issued MMAs have completed
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// bounded wait with cluster-scope acquire (arrivals from the peer CTA)
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort, int* status,
                                                  int site) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 63u) == 0u) {
      if (abort != nullptr && *abort) return false;
      if (globaltimer_ns() - t0 > FYB_WAIT_NS) {
        record_status(status, kMbarTimeout, site);
        if (abort != nullptr) *abort = 1;
        return false;
      }
    }
  }
}

// stores 32 values of one output row; returns the sum of squares of the stored bf16 values (sq epilogues)
template <int EPI>
__device__ __forceinline__ float store_row32(const uint32_t (&r)[32], void* Cv, const __nv_bfloat16* R, int row,
                                             int col, int N, int64_t ldc, int64_t ldr) {
  if (EPI == kE2F32) {
    float* C = reinterpret_cast<float*>(Cv) + static_cast<int64_t>(row) * ldc + col;
    if (col + 32 <= N && (ldc % 4) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(C + j) = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                        __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col + j < N) C[j] = __uint_as_float(r[j]);
    }
    return 0.f;
  }
  __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(Cv) + static_cast<int64_t>(row) * ldc + col;
  uint32_t p[16];
  if (e2_res(EPI)) {
    const __nv_bfloat16* Rr = R + static_cast<int64_t>(row) * ldr + col;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int e = 2 * j;
      const float r0 = col + e < N ? __bfloat162float(Rr[e]) : 0.f;
      const float r1 = col + e + 1 < N ? __bfloat162float(Rr[e + 1]) : 0.f;
      p[j] = pack_bf16(bf16_round(__uint_as_float(r[e])) + r0, bf16_round(__uint_as_float(r[e + 1])) + r1);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) p[j] = pack_bf16(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
  }
  if (col + 32 <= N && (ldc % 8) == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4*>(C + 8 * j) = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (col + j < N) {
        const uint16_t h =
            (j & 1) ? static_cast<uint16_t>(p[j >> 1] >> 16) : static_cast<uint16_t>(p[j >> 1] & 0xffffu);
        C[j] = __ushort_as_bfloat16(h);
      }
    }
  }
  float sq = 0.f;
  if (e2_sq(EPI)) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float2 x = unpack_bf16(p[j]);
      if (col + 2 * j < N) sq = fmaf(x.x, x.x, sq);
      if (col + 2 * j + 1 < N) sq = fmaf(x.y, x.y, sq);
    }
  }
  return sq;
}

__device__ __forceinline__ void store16x2(__nv_bfloat16* p, const uint32_t (&w)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4*>(p + 8 * j) = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}

__device__ __forceinline__ void load16x2(const __nv_bfloat16* p, uint32_t (&w)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 v = *reinterpret_cast<const uint4*>(p + 8 * j);
    w[4 * j] = v.x;
    w[4 * j + 1] = v.y;
    w[4 * j + 2] = v.z;
    w[4 * j + 3] = v.w;
  }
}

// 32 columns of a rotated block (col within [0, aux.i1), 16-byte aligned rows): pairs (2i, 2i + 1) of the head's
// 128 columns turned by the angle of position pos and frequency index i = (col mod 128) / 2 + pair
__device__ __forceinline__ void rope_store32(const uint32_t (&r)[32], __nv_bfloat16* C, const EpiAux& aux, int pos,
                                             int col) {
  uint32_t cw[8], sw[8];
  const int64_t t = static_cast<int64_t>(pos) * 64 + ((col & 127) >> 1);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const uint4 c4 = *reinterpret_cast<const uint4*>(aux.t0 + t + 8 * j);
    const uint4 s4 = *reinterpret_cast<const uint4*>(aux.t1 + t + 8 * j);
    cw[4 * j] = c4.x, cw[4 * j + 1] = c4.y, cw[4 * j + 2] = c4.z, cw[4 * j + 3] = c4.w;
    sw[4 * j] = s4.x, sw[4 * j + 1] = s4.y, sw[4 * j + 2] = s4.z, sw[4 * j + 3] = s4.w;
  }
  uint32_t p[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    // pair k uses table entry k: entries 2m, 2m + 1 of the 16 sit in word m
    const float2 cs2 = unpack_bf16(cw[k >> 1]), sn2 = unpack_bf16(sw[k >> 1]);
    const float cs = (k & 1) ? cs2.y : cs2.x, sn = (k & 1) ? sn2.y : sn2.x;
    float o0, o1;
    rope_rot(bf16_round(__uint_as_float(r[2 * k])), bf16_round(__uint_as_float(r[2 * k + 1])), cs, sn, o0, o1);
    p[k] = pack_bf16(o0, o1);
  }
  store16x2(C, p);
}

// The work of one CTA pair, the same sequence for its producer, MMA and epilogue warps.
//   uniform split-K (sk_per == 0): units u = cluster, cluster + clusters, ...: tile u / splits, K part u % splits of
//     `splits` equal parts; a partial's workspace slot is u.
//   stream-K (sk_per > 0): the pair's contiguous range [cluster sk_per, (cluster + 1) sk_per) of the tile-major K
//     iterations (tile t covers [t nk, (t + 1) nk)), cut at tile boundaries: every pair does the same number of K
//     blocks, and only the tiles cut by a range boundary are summed from parts. A pair has at most two partial
//     segments (the first and the last of its range), workspace slots 2 cluster + {0: starts the range, 1: ends it}.
struct Work {
  int t, kb0, kb1;   // tile, K blocks [kb0, kb1)
  int part, parts;   // this segment's index among the tile's K parts (in K order), their number
  int slot;          // workspace slot of this part
};

struct Sched {
  int cluster, clusters, splits, nk, k_chunk, num_units;
  int64_t per, g0, g, g1;
  int u;
  __device__ __forceinline__ Sched(int cluster_, int clusters_, int splits_, int nk_, int num_tiles, int64_t per_)
      : cluster(cluster_), clusters(clusters_), splits(splits_), nk(nk_), k_chunk((nk_ + splits_ - 1) / splits_),
        num_units(num_tiles * splits_), per(per_), u(cluster_) {
    const int64_t total = static_cast<int64_t>(num_tiles) * nk_;
    g0 = g = per_ > 0 ? min(total, static_cast<int64_t>(cluster_) * per_) : 0;
    g1 = per_ > 0 ? min(total, g0 + per_) : 0;
  }
  __device__ __forceinline__ bool next(Work& w) {
    if (per == 0) {
      if (u >= num_units) return false;
      w.t = u / splits;
      w.part = u % splits;
      w.parts = splits;
      w.kb0 = w.part * k_chunk;
      w.kb1 = min(nk, w.kb0 + k_chunk);
      w.slot = u;
      u += clusters;
      return true;
    }
    if (g >= g1) return false;
    const int64_t t = g / nk;
    w.t = static_cast<int>(t);
    w.kb0 = static_cast<int>(g - t * nk);
    w.kb1 = static_cast<int>(min(static_cast<int64_t>(nk), g1 - t * nk));
    const int64_t fc = (t * nk) / per, lc = ((t + 1) * nk - 1) / per;
    w.parts = static_cast<int>(lc - fc + 1);
    w.part = static_cast<int>(cluster - fc);
    w.slot = cluster * 2 + (g == g0 ? 0 : 1);
    g = t * nk + w.kb1;
    return true;
  }
  // workspace slot of part j of tile t
  __device__ __forceinline__ int64_t part_slot(int t, int j) const {
    if (per == 0) return static_cast<int64_t>(t) * splits + j;
    const int64_t cj = (static_cast<int64_t>(t) * nk) / per + j;
    const int64_t start = max(static_cast<int64_t>(t) * nk, cj * per);
    return cj * 2 + (start == cj * per ? 0 : 1);
  }
};

template <int BN, bool A_MN, bool B_MN, int EPI, bool GATHER = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GATHER ? kThreadsG : kThreads2, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, void* Cv,
                     const __nv_bfloat16* R, int M, int N, int K, int64_t ldc, int64_t ldr, int splits, int64_t sk_per,
                     float* ws, int* counters, int* status, float* sq_part, const EpiAux aux, const GatherArgs ga) {
  static_assert(!GATHER || !B_MN, "the gather form reads K-major weight rows");
  static_assert(EPI != kE2Swiglu || (BN == 256 && !B_MN), "the SwiGLU epilogue pairs two 128-row B halves");
  constexpr int kStages2 = PairCfg<BN>::STAGES;
  using S = Smem2<BN, kStages2>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* empty = full + kStages2;
  uint64_t* tfull = empty + kStages2;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_rank();            // 0: leader (issues the MMAs), 1: peer
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int num_m = (M + 2 * kBM - 1) / (2 * kBM);
  // kE2Swiglu: tile nb covers columns [128 nb, 128 nb + 128) of both halves
  const int num_n = EPI == kE2Swiglu ? (aux.i0 + 127) / 128 : (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_k = (K + kBK - 1) / kBK;
  // split-K (splits = 1 .. 4): work unit u = (tile u / splits, K part u % splits); the parts of a tile are
  // consecutive units, so they run in the same wave
  const int num_units = num_tiles * splits;
  // accumulator buffers at a power-of-two column stride (BN = 192 uses columns [0, 192) and [256, 448))
  constexpr uint32_t ACC_STRIDE = BN <= 128 ? 128u : 256u;
  constexpr uint32_t TMEM_COLS = 2 * ACC_STRIDE;
  // bytes one CTA's loads deliver per stage: the K-major B half is BN / 2 rows of 128 bytes; the MN-major half is
  // whole 64-wide atoms (BN = 192: 128 columns loaded, 96 used by the MMA)
  constexpr uint32_t TX_BYTES = S::A_BYTES + (B_MN ? S::B_BYTES : (BN / 2) * kBK * 2);
  constexpr uint32_t IDESC = idesc_bf16(2 * kBM, BN, A_MN, B_MN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(&full[s], 1);       // the leader's producer arms it with the pair's bytes
      mbar_init(&empty[s], 1);      // one commit from the leader's MMA thread
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);      // one commit from the leader's MMA thread
      mbar_init(&tempty[b], 8);     // 4 epilogue warps of each CTA (only the leader's is used)
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();                    // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      Sched sc(cluster_id, num_clusters, splits, num_k, num_tiles, sk_per);
      Work w;
      while (ok && sc.next(w)) {
        const int t = w.t;
        const int mb = t % num_m, nb = t / num_m;
        const int m0 = mb * 2 * kBM + static_cast<int>(crank) * kBM;
        const int n0 = EPI == kE2Swiglu ? nb * 128 + static_cast<int>(crank) * aux.i0
                                        : nb * BN + static_cast<int>(crank) * (BN / 2);
        const int kb0 = w.kb0, kb1 = w.kb1;
        if constexpr (GATHER) {
          // every share of tile column nb pulled into this replica (then visible to the TMA loads below)
          if (!wait_count(ga.counters + nb, 2 * num_m, abort_flag, status, 27)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, status, 21)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * S::STAGE_BYTES;
          uint8_t* sb = sa + S::A_BYTES;
          const uint32_t bar = mapa_u32(&full[s], 0);
          if (crank == 0) mbar_arrive_expect_tx(&full[s], 2 * TX_BYTES);
          if (!A_MN) {
            tma_load_2d_pair(sa, &tmA, bar, kb * kBK, m0);
          } else {
#pragma unroll
            for (int j = 0; j < kBM / 64; ++j) tma_load_2d_pair(sa + j * 8192, &tmA, bar, m0 + 64 * j, kb * kBK);
          }
          if (!B_MN) {
            tma_load_2d_pair(sb, &tmB, bar, kb * kBK, n0);
          } else {
#pragma unroll
            for (int j = 0; j < S::B_ATOMS; ++j) tma_load_2d_pair(sb + j * 8192, &tmB, bar, n0 + 64 * j, kb * kBK);
          }
          if (++s == kStages2) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // drain: every issued stage must have been consumed before the CTA may exit
      for (int i = 0; i < kStages2; ++i) {
        mbar_wait(&empty[s], ph ^ 1u, nullptr, status, 22);
        if (++s == kStages2) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------------------------------- UMMA issuer (leader)
    if (crank == 0 && lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t acc_ph = 0;
      bool ok = true;
      Sched sc(cluster_id, num_clusters, splits, num_k, num_tiles, sk_per);
      Work w;
      while (ok && sc.next(w)) {
        if (!mbar_wait_cluster(&tempty[acc], acc_ph ^ 1u, abort_flag, status, 23)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc) * ACC_STRIDE;
        const int kb0 = w.kb0, kb1 = w.kb1;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag, status, 24)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + s * S::STAGE_BYTES);
          const uint32_t b0 = a0 + S::A_BYTES;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = A_MN ? sw128_desc(a0 + k * 2048, 8192, 1024) : sw128_desc(a0 + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sw128_desc(b0 + k * 2048, 8192, 1024) : sw128_desc(b0 + k * 32, 16, 1024);
            umma_bf16_pair(d, ad, bd, IDESC, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          // the stage may be refilled in both CTAs once these MMAs have read it
          umma_commit_pair(mapa_u32(&empty[s], 0));
          umma_commit_pair(mapa_u32(&empty[s], 1));
          if (++s == kStages2) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(mapa_u32(&tfull[acc], 0));   // accumulator rows ready in both CTAs' TMEM
        umma_commit_pair(mapa_u32(&tfull[acc], 1));
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1u;
      }
    }
  } else if (GATHER && warp >= kThreads2 / 32) {
    // ---------------------------------------------------------------------------------------- gather (pull)
    const int gt = threadIdx.x - kThreads2;
    const int shares = 2 * num_m;
#pragma unroll 1
    for (int u = cluster_id; u < num_units; u += num_clusters) {
      const int mb = u % num_m, nb = u / num_m;
      int64_t lo_all, tot, per;
      int share;
      if constexpr (EPI == kE2Swiglu) {
        // the tile reads rows [128 nb, 128 nb + 128) of the fc1 half (CTA 0's B half) and the same rows of the gate
        // half (CTA 1's): each CTA pulls share mb of num_m of its own half
        const int f = aux.i0;
        const int r0 = static_cast<int>(crank) * f + nb * 128;
        const int r1 = min(static_cast<int>(crank) * f + f, r0 + 128);
        lo_all = ga.w_off + static_cast<int64_t>(r0) * K;
        tot = static_cast<int64_t>(max(0, r1 - r0)) * K;
        per = ((tot / 8 + num_m - 1) / num_m) * 8;
        share = mb;
      } else {
        lo_all = ga.w_off + static_cast<int64_t>(nb) * BN * K;
        tot = static_cast<int64_t>(min(N, (nb + 1) * BN) - nb * BN) * K;
        per = ((tot / 8 + shares - 1) / shares) * 8;      // whole 16-byte vectors per share
        share = mb * 2 + static_cast<int>(crank);
      }
      const int64_t lo = lo_all + min(tot, share * per), hi = lo_all + min(tot, (share + 1) * per);
      gather_range(ga, lo, hi, gt);
      asm volatile("bar.sync 1, %0;" ::"n"(kGatherThreads) : "memory");   // the gather warps only
      if (gt == 0) {
        fence_proxy_async_global();
        asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(ga.counters + nb), "r"(1) : "memory");
      }
    }
  } else {
    // ---------------------------------------------------------------------------------------- epilogue
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_ph = 0;
    Sched sc(cluster_id, num_clusters, splits, num_k, num_tiles, sk_per);
    Work w;
    while (sc.next(w)) {
      const int t = w.t;
      const int mb = t % num_m, nb = t / num_m;
      if constexpr (EPI == kE2SwigluBwd) {
        // the saved a, b of this tile's rows into L2 while its mainloop still runs (the chunk loop below then
        // waits for L2, not DRAM): per thread its row's BN columns of both halves, 128-byte lines
        const int prow = mb * 2 * kBM + static_cast<int>(crank) * kBM + q * 32 + lane;
        if (prow < M) {
          const __nv_bfloat16* u = aux.t0 + static_cast<int64_t>(prow) * aux.ld2;
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) {
            const int pc = nb * BN + 64 * j;
            if (pc < N) {
              prefetch_l2(u + pc);
              prefetch_l2(u + aux.i0 + pc);
            }
          }
        }
      }
      if (!mbar_wait(&tfull[acc], acc_ph, abort_flag, status, 25)) break;
      tc_fence_after();
      const int row = mb * 2 * kBM + static_cast<int>(crank) * kBM + q * 32 + lane;
      const uint32_t tb = tmem_base + static_cast<uint32_t>(acc) * ACC_STRIDE + (static_cast<uint32_t>(q * 32) << 16);
      bool last = true;
      const float4* pp[4] = {nullptr, nullptr, nullptr, nullptr};   // the last arriver: every part's words of
      int my_split = 0;                                                // this lane's row (its own read from TMEM)
      const int nparts = w.parts;
      if (nparts >= 2) {
        // publish this K part's partial (this warp's 32 rows x BN, fp32), then count the warp's arrival for the
        // tile: the last of the parts to arrive sums them in K order ((p0 + p1) + p2) + p3 -- its own from TMEM --
        // and stores, so the result does not depend on the order of arrival.
        // workspace layout per (slot, CTA): 16-byte word w = 4 consecutive columns of row r at float4 index
        // w x 128 + r, so the 32 lanes of a warp (32 consecutive rows) store / load 512 contiguous bytes
        float4* mine =
            reinterpret_cast<float4*>(ws + (static_cast<int64_t>(w.slot) * 2 + crank) * kBM * BN) + q * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tb + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            mine[(c * 8 + j / 4) * kBM] = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                      __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
        }
        __threadfence();
        __syncwarp();
        int* cnt = counters + (static_cast<int64_t>(t) * 2 + crank) * 4 + q;
        int prev = 0;
        if (lane == 0) prev = atomicAdd(cnt, 1);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        last = prev == nparts - 1;
        if (last) {
          __threadfence();
          if (lane == 0) *cnt = 0;                   // ready for the next GEMM that uses these counters
          my_split = w.part;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (j < nparts)
              pp[j] = reinterpret_cast<const float4*>(ws + (sc.part_slot(t, j) * 2 + crank) * kBM * BN) + q * 32 +
                      lane;
        }
      }
      float sq = 0.f;
      if constexpr (EPI == kE2Swiglu) {
        // TMEM columns [0, 128): a = fc1 columns j0.., [128, 256): b = gate columns f + j0..
        const int f = aux.i0;
        __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(Cv);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t ra[32], rb[32];
          tmem_ld32(tb + c * 32, ra);
          tmem_ld32(tb + 128 + c * 32, rb);
          tmem_ld_wait();
          const int j = nb * 128 + c * 32;
          if (row < M && j < f) {
            uint32_t pa[16], pb[16], ph[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              pa[k] = pack_bf16(__uint_as_float(ra[2 * k]), __uint_as_float(ra[2 * k + 1]));
              pb[k] = pack_bf16(__uint_as_float(rb[2 * k]), __uint_as_float(rb[2 * k + 1]));
              const float2 a = unpack_bf16(pa[k]), b = unpack_bf16(pb[k]);
              ph[k] = pack_bf16(swiglu_val(a.x, b.x), swiglu_val(a.y, b.y));
            }
            __nv_bfloat16* crow = C + static_cast<int64_t>(row) * ldc;
            store16x2(crow + j, pa);
            store16x2(crow + f + j, pb);
            store16x2(aux.out2 + static_cast<int64_t>(row) * aux.ld2 + j, ph);
          }
        }
      }
      const int pos = EPI == kE2Rope && row < M ? row % aux.i0 : 0;
      // kE2SwigluBwd: the saved a, b of chunk c + 1 are loaded while chunk c is processed
      uint32_t ua[16], ub[16];
      if (EPI == kE2SwigluBwd && row < M && nb * BN < N) {
        const __nv_bfloat16* u = aux.t0 + static_cast<int64_t>(row) * aux.ld2 + nb * BN;
        load16x2(u, ua);
        load16x2(u + aux.i0, ub);
      }
#pragma unroll 1
      for (int c = 0; EPI != kE2Swiglu && last && c < BN / 32; ++c) {
        uint32_t r[32];
        const int col = nb * BN + c * 32;
        tmem_ld32(tb + c * 32, r);        // warp-collective: every lane, whatever its row
        tmem_ld_wait();
        if constexpr (EPI == kE2SwigluBwd) {
          if (row < M && col < N) {
            uint32_t pa[16], pb[16];
            uint32_t ca[16], cb[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) ca[k] = ua[k], cb[k] = ub[k];
            if (c + 1 < BN / 32 && col + 32 < N) {
              const __nv_bfloat16* u = aux.t0 + static_cast<int64_t>(row) * aux.ld2 + col + 32;
              load16x2(u, ua);
              load16x2(u + aux.i0, ub);
            }
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const float2 a = unpack_bf16(ca[k]), b = unpack_bf16(cb[k]);
              const float g0 = bf16_round(__uint_as_float(r[2 * k])), g1 = bf16_round(__uint_as_float(r[2 * k + 1]));
              float da0, db0, da1, db1;
              swiglu_grad(a.x, b.x, g0, da0, db0);
              swiglu_grad(a.y, b.y, g1, da1, db1);
              pa[k] = pack_bf16(da0, da1);
              pb[k] = pack_bf16(db0, db1);
            }
            __nv_bfloat16* crow = reinterpret_cast<__nv_bfloat16*>(Cv) + static_cast<int64_t>(row) * ldc;
            store16x2(crow + col, pa);
            store16x2(crow + aux.i0 + col, pb);
          }
          continue;
        }
        if constexpr (EPI == kE2Rope) {
          if (row < M && col < N) {
            if (col < aux.i1)
              rope_store32(r, reinterpret_cast<__nv_bfloat16*>(Cv) + static_cast<int64_t>(row) * ldc + col, aux, pos,
                           col);
            else
              store_row32<kE2Bf16>(r, Cv, R, row, col, N, ldc, ldr);
          }
          continue;
        }
        if (pp[0] != nullptr) {
          // sum of the K parts in K order; this unit's part is the accumulator just read
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            float4 tot = my_split == 0 ? make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                     __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]))
                                       : pp[0][(c * 8 + j / 4) * kBM];
#pragma unroll
            for (int sp = 1; sp < 4; ++sp) {
              if (sp >= nparts) break;
              const float4 o = sp == my_split
                                   ? make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                 __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]))
                                   : pp[sp][(c * 8 + j / 4) * kBM];
              tot.x += o.x;
              tot.y += o.y;
              tot.z += o.z;
              tot.w += o.w;
            }
            r[j] = __float_as_uint(tot.x);
            r[j + 1] = __float_as_uint(tot.y);
            r[j + 2] = __float_as_uint(tot.z);
            r[j + 3] = __float_as_uint(tot.w);
          }
        }
        if (row < M && col < N) sq += store_row32<EPI>(r, Cv, R, row, col, N, ldc, ldr);
      }
      if (e2_sq(EPI) && last) {
        // one partial per (tile, CTA, epilogue warp), every slot written exactly once (no clearing needed)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) sq_part[(static_cast<int64_t>(t) * 2 + crank) * 4 + q] = sq;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_u32(&tempty[acc], 0));
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1u;
    }
  }

  tc_fence_before();
  cluster_sync();                    // both CTAs done with TMEM and with each other's barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

struct PairArgs {
  int splits;
  float* ws;
  int* counters;
  float* sq_part;
  int64_t sk_per = 0;       // stream-K: K iterations per CTA pair (0: uniform split-K / none)
  int sk_clusters = 0;      // stream-K: CTA pairs launched
};

template <int BN, bool A_MN, bool B_MN, int EPI, bool GATHER = false>
void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, void* C, const __nv_bfloat16* R, int M, int N, int K,
                 int64_t ldc, int64_t ldr, const PairArgs& pa, cudaStream_t stream, const EpiAux& aux = EpiAux{},
                 const GatherArgs& ga = GatherArgs{}) {
  using S = Smem2<BN, PairCfg<BN>::STAGES>;
  auto kern = gemm_pair_kernel<BN, A_MN, B_MN, EPI, GATHER>;
  static bool attr_set = false;
  if (!attr_set) {
    FYB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL));
    attr_set = true;
  }
  const int units = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + BN - 1) / BN) * pa.splits;
  const int clusters = pa.sk_per > 0 ? pa.sk_clusters : std::max(1, std::min(units, num_sms() / 2));
  kern<<<2 * clusters, GATHER ? kThreadsG : kThreads2, S::TOTAL, stream>>>(
      ta, tb, C, R, M, N, K, ldc, ldr, pa.splits, pa.sk_per, pa.ws, pa.counters, status_ptr(), pa.sq_part, aux, ga);
  check_launch("gemm_pair");
}

template <int BN, int EPI>
void dispatch_pair(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, void* C,
                   const __nv_bfloat16* R, int M, int N, int K, int64_t ldc, int64_t ldr, const PairArgs& pa,
                   cudaStream_t st) {
  if (!a_mn && !b_mn) launch_pair<BN, false, false, EPI>(ta, tb, C, R, M, N, K, ldc, ldr, pa, st);
  else if (!a_mn && b_mn) launch_pair<BN, false, true, EPI>(ta, tb, C, R, M, N, K, ldc, ldr, pa, st);
  else if (a_mn && b_mn) launch_pair<BN, true, true, EPI>(ta, tb, C, R, M, N, K, ldc, ldr, pa, st);
  else launch_pair<BN, true, false, EPI>(ta, tb, C, R, M, N, K, ldc, ldr, pa, st);
}

template <int EPI>
void dispatch_pair_bn(int bn, bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, void* C,
                      const __nv_bfloat16* R, int M, int N, int K, int64_t ldc, int64_t ldr, const PairArgs& pa,
                      cudaStream_t st) {
  if (bn == 256) dispatch_pair<256, EPI>(a_mn, b_mn, ta, tb, C, R, M, N, K, ldc, ldr, pa, st);
  else if (bn == 192) dispatch_pair<192, EPI>(a_mn, b_mn, ta, tb, C, R, M, N, K, ldc, ldr, pa, st);
  else dispatch_pair<128, EPI>(a_mn, b_mn, ta, tb, C, R, M, N, K, ldc, ldr, pa, st);
}

// Arrival counters of the split-K epilogue, one per (tile, CTA of the pair, epilogue warp): zeroed once per device
// and left zero by every GEMM (the second arrival resets its counter), so one buffer serves every call on the
// stream. Sized for 16 Ki tiles.
constexpr int kMaxPairTiles = 16384;
int* pair_counters() {
  static int* ptr[64] = {nullptr};
  int dev = 0;
  FYB_CUDA(cudaGetDevice(&dev));
  FYB_CHECK(dev >= 0 && dev < 64, "gemm_pair: device index out of range");
  if (ptr[dev] == nullptr) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    FYB_CUDA(cudaStreamIsCapturing(cur_stream(), &cs));
    FYB_CHECK(cs == cudaStreamCaptureStatusNone,
              "gemm_pair: the first split-K GEMM on a device must run before any stream capture");
    FYB_CUDA(cudaMalloc(&ptr[dev], sizeof(int) * kMaxPairTiles * 8));
    FYB_CUDA(cudaMemset(ptr[dev], 0, sizeof(int) * kMaxPairTiles * 8));
    FYB_CUDA(cudaDeviceSynchronize());
  }
  return ptr[dev];
}

}  // namespace

// C = A @ B^T on CTA pairs (operand conventions as gemm()). C: bf16 or fp32 [M, N]; R: bf16 residual.
// bn: output tile width, 256, 192 or 128; splits: 1 .. 4 (each tile's K range in `splits` parts on as many pairs,
// summed in part order by the epilogue of the last to finish; the fp32 workspace is allocated here), or 0 for
// stream-K (every pair takes an equal contiguous share of the tile-major K iterations; only the tiles cut by a share
// boundary are summed from parts).
void gemm_pair(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool a_mn, bool b_mn,
               const c10::optional<at::Tensor>& R, int64_t bn, int64_t splits) {
  FYB_RANGE("fyb::gemm_pair");
  FYB_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm_pair: CUDA tensors expected");
  FYB_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm_pair: bf16 operands expected");
  FYB_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm_pair: 2-D tensors expected");
  FYB_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm_pair: last dimension must be contiguous");
  const int64_t M = a_mn ? A.size(1) : A.size(0);
  const int64_t K = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0);
  const int64_t Kb = b_mn ? B.size(0) : B.size(1);
  FYB_CHECK(K == Kb && K > 0, "gemm_pair: inner dimensions differ or are empty");
  FYB_CHECK(C.size(0) == M && C.size(1) == N, "gemm_pair: output shape mismatch");
  FYB_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm_pair: dimension too large");
  const bool f32 = C.scalar_type() == at::kFloat;
  FYB_CHECK(f32 || C.scalar_type() == at::kBFloat16, "gemm_pair: output must be bf16 or fp32");
  const __nv_bfloat16* Rp = nullptr;
  int64_t ldr = 0;
  if (R.has_value() && R->defined()) {
    FYB_CHECK(!f32, "gemm_pair: residual needs a bf16 output");
    FYB_CHECK(R->scalar_type() == at::kBFloat16 && R->dim() == 2 && R->size(0) == M && R->size(1) == N &&
                  R->stride(1) == 1,
              "gemm_pair: residual must be bf16 [M, N] with contiguous rows");
    Rp = reinterpret_cast<const __nv_bfloat16*>(R->data_ptr());
    ldr = R->stride(0);
  }
  FYB_CHECK(bn == 256 || bn == 192 || bn == 128, "gemm_pair: tile width must be 256, 192 or 128");
  FYB_CHECK(splits >= 0 && splits <= 4, "gemm_pair: splits must be 0 (stream-K) or 1 .. 4");
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(A.device());
  cudaStream_t st = cur_stream();
  const int64_t tiles = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + bn - 1) / bn);
  const int64_t num_k = (K + kBK - 1) / kBK;
  PairArgs pa{static_cast<int>(splits), nullptr, nullptr, nullptr};
  at::Tensor ws;
  if (splits == 0) {
    // stream-K: every CTA pair takes the same number of the tile-major K iterations
    const int64_t total = tiles * num_k;
    const int64_t clusters = std::max<int64_t>(1, std::min<int64_t>(num_sms() / 2, total));
    // at least a third of a tile's K blocks per pair, so a tile is cut into at most 4 parts
    const int64_t per = std::max((total + clusters - 1) / clusters, (num_k + 2) / 3);
    FYB_CHECK((num_k + per - 1) / per + 1 <= 4, "gemm_pair: stream-K would cut a tile into more than 4 parts");
    FYB_CHECK(tiles <= kMaxPairTiles, "gemm_pair: too many tiles for stream-K");
    pa.splits = 1;
    pa.sk_per = per;
    pa.sk_clusters = static_cast<int>((total + per - 1) / per);
    ws = at::empty({static_cast<int64_t>(pa.sk_clusters) * 2 * 2 * kBM, bn}, A.options().dtype(at::kFloat));
    pa.ws = ws.data_ptr<float>();
    pa.counters = pair_counters();
  } else if (splits >= 2) {
    FYB_CHECK((splits - 1) * ((num_k + splits - 1) / splits) < num_k,
              "gemm_pair: split-K needs at least one K block in every part");
    FYB_CHECK(tiles <= kMaxPairTiles, "gemm_pair: too many tiles for split-K");
    ws = at::empty({tiles * splits * 2 * kBM, bn}, A.options().dtype(at::kFloat));
    pa.ws = ws.data_ptr<float>();
    pa.counters = pair_counters();
  }
  const CUtensorMap ta = a_mn ? make_tmap_2d(A.data_ptr(), K, M, A.stride(0), 64)
                              : make_tmap_2d(A.data_ptr(), M, K, A.stride(0), kBM);
  const CUtensorMap tb = b_mn ? make_tmap_2d(B.data_ptr(), K, N, B.stride(0), 64)
                              : make_tmap_2d(B.data_ptr(), N, K, B.stride(0), static_cast<int>(bn / 2));
  void* Cp = C.data_ptr();
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  const int64_t ldc = C.stride(0);
  const int b = static_cast<int>(bn);
  if (f32) dispatch_pair_bn<kE2F32>(b, a_mn, b_mn, ta, tb, Cp, Rp, m, n, k, ldc, ldr, pa, st);
  else if (Rp != nullptr) dispatch_pair_bn<kE2Bf16Res>(b, a_mn, b_mn, ta, tb, Cp, Rp, m, n, k, ldc, ldr, pa, st);
  else dispatch_pair_bn<kE2Bf16>(b, a_mn, b_mn, ta, tb, Cp, Rp, m, n, k, ldc, ldr, pa, st);
}

// partials a gemm_pair_sq call writes: one per (256 x 256 tile, CTA of the pair, epilogue warp)
int64_t gemm_pair_sq_slots(int64_t M, int64_t N) { return ((M + 255) / 256) * ((N + 255) / 256) * 8; }

// Weight gradient on CTA pairs: C = A^T B (A = dy [K, M], B = x [K, N], both MN-major), bf16, optionally added to C's
// current contents (earlier micro-batches), with the sum of squares of the stored values in sq_part (every one of
// gemm_pair_sq_slots(M, N) partials written). Returns the number of partials.
int64_t gemm_pair_sq(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool accumulate, at::Tensor& sq_part) {
  FYB_RANGE("fyb::gemm_pair_sq");
  const int64_t K = A.size(0), M = A.size(1), N = B.size(1);
  FYB_CHECK(B.size(0) == K && C.size(0) == M && C.size(1) == N && K > 0, "gemm_pair_sq: shape mismatch");
  FYB_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm_pair_sq: contiguous rows expected");
  FYB_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm_pair_sq: dimension too large");
  const int64_t slots = gemm_pair_sq_slots(M, N);
  FYB_CHECK(sq_part.scalar_type() == at::kFloat && sq_part.is_contiguous() && sq_part.numel() >= slots,
            "gemm_pair_sq: partials buffer too small");
  if (M == 0 || N == 0) return 0;
  c10::cuda::CUDAGuard guard(A.device());
  cudaStream_t st = cur_stream();
  const CUtensorMap ta = make_tmap_2d(A.data_ptr(), K, M, A.stride(0), 64);
  const CUtensorMap tb = make_tmap_2d(B.data_ptr(), K, N, B.stride(0), 64);
  PairArgs pa{1, nullptr, nullptr, sq_part.data_ptr<float>()};
  void* Cp = C.data_ptr();
  const __nv_bfloat16* Rp = accumulate ? reinterpret_cast<const __nv_bfloat16*>(Cp) : nullptr;
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  const int64_t ldc = C.stride(0);
  if (accumulate) launch_pair<256, true, true, kE2Bf16ResSq>(ta, tb, Cp, Rp, m, n, k, ldc, ldc, pa, st);
  else launch_pair<256, true, true, kE2Bf16Sq>(ta, tb, Cp, Rp, m, n, k, ldc, ldc, pa, st);
  return slots;
}

namespace {
// bf16 [rows, cols] with contiguous, 16-byte aligned rows (the fused epilogues store 16 bytes at a time)
void check_rows16(const at::Tensor& t, const char* what) {
  FYB_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1 &&
                t.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
            what);
}
}  // namespace

// C = A @ B^T (A [M, K], B [N, K], both K-major) with the interleaved rotary embedding applied in the epilogue to
// the leading rot_cols columns (the q / k head blocks of a projection), token row r at position r mod L.
// cos / sin: bf16 [>= L, 64] (head dim 128), the tables rope_fwd takes. Rounding as gemm() followed by rope_fwd.
// bn: output tile width of the pair kernel (256, 192 or 128; the routed width of the plain GEMM of this shape).
void gemm_rope(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, const at::Tensor& cos_t,
               const at::Tensor& sin_t, int64_t L, int64_t rot_cols, int64_t bn) {
  FYB_RANGE("fyb::gemm_rope");
  check_rows16(A, "gemm_rope: A must be bf16 [M, K] with 16-byte aligned rows");
  check_rows16(B, "gemm_rope: B must be bf16 [N, K] with 16-byte aligned rows");
  check_rows16(C, "gemm_rope: C must be bf16 [M, N] with 16-byte aligned rows");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  FYB_CHECK(B.size(1) == K && K > 0 && C.size(0) == M && C.size(1) == N, "gemm_rope: shape mismatch");
  FYB_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm_rope: dimension too large");
  FYB_CHECK(L > 0 && M % L == 0, "gemm_rope: rows must be whole sequences of length L");
  FYB_CHECK(rot_cols >= 0 && rot_cols % 128 == 0 && rot_cols <= N, "gemm_rope: rotated columns: whole 128 heads");
  for (const at::Tensor* t : {&cos_t, &sin_t})
    FYB_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->dim() == 2 &&
                  t->size(0) >= L && t->size(1) == 64 && reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
              "gemm_rope: cos / sin must be contiguous bf16 [>= L, 64]");
  FYB_CHECK(bn == 256 || bn == 192 || bn == 128, "gemm_rope: tile width must be 256, 192 or 128");
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(A.device());
  const CUtensorMap ta = make_tmap_2d(A.data_ptr(), M, K, A.stride(0), kBM);
  const CUtensorMap tb = make_tmap_2d(B.data_ptr(), N, K, B.stride(0), static_cast<int>(bn / 2));
  const EpiAux aux{reinterpret_cast<const __nv_bfloat16*>(cos_t.data_ptr()),
                   reinterpret_cast<const __nv_bfloat16*>(sin_t.data_ptr()), nullptr, 0, static_cast<int>(L),
                   static_cast<int>(rot_cols)};
  const PairArgs pa{1, nullptr, nullptr, nullptr};
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  if (bn == 256) launch_pair<256, false, false, kE2Rope>(ta, tb, C.data_ptr(), nullptr, m, n, k, C.stride(0), 0, pa,
                                                         cur_stream(), aux);
  else if (bn == 192) launch_pair<192, false, false, kE2Rope>(ta, tb, C.data_ptr(), nullptr, m, n, k, C.stride(0), 0,
                                                              pa, cur_stream(), aux);
  else launch_pair<128, false, false, kE2Rope>(ta, tb, C.data_ptr(), nullptr, m, n, k, C.stride(0), 0, pa,
                                               cur_stream(), aux);
}

// The merged fc1 | gate projection with SwiGLU in the epilogue: u = A @ B^T (A [M, K], B = [fc1; gate] [2f, K], both
// K-major) and h = silu(u[:, :f]) * u[:, f:]. Returns {u [M, 2f] (kept for the backward), h [M, f]}; the values
// equal gemm() followed by swiglu_fwd.
std::vector<at::Tensor> gemm_swiglu(const at::Tensor& A, const at::Tensor& B) {
  FYB_RANGE("fyb::gemm_swiglu");
  check_rows16(A, "gemm_swiglu: A must be bf16 [M, K] with 16-byte aligned rows");
  check_rows16(B, "gemm_swiglu: B must be bf16 [2f, K] with 16-byte aligned rows");
  const int64_t M = A.size(0), K = A.size(1), N2 = B.size(0);
  FYB_CHECK(B.size(1) == K && K > 0 && N2 % 64 == 0, "gemm_swiglu: B must be [2f, K] with f a multiple of 32");
  FYB_CHECK(M < (1ll << 31) && N2 < (1ll << 31) && K < (1ll << 31), "gemm_swiglu: dimension too large");
  const int64_t f = N2 / 2;
  at::Tensor u = at::empty({M, N2}, A.options());
  at::Tensor h = at::empty({M, f}, A.options());
  if (M == 0) return {u, h};
  c10::cuda::CUDAGuard guard(A.device());
  const CUtensorMap ta = make_tmap_2d(A.data_ptr(), M, K, A.stride(0), kBM);
  const CUtensorMap tb = make_tmap_2d(B.data_ptr(), N2, K, B.stride(0), 128);
  const EpiAux aux{nullptr, nullptr, reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), f, static_cast<int>(f), 0};
  launch_pair<256, false, false, kE2Swiglu>(ta, tb, u.data_ptr(), nullptr, static_cast<int>(M), static_cast<int>(N2),
                                            static_cast<int>(K), N2, 0, PairArgs{1, nullptr, nullptr, nullptr},
                                            cur_stream(), aux);
  return {u, h};
}

// The fc2 input gradient with the SwiGLU backward in the epilogue: dh = G @ W (G [M, K]; W = fc2 weight [K, f]
// (w_mn) or [f, K]) is not stored; with u = [a | b] the saved fc1 | gate output ([M, 2f], any 16-byte aligned row
// stride) the epilogue writes dU[:, :f] = d silu(a) b / da and dU[:, f:] = d / db. Values equal gemm() followed by
// swiglu_bwd.
void gemm_swiglu_bwd(const at::Tensor& G, const at::Tensor& W, bool w_mn, const at::Tensor& U, at::Tensor& dU) {
  FYB_RANGE("fyb::gemm_swiglu_bwd");
  check_rows16(G, "gemm_swiglu_bwd: G must be bf16 [M, K] with 16-byte aligned rows");
  check_rows16(W, "gemm_swiglu_bwd: W must be bf16 with 16-byte aligned rows");
  check_rows16(U, "gemm_swiglu_bwd: u must be bf16 [M, 2f] with 16-byte aligned rows");
  check_rows16(dU, "gemm_swiglu_bwd: du must be bf16 [M, 2f] with 16-byte aligned rows");
  const int64_t M = G.size(0), K = G.size(1);
  const int64_t f = w_mn ? W.size(1) : W.size(0);
  FYB_CHECK((w_mn ? W.size(0) : W.size(1)) == K && K > 0, "gemm_swiglu_bwd: inner dimensions differ");
  FYB_CHECK(f % 32 == 0 && U.size(0) == M && U.size(1) == 2 * f && dU.size(0) == M && dU.size(1) == 2 * f,
            "gemm_swiglu_bwd: u / du must be [M, 2f] with f a multiple of 32");
  FYB_CHECK(M < (1ll << 31) && f < (1ll << 30) && K < (1ll << 31), "gemm_swiglu_bwd: dimension too large");
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(G.device());
  const CUtensorMap ta = make_tmap_2d(G.data_ptr(), M, K, G.stride(0), kBM);
  const CUtensorMap tb = w_mn ? make_tmap_2d(W.data_ptr(), K, f, W.stride(0), 64)
                              : make_tmap_2d(W.data_ptr(), f, K, W.stride(0), 128);
  const EpiAux aux{reinterpret_cast<const __nv_bfloat16*>(U.data_ptr()), nullptr, nullptr, U.stride(0),
                   static_cast<int>(f), 0};
  const PairArgs pa{1, nullptr, nullptr, nullptr};
  const int m = static_cast<int>(M), n = static_cast<int>(f), k = static_cast<int>(K);
  if (w_mn)
    launch_pair<256, false, true, kE2SwigluBwd>(ta, tb, dU.data_ptr(), nullptr, m, n, k, dU.stride(0), 0, pa,
                                                cur_stream(), aux);
  else
    launch_pair<256, false, false, kE2SwigluBwd>(ta, tb, dU.data_ptr(), nullptr, m, n, k, dU.stride(0), 0, pa,
                                                 cur_stream(), aux);
}

// C = A @ B^T with the ZeRO parameter all-gather of B fused in (GatherArgs): A [M, K] K-major activations; B a
// contiguous [N, K] weight view of `flat`, this rank's parameter replica, whose rows owned by other ranks are stale;
// peers: int64 [world] device tensor of every rank's replica base address (entry `rank` unused); seg / chunk: the
// owner map (chunk 0: contiguous segments of seg elements). On return B's rows are every owner's current values and
// C = A @ B^T. With cos / sin (the rope tables), the leading rot_cols columns are rotated as in gemm_rope (L: sequence
// length). bn: 256 or 192.
namespace {
GatherArgs make_gather_args(const at::Tensor& A, const at::Tensor& B, const at::Tensor& flat, const at::Tensor& peers,
                            int64_t seg, int64_t chunk, int64_t rank, int64_t num_n, at::Tensor& counters) {
  const int64_t K = A.size(1), N = B.size(0);
  FYB_CHECK(B.is_cuda() && B.scalar_type() == at::kBFloat16 && B.dim() == 2 && B.size(1) == K && B.is_contiguous(),
            "gemm_gather: B must be a contiguous bf16 [N, K] weight");
  FYB_CHECK(flat.is_cuda() && flat.scalar_type() == at::kBFloat16 && flat.is_contiguous(),
            "gemm_gather: flat must be the contiguous bf16 replica");
  const int64_t w_off = (reinterpret_cast<intptr_t>(B.data_ptr()) - reinterpret_cast<intptr_t>(flat.data_ptr())) / 2;
  FYB_CHECK(w_off >= 0 && w_off + N * K <= flat.numel() && w_off % 8 == 0,
            "gemm_gather: B must lie inside flat at a 16-byte aligned element offset");
  FYB_CHECK(reinterpret_cast<uintptr_t>(flat.data_ptr()) % 16 == 0 && K % 8 == 0 && K > 0,
            "gemm_gather: 16-byte aligned replica and K a multiple of 8");
  FYB_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong && peers.is_contiguous() && peers.dim() == 1,
            "gemm_gather: peers must be a device int64 [world] tensor");
  const int64_t world = peers.numel();
  FYB_CHECK(world >= 1 && rank >= 0 && rank < world, "gemm_gather: rank out of range");
  FYB_CHECK(seg > 0 && seg % 8 == 0 && chunk >= 0 && chunk % 8 == 0,
            "gemm_gather: owner map sizes must be multiples of 8 elements");
  FYB_CHECK(flat.numel() <= world * seg, "gemm_gather: flat larger than world x seg");
  counters = at::zeros({num_n}, A.options().dtype(at::kInt));
  return GatherArgs{peers.data_ptr<int64_t>(), reinterpret_cast<__nv_bfloat16*>(flat.data_ptr()), w_off, seg, chunk,
                    counters.data_ptr<int>(), static_cast<int>(world), static_cast<int>(rank)};
}
}  // namespace

// The fc1 | gate projection with the all-gather of its merged weight fused in (gemm_gather) and SwiGLU in the
// epilogue (gemm_swiglu): returns {u, h}.
std::vector<at::Tensor> gemm_gather_swiglu(const at::Tensor& A, const at::Tensor& B, const at::Tensor& flat,
                                           const at::Tensor& peers, int64_t seg, int64_t chunk, int64_t rank) {
  FYB_RANGE("fyb::gemm_gather_swiglu");
  check_rows16(A, "gemm_gather_swiglu: A must be bf16 [M, K] with 16-byte aligned rows");
  const int64_t M = A.size(0), K = A.size(1), N2 = B.size(0);
  FYB_CHECK(B.dim() == 2 && B.size(1) == K && N2 % 64 == 0, "gemm_gather_swiglu: B must be [2f, K], f % 32 == 0");
  FYB_CHECK(M < (1ll << 31) && N2 < (1ll << 31) && K < (1ll << 31), "gemm_gather_swiglu: dimension too large");
  const int64_t f = N2 / 2;
  at::Tensor u = at::empty({M, N2}, A.options());
  at::Tensor h = at::empty({M, f}, A.options());
  c10::cuda::CUDAGuard guard(A.device());
  at::Tensor counters;
  const GatherArgs ga = make_gather_args(A, B, flat, peers, seg, chunk, rank, (f + 127) / 128, counters);
  if (M == 0) return {u, h};
  const CUtensorMap ta = make_tmap_2d(A.data_ptr(), M, K, A.stride(0), kBM);
  const CUtensorMap tb = make_tmap_2d(B.data_ptr(), N2, K, K, 128);
  const EpiAux aux{nullptr, nullptr, reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), f, static_cast<int>(f), 0};
  launch_pair<256, false, false, kE2Swiglu, true>(ta, tb, u.data_ptr(), nullptr, static_cast<int>(M),
                                                  static_cast<int>(N2), static_cast<int>(K), N2, 0,
                                                  PairArgs{1, nullptr, nullptr, nullptr}, cur_stream(), aux, ga);
  return {u, h};
}

void gemm_gather(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, const at::Tensor& flat,
                 const at::Tensor& peers, int64_t seg, int64_t chunk, int64_t rank, int64_t bn,
                 const c10::optional<at::Tensor>& cos_t, const c10::optional<at::Tensor>& sin_t, int64_t L,
                 int64_t rot_cols, const c10::optional<at::Tensor>& residual) {
  FYB_RANGE("fyb::gemm_gather");
  check_rows16(A, "gemm_gather: A must be bf16 [M, K] with 16-byte aligned rows");
  check_rows16(C, "gemm_gather: C must be bf16 [M, N] with 16-byte aligned rows");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  FYB_CHECK(C.size(0) == M && C.size(1) == N, "gemm_gather: output shape mismatch");
  FYB_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm_gather: dimension too large");
  FYB_CHECK(bn == 256 || bn == 192, "gemm_gather: tile width must be 256 or 192");
  const __nv_bfloat16* Rp = nullptr;
  int64_t ldr = 0;
  if (residual.has_value() && residual->defined()) {
    FYB_CHECK(residual->scalar_type() == at::kBFloat16 && residual->dim() == 2 && residual->size(0) == M &&
                  residual->size(1) == N && residual->stride(1) == 1,
              "gemm_gather: residual must be bf16 [M, N] with contiguous rows");
    Rp = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    ldr = residual->stride(0);
  }
  const bool rope = cos_t.has_value() && cos_t->defined();
  if (rope) {
    FYB_CHECK(sin_t.has_value() && sin_t->defined(), "gemm_gather: cos without sin");
    FYB_CHECK(L > 0 && M % L == 0 && rot_cols >= 0 && rot_cols % 128 == 0 && rot_cols <= N,
              "gemm_gather: rope rows / columns");
    for (const at::Tensor* t : {&*cos_t, &*sin_t})
      FYB_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->dim() == 2 &&
                    t->size(0) >= L && t->size(1) == 64 && reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
                "gemm_gather: cos / sin must be contiguous bf16 [>= L, 64]");
  }
  FYB_CHECK(!(rope && Rp != nullptr), "gemm_gather: rope and residual do not combine");
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(A.device());
  at::Tensor counters;
  const GatherArgs ga = make_gather_args(A, B, flat, peers, seg, chunk, rank, (N + bn - 1) / bn, counters);
  const CUtensorMap ta = make_tmap_2d(A.data_ptr(), M, K, A.stride(0), kBM);
  const CUtensorMap tb = make_tmap_2d(B.data_ptr(), N, K, K, static_cast<int>(bn / 2));
  EpiAux aux{};
  if (rope)
    aux = EpiAux{reinterpret_cast<const __nv_bfloat16*>(cos_t->data_ptr()),
                 reinterpret_cast<const __nv_bfloat16*>(sin_t->data_ptr()), nullptr, 0, static_cast<int>(L),
                 static_cast<int>(rot_cols)};
  const PairArgs pa{1, nullptr, nullptr, nullptr};
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  void* Cp = C.data_ptr();
  const int64_t ldc = C.stride(0);
  cudaStream_t st = cur_stream();
  if (bn == 256) {
    if (rope) launch_pair<256, false, false, kE2Rope, true>(ta, tb, Cp, nullptr, m, n, k, ldc, 0, pa, st, aux, ga);
    else if (Rp) launch_pair<256, false, false, kE2Bf16Res, true>(ta, tb, Cp, Rp, m, n, k, ldc, ldr, pa, st, aux, ga);
    else launch_pair<256, false, false, kE2Bf16, true>(ta, tb, Cp, nullptr, m, n, k, ldc, 0, pa, st, aux, ga);
  } else {
    if (rope) launch_pair<192, false, false, kE2Rope, true>(ta, tb, Cp, nullptr, m, n, k, ldc, 0, pa, st, aux, ga);
    else if (Rp) launch_pair<192, false, false, kE2Bf16Res, true>(ta, tb, Cp, Rp, m, n, k, ldc, ldr, pa, st, aux, ga);
    else launch_pair<192, false, false, kE2Bf16, true>(ta, tb, Cp, nullptr, m, n, k, ldc, 0, pa, st, aux, ga);
  }
}

}  // namespace fyb
