// Persistent tcgen05 GEMM for sm_100a: C[M,N] = sum_k A(m,k) * B(n,k)  (+ R[M,N])
//
// The reference runs every projection through cuBLAS (F.linear: yoco/models/decoder/gate_retention.py:64-72,108,
// feedforward_network.py:31, cross_attention.py:38,45, yoco.py:235,320). Here one kernel family covers the forward
// (A, B both K-major), the input gradient (B MN-major) and the weight gradient (A, B both MN-major) without any
// transposed copies: the MN-major operands are described to the tensor core by the UMMA descriptor's major bit.
//
// CTA = 6 warps, one CTA per SM, persistent over output tiles of 128 x BN:
//   warp 0      : TMA producer (one lane) -- STAGES-deep ring of (A 128x64, B BNx64) bf16 tiles, 128B swizzle
//   warp 1      : TMEM allocator + UMMA issuer (one lane): 4 x tcgen05.mma (M=128, N=BN, K=16) per stage
//   warps 2..5  : epilogue -- tcgen05.ld of the fp32 accumulator, bf16 convert (+ residual), global store
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue of tile i overlaps the MMAs of i+1.
// Each CTA loads its own tiles with plain TMA loads of this GPU's memory (this kernel also runs on operands that other ranks wrote).
#include <ATen/ATen.h>
#include <c10/util/Optional.h>

#include "common/host.h"
#include "common/ptx.cuh"
#include "common/zero_map.cuh"

namespace fyb {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

// kEpiScatter / kEpiScatterRes: the owner-scatter epilogue (OwnerScatter, zero_map.cuh) -- the GEMM fused with the
// ZeRO reduce-scatter: element (row, col) of C has flat index x0 + row * ldc + col in the gradient buffer.
// kEpiBf16Sq / kEpiBf16ResSq: the bf16 store plus the sum of squares of the stored (bf16-rounded) values, one fp32
// partial per (tile, epilogue warp) in sq_part[unit * 4 + warp quadrant] -- the weight gradient's share of the
// gradient norm without a second pass over it (deterministic: no atomics, fixed slots).
enum Epi : int {
  kEpiBf16 = 0, kEpiBf16Res = 1, kEpiF32 = 2, kEpiScatter = 3, kEpiScatterRes = 4, kEpiBf16Sq = 5, kEpiBf16ResSq = 6
};

__host__ __device__ constexpr bool epi_scatter(int e) { return e == kEpiScatter || e == kEpiScatterRes; }
__host__ __device__ constexpr bool epi_res(int e) {
  return e == kEpiBf16Res || e == kEpiScatterRes || e == kEpiBf16ResSq;
}
__host__ __device__ constexpr bool epi_sq(int e) { return e == kEpiBf16Sq || e == kEpiBf16ResSq; }

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;   // barriers + slack for 1024-byte alignment
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  constexpr int GROUP_M = 16;
  const int per_group = GROUP_M * num_n;
  const int g = t / per_group;
  const int first_m = g * GROUP_M;
  const int gm = min(num_m - first_m, GROUP_M);
  const int r = t - g * per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, void* Cv,
                        const __nv_bfloat16* R, int M, int N, int K, int64_t ldc, int64_t ldr, int splits,
                        float* ws, int* status, const OwnerScatter sc, float* sq_part) {
  using S = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_k = (K + BK - 1) / BK;
  // split-K: work unit u = (tile u / splits, K slice u % splits); slices write fp32 partials to ws[slice, M, N]
  const int num_units = num_tiles * splits;
  const int k_chunk = (num_k + splits - 1) / splits;
  // accumulator buffers at a power-of-two column stride (BN = 192 uses columns [0, 192) and [256, 448))
  constexpr uint32_t ACC_STRIDE = BN <= 128 ? 128u : 256u;
  constexpr uint32_t TMEM_COLS = 2 * ACC_STRIDE;
  constexpr uint32_t IDESC = idesc_bf16(BM, BN, A_MN, B_MN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int mb, nb;
        tile_coords(u / splits, num_m, num_n, mb, nb);
        const int kb0 = (u % splits) * k_chunk, kb1 = min(num_k, kb0 + k_chunk);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, status, 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * S::STAGE_BYTES;
          uint8_t* sb = sa + S::A_BYTES;
          mbar_arrive_expect_tx(&full[s], S::STAGE_BYTES);
          if (!A_MN) {
            tma_load_2d(sa, &tmA, &full[s], kb * BK, mb * BM);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(sa + j * 8192, &tmA, &full[s], mb * BM + 64 * j, kb * BK);
          }
          if (!B_MN) {
            tma_load_2d(sb, &tmB, &full[s], kb * BK, nb * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * 8192, &tmB, &full[s], nb * BN + 64 * j, kb * BK);
          }
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // drain: every issued stage must have landed before the CTA may exit
      for (int i = 0; i < STAGES; ++i) {
        mbar_wait(&empty[s], ph ^ 1u, nullptr, status, 11);
        if (++s == STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------------------------------- UMMA issuer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t acc_ph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_ph ^ 1u, abort_flag, status, 2)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc) * ACC_STRIDE;
        const int kb0 = (u % splits) * k_chunk, kb1 = min(num_k, kb0 + k_chunk);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag, status, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + s * S::STAGE_BYTES);
          const uint32_t b0 = a0 + S::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? sw128_desc(a0 + k * 2048, 8192, 1024) : sw128_desc(a0 + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sw128_desc(b0 + k * 2048, 8192, 1024) : sw128_desc(b0 + k * 32, 16, 1024);
            umma_bf16(d, ad, bd, IDESC, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);   // frees the smem stage once these MMAs have read it
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);   // accumulator ready for the epilogue
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1u;
      }
    }
  } else {
    // ---------------------------------------------------------------------------------------- epilogue
    const int q = warp & 3;   // TMEM lane quadrant this warp may access
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
      int mb, nb;
      tile_coords(u / splits, num_m, num_n, mb, nb);
      float* wsl = splits > 1 ? ws + static_cast<int64_t>(u % splits) * M * N : nullptr;
      if (!mbar_wait(&tfull[acc], acc_ph, abort_flag, status, 4)) break;
      tc_fence_after();
      float ss = 0.f;                       // sum of squares of this thread's stored values (epi_sq)
      const int row = mb * BM + q * 32 + lane;
      const uint32_t tb = tmem_base + static_cast<uint32_t>(acc) * ACC_STRIDE + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tb + c * 32, r);
        tmem_ld_wait();
        const int col = nb * BN + c * 32;
        if (row < M && col < N && wsl != nullptr) {
          float* W = wsl + static_cast<int64_t>(row) * N + col;
          if (col + 32 <= N && (N % 4) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(W + j) = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                              __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col + j < N) W[j] = __uint_as_float(r[j]);
          }
        } else if (row < M && col < N) {
          if (EPI == kEpiF32) {
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
          } else {
            __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(Cv) + static_cast<int64_t>(row) * ldc + col;
            uint32_t p[16];
            if (epi_res(EPI)) {
              const __nv_bfloat16* Rr = R + static_cast<int64_t>(row) * ldr + col;
              if (col + 32 <= N && (ldr % 8) == 0) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint4 rv = *reinterpret_cast<const uint4*>(Rr + 8 * j);
                  const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                  for (int h = 0; h < 4; ++h) {
                    const float2 res = unpack_bf16(rw[h]);
                    const int e = 8 * j + 2 * h;
                    p[4 * j + h] = pack_bf16(bf16_round(__uint_as_float(r[e])) + res.x,
                                             bf16_round(__uint_as_float(r[e + 1])) + res.y);
                  }
                }
              } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const int e = 2 * j;
                  const float r0 = col + e < N ? __bfloat162float(Rr[e]) : 0.f;
                  const float r1 = col + e + 1 < N ? __bfloat162float(Rr[e + 1]) : 0.f;
                  p[j] = pack_bf16(bf16_round(__uint_as_float(r[e])) + r0, bf16_round(__uint_as_float(r[e + 1])) + r1);
                }
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) p[j] = pack_bf16(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
            }
            if (epi_sq(EPI)) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float2 f = unpack_bf16(p[j]);
                if (col + 2 * j < N) ss += f.x * f.x;
                if (col + 2 * j + 1 < N) ss += f.y * f.y;
              }
            }
            if (epi_scatter(EPI)) {
              const int64_t x = sc.x0 + static_cast<int64_t>(row) * ldc + col;
              if (col + 32 <= N) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  if (__nv_bfloat16* d = owner_dst(sc, x + 8 * j))
                    *reinterpret_cast<uint4*>(d) = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  if (col + j < N) {
                    const uint16_t h = (j & 1) ? static_cast<uint16_t>(p[j >> 1] >> 16)
                                               : static_cast<uint16_t>(p[j >> 1] & 0xffffu);
                    if (__nv_bfloat16* d = owner_dst(sc, x + j)) *d = __ushort_as_bfloat16(h);
                  }
                }
              }
            } else if (col + 32 <= N && (ldc % 8) == 0) {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                *reinterpret_cast<uint4*>(C + 8 * j) = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (col + j < N) {
                  const uint16_t h = (j & 1) ? static_cast<uint16_t>(p[j >> 1] >> 16)
                                             : static_cast<uint16_t>(p[j >> 1] & 0xffffu);
                  C[j] = __ushort_as_bfloat16(h);
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (epi_sq(EPI) && wsl == nullptr) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) sq_part[static_cast<int64_t>(u) * 4 + q] = ss;
      }
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// C = sum over slices of ws[slice] (+ R), fp32 sum in slice order
template <int EPI>
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, void* Cv, const __nv_bfloat16* R,
                                     int M, int N, int64_t ldc, int64_t ldr, const OwnerScatter sc) {
  const int64_t i4 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  const int64_t total = static_cast<int64_t>(M) * N;
  if (i4 >= total) return;
  if ((N % 4) == 0 && (ldc % 4) == 0 && (R == nullptr || (ldr % 4) == 0)) {
    // 4 consecutive columns of one row
    float4 acc = *reinterpret_cast<const float4*>(ws + i4);
    for (int sp = 1; sp < splits; ++sp) {
      const float4 v = *reinterpret_cast<const float4*>(ws + sp * total + i4);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    const int64_t row = i4 / N, col = i4 % N;
    if (EPI == kEpiF32) {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(Cv) + row * ldc + col) = acc;
    } else {
      if (epi_res(EPI)) {
        const uint2 ru = *reinterpret_cast<const uint2*>(R + row * ldr + col);
        const float2 r0 = unpack_bf16(ru.x), r1 = unpack_bf16(ru.y);
        acc = make_float4(bf16_round(acc.x) + r0.x, bf16_round(acc.y) + r0.y, bf16_round(acc.z) + r1.x,
                          bf16_round(acc.w) + r1.y);
      }
      __nv_bfloat16* dst = epi_scatter(EPI) ? owner_dst(sc, sc.x0 + row * ldc + col)
                                            : reinterpret_cast<__nv_bfloat16*>(Cv) + row * ldc + col;
      if (dst != nullptr) *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16(acc.x, acc.y), pack_bf16(acc.z, acc.w));
    }
    return;
  }
  for (int64_t i = i4; i < i4 + 4 && i < total; ++i) {
    float acc = 0.f;
    for (int sp = 0; sp < splits; ++sp) acc += ws[sp * total + i];
    const int64_t row = i / N, col = i % N;
    if (EPI == kEpiF32) {
      reinterpret_cast<float*>(Cv)[row * ldc + col] = acc;
    } else {
      const float v = epi_res(EPI) ? bf16_round(acc) + __bfloat162float(R[row * ldr + col]) : acc;
      __nv_bfloat16* dst = epi_scatter(EPI) ? owner_dst(sc, sc.x0 + row * ldc + col)
                                            : reinterpret_cast<__nv_bfloat16*>(Cv) + row * ldc + col;
      if (dst != nullptr) *dst = __float2bfloat16_rn(v);
    }
  }
}

// split-K reduction for the bf16 outputs with the sum of squares of the stored values: one partial per block in
// sq_part[blockIdx.x] (every block writes its slot; no early exit before the block reduction)
template <bool RES>
__global__ void splitk_reduce_sq_kernel(const float* __restrict__ ws, int splits, void* Cv, const __nv_bfloat16* R,
                                        int M, int N, int64_t ldc, int64_t ldr, float* __restrict__ sq_part) {
  const int64_t i4 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  const int64_t total = static_cast<int64_t>(M) * N;
  float ss = 0.f;
  if (i4 < total) {
    for (int64_t i = i4; i < i4 + 4 && i < total; ++i) {
      float acc = 0.f;
      for (int sp = 0; sp < splits; ++sp) acc += ws[sp * total + i];
      const int64_t row = i / N, col = i % N;
      const float v = RES ? bf16_round(acc) + __bfloat162float(R[row * ldr + col]) : acc;
      const __nv_bfloat16 o = __float2bfloat16_rn(v);
      reinterpret_cast<__nv_bfloat16*>(Cv)[row * ldc + col] = o;
      const float f = __bfloat162float(o);
      ss += f * f;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    sq_part[blockIdx.x] = t;
  }
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, void* C, const __nv_bfloat16* R, int M, int N, int K,
            int64_t ldc, int64_t ldr, int splits, float* ws, cudaStream_t stream,
            const OwnerScatter& sc = OwnerScatter{}, float* sq_part = nullptr) {
  using S = GemmSmem<BN, STAGES>;
  auto kern = gemm_tcgen05_kernel<BN, STAGES, A_MN, B_MN, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    FYB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL));
    attr_set = true;
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN) * splits;
  const int grid = std::min(tiles, num_sms());
  kern<<<grid, kThreads, S::TOTAL, stream>>>(ta, tb, C, R, M, N, K, ldc, ldr, splits, ws, status_ptr(), sc, sq_part);
  check_launch("gemm_tcgen05");
  if (splits > 1) {
    const int64_t total = static_cast<int64_t>(M) * N;
    const int blocks = static_cast<int>((total / 4 + 255) / 256 + 1);
    if constexpr (epi_sq(EPI)) {
      splitk_reduce_sq_kernel<epi_res(EPI)><<<blocks, 256, 0, stream>>>(ws, splits, C, R, M, N, ldc, ldr, sq_part);
    } else {
      splitk_reduce_kernel<EPI><<<blocks, 256, 0, stream>>>(ws, splits, C, R, M, N, ldc, ldr, sc);
    }
    check_launch("gemm_splitk_reduce");
  }
}

// partial-sum slots a gemm_sq call writes: one per (tile, epilogue warp), or one per split-K reduction block
int64_t sq_slots(int M, int N, int bn, int splits) {
  if (splits > 1) return (static_cast<int64_t>(M) * N / 4 + 255) / 256 + 1;
  return static_cast<int64_t>((M + BM - 1) / BM) * ((N + bn - 1) / bn) * 4;
}

template <int BN, int STAGES, int EPI>
void dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, void* C,
                    const __nv_bfloat16* R, int M, int N, int K, int64_t ldc, int64_t ldr, int sp, float* ws,
                    cudaStream_t st) {
  if (!a_mn && !b_mn) launch<BN, STAGES, false, false, EPI>(ta, tb, C, R, M, N, K, ldc, ldr, sp, ws, st);
  else if (!a_mn && b_mn) launch<BN, STAGES, false, true, EPI>(ta, tb, C, R, M, N, K, ldc, ldr, sp, ws, st);
  else if (a_mn && b_mn) launch<BN, STAGES, true, true, EPI>(ta, tb, C, R, M, N, K, ldc, ldr, sp, ws, st);
  else launch<BN, STAGES, true, false, EPI>(ta, tb, C, R, M, N, K, ldc, ldr, sp, ws, st);
}

struct Plan {
  int bn, splits;
  double cost;
};

// Tile width and split-K factor: minimise (waves x per-unit work) + the fp32 split reduction, in tile-k-block
// units. A unit of a BN-wide tile over kc k-blocks costs ~ BN * kc (narrower tiles a little more per column: more
// operand traffic per FLOP); the last partial wave costs a full wave. The 192-wide tile exists for the 3,072-wide
// outputs at M = 2,048: 16 x 16 = 256 tiles fill two waves of 148 SMs, where 256-wide tiles leave the second wave
// 30 % full.
Plan pick_plan(int M, int N, int K) {
  const int sms = num_sms();
  const int tm = (M + BM - 1) / BM;
  const int nk = (K + BK - 1) / BK;
  Plan best{256, 1, 1e30};
  // three or more K slices only where the tiles alone leave most SMs idle or K dwarfs the output (measured: on the
  // 3,072-wide outputs at M = 2,048 the fp32 partials of a 3-way split cost more than its balance gains)
  const long tiles256 = static_cast<long>(tm) * ((N + 255) / 256);
  const bool deep_split = 2 * tiles256 < sms || static_cast<long>(K) > 8l * std::max(M, N);
  for (int bn : {256, 192, 128}) {
    const long tiles = static_cast<long>(tm) * ((N + bn - 1) / bn);
    for (int sp : {1, 2, 3, 4, 6, 8}) {
      if (sp > 1 && nk / sp < 8) break;                  // keep at least 8 k-blocks per slice
      if (sp > 2 && !deep_split) break;
      const long units = tiles * sp;
      const long waves = (units + sms - 1) / sms;
      const int kc = (nk + sp - 1) / sp;
      const double width = bn == 256 ? 1.0 : (bn == 192 ? 1.10 : 1.25);
      double cost = static_cast<double>(waves) * bn * kc * width;
      // fp32 partials written and re-read once: ~ M*N*(sp+1)*4 bytes at HBM speed, in the same units
      // (one BN=256 k-block of one SM ~ 512 tensor cycles ~ 2 units per cycle)
      if (sp > 1) cost += static_cast<double>(M) * N * (sp + 1) * 6.0e-4;
      if (cost < best.cost * 0.97) best = Plan{bn, sp, cost};
    }
  }
  return best;
}

}  // namespace

// Kernel choice for C[M, N] = A B^T with K-deep products: {kernel (0 = one-CTA, 1 = CTA pair), tile width, splits}, by the
// cost model of pick_plan (waves x tile width x K blocks) for both kernels. Measured on the YOCO-3B shapes (one
// B200): the pair kernel with 256-wide tiles where they fill the rounds well (QKVG, fc1 / gate forward, fc2's input
// gradient, the output projection's forward, the weight gradients); the one-CTA kernel with 192-wide tiles for the
// 3,072-wide outputs at M = 2,048 (256 tiles in two waves of 148 SMs, where 256-wide ones leave the second wave 30 %
// full); the output projection's input gradient (K = 100,288) on the one-CTA kernel's split-K plan. The pair
// kernel's 192-wide tiles and its two-way split-K are not routed to: both measured slower on these shapes.
std::vector<int64_t> gemm_route(int64_t M, int64_t N, int64_t K) {
  const Plan one = pick_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K));
  static const bool pair_off = [] {
    const char* e = std::getenv("FYB_GEMM_PAIR");
    return e != nullptr && e[0] == '0';
  }();
  if (pair_off) return {0, one.bn, one.splits};          // FYB_GEMM_PAIR=0: the one-CTA kernel everywhere
  // a K several times longer than the output needs the one-CTA kernel's split-K (no pair plan comes close)
  if (one.splits > 2) return {0, one.bn, one.splits};
  // the pair kernel's 256 x 256 tile = two one-CTA 128 x 256 tiles per round of clusters, at ~0.90 of the one-CTA
  // kernel's time per unit (measured on the YOCO-3B shapes: half the B operand traffic per SM)
  const int64_t clusters = std::max(1, num_sms() / 2);
  const int64_t nk = (K + BK - 1) / BK;
  int64_t best_bn = 0;
  double best = one.cost;
  {
    const int64_t bn = 256;        // the pair kernel's 192-wide tiles measured slower than the one-CTA kernel's
    const int64_t tiles = ((M + 255) / 256) * ((N + bn - 1) / bn);
    const double cost = static_cast<double>((tiles + clusters - 1) / clusters) * bn * nk * 0.90;
    if (cost < best) {
      best = cost;
      best_bn = bn;
    }
  }
  // long-K shapes whose 256 x 256 tiles leave the last round poorly filled: the pair kernel's in-kernel two-way
  // split-K (each half publishes fp32 rows, the later one adds and stores) measured ahead of every other plan once a
  // K half has at least 128 blocks (fc1 / gate input gradient, K = 16,384: 0.170 vs 0.186 ms)
  {
    const int64_t tiles = ((M + 255) / 256) * ((N + 255) / 256);
    const int64_t r1 = (tiles + clusters - 1) / clusters, r2 = (2 * tiles + clusters - 1) / clusters;
    if (nk >= 256 && 2 * r1 > r2 && tiles <= 16384) {
      const double cost = static_cast<double>(r2) * 256.0 * (nk / 2) * 0.90 * 1.05;
      if (cost < best) return {1, 256, 2};
    }
  }
  if (best_bn == 0) return {0, one.bn, one.splits};
  return {1, best_bn, 1};
}

// C = A @ B^T in the operand conventions above. C: bf16 or fp32 [M, N] (any row stride); R: optional bf16 residual.
void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool a_mn, bool b_mn,
          const c10::optional<at::Tensor>& R) {
  FYB_RANGE("fyb::gemm");
  FYB_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm: CUDA tensors expected");
  FYB_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm: bf16 operands expected");
  FYB_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm: 2-D tensors expected");
  FYB_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm: last dimension must be contiguous");
  const int64_t M = a_mn ? A.size(1) : A.size(0);
  const int64_t K = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0);
  const int64_t Kb = b_mn ? B.size(0) : B.size(1);
  FYB_CHECK(K == Kb, "gemm: inner dimensions differ");
  FYB_CHECK(C.size(0) == M && C.size(1) == N, "gemm: output shape mismatch");
  FYB_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm: dimension too large");
  const bool f32 = C.scalar_type() == at::kFloat;
  FYB_CHECK(f32 || C.scalar_type() == at::kBFloat16, "gemm: output must be bf16 or fp32");
  const __nv_bfloat16* Rp = nullptr;
  int64_t ldr = 0;
  if (R.has_value() && R->defined()) {
    FYB_CHECK(!f32, "gemm: residual needs a bf16 output");
    FYB_CHECK(R->scalar_type() == at::kBFloat16 && R->dim() == 2 && R->size(0) == M && R->size(1) == N &&
                  R->stride(1) == 1,
              "gemm: residual must be bf16 [M, N] with contiguous rows");
    Rp = reinterpret_cast<const __nv_bfloat16*>(R->data_ptr());
    ldr = R->stride(0);
  }
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(A.device());
  cudaStream_t st = cur_stream();
  if (K == 0) {
    if (Rp != nullptr) C.copy_(*R);
    else C.zero_();
    return;
  }
  const Plan plan = pick_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K));
  const int bn = plan.bn;
  at::Tensor ws;
  float* wsp = nullptr;
  if (plan.splits > 1) {
    ws = at::empty({plan.splits, M, N}, A.options().dtype(at::kFloat));
    wsp = ws.data_ptr<float>();
  }
  const int sp = plan.splits;
  const CUtensorMap ta = a_mn ? make_tmap_2d(A.data_ptr(), K, M, A.stride(0), 64)
                              : make_tmap_2d(A.data_ptr(), M, K, A.stride(0), BM);
  const CUtensorMap tb = b_mn ? make_tmap_2d(B.data_ptr(), K, N, B.stride(0), 64)
                              : make_tmap_2d(B.data_ptr(), N, K, B.stride(0), bn);
  void* Cp = C.data_ptr();
  const int epi = f32 ? kEpiF32 : (Rp != nullptr ? kEpiBf16Res : kEpiBf16);
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  const int64_t ldc = C.stride(0);
  if (bn == 256) {
    if (epi == kEpiBf16) dispatch_major<256, 4, kEpiBf16>(a_mn, b_mn, ta, tb, Cp, Rp, m, n, k, ldc, ldr, sp, wsp, st);
    else if (epi == kEpiBf16Res)
      dispatch_major<256, 4, kEpiBf16Res>(a_mn, b_mn, ta, tb, Cp, Rp, m, n, k, ldc, ldr, sp, wsp, st);
    else dispatch_major<256, 4, kEpiF32>(a_mn, b_mn, ta, tb, Cp, Rp, m, n, k, ldc, ldr, sp, wsp, st);
  } else if (bn == 192) {
    if (epi == kEpiBf16) dispatch_major<192, 5, kEpiBf16>(a_mn, b_mn, ta, tb, Cp, Rp, m, n, k, ldc, ldr, sp, wsp, st);
    else if (epi == kEpiBf16Res)
      dispatch_major<192, 5, kEpiBf16Res>(a_mn, b_mn, ta, tb, Cp, Rp, m, n, k, ldc, ldr, sp, wsp, st);
    else dispatch_major<192, 5, kEpiF32>(a_mn, b_mn, ta, tb, Cp, Rp, m, n, k, ldc, ldr, sp, wsp, st);
  } else {
    if (epi == kEpiBf16) dispatch_major<128, 6, kEpiBf16>(a_mn, b_mn, ta, tb, Cp, Rp, m, n, k, ldc, ldr, sp, wsp, st);
    else if (epi == kEpiBf16Res)
      dispatch_major<128, 6, kEpiBf16Res>(a_mn, b_mn, ta, tb, Cp, Rp, m, n, k, ldc, ldr, sp, wsp, st);
    else dispatch_major<128, 6, kEpiF32>(a_mn, b_mn, ta, tb, Cp, Rp, m, n, k, ldc, ldr, sp, wsp, st);
  }
}

// Weight gradient fused with the ZeRO reduce-scatter: dW = A^T B (A = dy [T, M], B = x [T, N], both MN-major) with
// every element stored where its owner sums it (OwnerScatter above). C is dW's slot inside grad_flat (only its
// position is used: C's own memory receives the rows this rank owns); with `accumulate`, C's current contents (the
// earlier micro-batches of the update, held locally) are added first, as the residual. bases: int64 [world] device
// tensor of every rank's staging buffer address (this rank's entry is not read).
void gemm_scatter(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool accumulate, const at::Tensor& grad_flat,
                  const at::Tensor& bases, int64_t seg, int64_t rank, int64_t chunk) {
  FYB_RANGE("fyb::gemm_scatter");
  FYB_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda() && bases.is_cuda(), "gemm_scatter: CUDA tensors expected");
  FYB_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 &&
                C.scalar_type() == at::kBFloat16 && grad_flat.scalar_type() == at::kBFloat16,
            "gemm_scatter: bf16 tensors expected");
  FYB_CHECK(bases.scalar_type() == at::kLong && bases.dim() == 1 && rank >= 0 && rank < bases.size(0),
            "gemm_scatter: bases must be int64 [world]");
  FYB_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1 && C.is_contiguous(),
            "gemm_scatter: 2-D operands with contiguous rows and a contiguous output expected");
  const int64_t K = A.size(0), M = A.size(1), N = B.size(1);
  FYB_CHECK(B.size(0) == K && C.size(0) == M && C.size(1) == N, "gemm_scatter: shape mismatch");
  FYB_CHECK(K > 0 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm_scatter: bad dimensions");
  const auto base = reinterpret_cast<uintptr_t>(grad_flat.data_ptr());
  const auto cptr = reinterpret_cast<uintptr_t>(C.data_ptr());
  FYB_CHECK(cptr >= base && cptr + C.numel() * 2 <= base + grad_flat.numel() * 2,
            "gemm_scatter: C must be a slot of grad_flat");
  const int64_t x0 = static_cast<int64_t>((cptr - base) / 2);
  FYB_CHECK(seg > 0 && seg % 8 == 0 && chunk % 8 == 0 && x0 % 8 == 0 && N % 8 == 0,
            "gemm_scatter: segment size, chunk, slot offset and row length must be multiples of 8 elements");
  FYB_CHECK(x0 + C.numel() <= bases.size(0) * seg, "gemm_scatter: slot beyond the last owner");
  FYB_CHECK(chunk == 0 || seg % chunk == 0, "gemm_scatter: the segment must hold whole chunks");
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(A.device());
  cudaStream_t st = cur_stream();
  OwnerScatter sc;
  sc.bases = reinterpret_cast<const unsigned long long*>(bases.data_ptr<int64_t>());
  sc.own = reinterpret_cast<__nv_bfloat16*>(grad_flat.data_ptr());
  sc.x0 = x0;
  sc.seg = seg;
  sc.chunk = chunk;
  sc.rank = static_cast<int>(rank);
  sc.world = static_cast<int>(bases.size(0));
  const Plan plan = pick_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K));
  at::Tensor ws;
  float* wsp = nullptr;
  if (plan.splits > 1) {
    ws = at::empty({plan.splits, M, N}, A.options().dtype(at::kFloat));
    wsp = ws.data_ptr<float>();
  }
  const CUtensorMap ta = make_tmap_2d(A.data_ptr(), K, M, A.stride(0), 64);
  const CUtensorMap tb = make_tmap_2d(B.data_ptr(), K, N, B.stride(0), 64);
  void* Cp = C.data_ptr();
  const __nv_bfloat16* Rp = accumulate ? reinterpret_cast<const __nv_bfloat16*>(Cp) : nullptr;
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  const int64_t ld = N;
  if (plan.bn == 256) {
    if (accumulate) launch<256, 4, true, true, kEpiScatterRes>(ta, tb, Cp, Rp, m, n, k, ld, ld, plan.splits, wsp, st, sc);
    else launch<256, 4, true, true, kEpiScatter>(ta, tb, Cp, Rp, m, n, k, ld, ld, plan.splits, wsp, st, sc);
  } else if (plan.bn == 192) {
    if (accumulate) launch<192, 5, true, true, kEpiScatterRes>(ta, tb, Cp, Rp, m, n, k, ld, ld, plan.splits, wsp, st, sc);
    else launch<192, 5, true, true, kEpiScatter>(ta, tb, Cp, Rp, m, n, k, ld, ld, plan.splits, wsp, st, sc);
  } else {
    if (accumulate) launch<128, 6, true, true, kEpiScatterRes>(ta, tb, Cp, Rp, m, n, k, ld, ld, plan.splits, wsp, st, sc);
    else launch<128, 6, true, true, kEpiScatter>(ta, tb, Cp, Rp, m, n, k, ld, ld, plan.splits, wsp, st, sc);
  }
}

// Weight gradient (both operands MN-major: dW = A^T B) stored as bf16 into C (optionally + C's current contents,
// the earlier micro-batches) with the sum of squares of the stored values as fp32 partials in sq_part: one per
// (tile, epilogue warp), or one per split-K reduction block. Returns the number of partials written (the first
// entries of sq_part; the caller sums them). sq_part must hold at least gemm_sq_slots(...) floats.
int64_t gemm_pair_sq_slots(int64_t M, int64_t N);
int64_t gemm_pair_sq(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool accumulate, at::Tensor& sq_part);

int64_t gemm_sq_slots(int64_t M, int64_t N, int64_t K) {
  if (gemm_route(M, N, K)[0] == 1) return gemm_pair_sq_slots(M, N);
  const Plan plan = pick_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K));
  return sq_slots(static_cast<int>(M), static_cast<int>(N), plan.bn, plan.splits);
}

int64_t gemm_sq(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool accumulate, at::Tensor& sq_part) {
  FYB_RANGE("fyb::gemm_sq");
  FYB_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda() && sq_part.is_cuda(), "gemm_sq: CUDA tensors expected");
  FYB_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 && C.scalar_type() == at::kBFloat16,
            "gemm_sq: bf16 tensors expected");
  FYB_CHECK(sq_part.scalar_type() == at::kFloat && sq_part.is_contiguous(), "gemm_sq: fp32 partials expected");
  FYB_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1,
            "gemm_sq: 2-D operands with contiguous rows expected");
  const int64_t K = A.size(0), M = A.size(1), N = B.size(1);
  FYB_CHECK(B.size(0) == K && C.size(0) == M && C.size(1) == N && K > 0, "gemm_sq: shape mismatch");
  FYB_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm_sq: dimension too large");
  // the shapes the cost model gives to the CTA-pair kernel run there (its epilogue writes every partial slot)
  if (gemm_route(M, N, K)[0] == 1) return gemm_pair_sq(A, B, C, accumulate, sq_part);
  const Plan plan = pick_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K));
  const int64_t slots = sq_slots(static_cast<int>(M), static_cast<int>(N), plan.bn, plan.splits);
  FYB_CHECK(sq_part.numel() >= slots, "gemm_sq: partials buffer too small");
  if (M == 0 || N == 0) return 0;
  c10::cuda::CUDAGuard guard(A.device());
  cudaStream_t st = cur_stream();
  FYB_CUDA(cudaMemsetAsync(sq_part.data_ptr(), 0, slots * sizeof(float), st));
  at::Tensor ws;
  float* wsp = nullptr;
  if (plan.splits > 1) {
    ws = at::empty({plan.splits, M, N}, A.options().dtype(at::kFloat));
    wsp = ws.data_ptr<float>();
  }
  const CUtensorMap ta = make_tmap_2d(A.data_ptr(), K, M, A.stride(0), 64);
  const CUtensorMap tb = make_tmap_2d(B.data_ptr(), K, N, B.stride(0), 64);
  void* Cp = C.data_ptr();
  const __nv_bfloat16* Rp = accumulate ? reinterpret_cast<const __nv_bfloat16*>(Cp) : nullptr;
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  const int64_t ldc = C.stride(0);
  float* sp = sq_part.data_ptr<float>();
  if (plan.bn == 256) {
    if (accumulate) launch<256, 4, true, true, kEpiBf16ResSq>(ta, tb, Cp, Rp, m, n, k, ldc, ldc, plan.splits, wsp, st,
                                                              OwnerScatter{}, sp);
    else launch<256, 4, true, true, kEpiBf16Sq>(ta, tb, Cp, Rp, m, n, k, ldc, ldc, plan.splits, wsp, st,
                                                OwnerScatter{}, sp);
  } else if (plan.bn == 192) {
    if (accumulate) launch<192, 5, true, true, kEpiBf16ResSq>(ta, tb, Cp, Rp, m, n, k, ldc, ldc, plan.splits, wsp, st,
                                                              OwnerScatter{}, sp);
    else launch<192, 5, true, true, kEpiBf16Sq>(ta, tb, Cp, Rp, m, n, k, ldc, ldc, plan.splits, wsp, st,
                                                OwnerScatter{}, sp);
  } else {
    if (accumulate) launch<128, 6, true, true, kEpiBf16ResSq>(ta, tb, Cp, Rp, m, n, k, ldc, ldc, plan.splits, wsp, st,
                                                              OwnerScatter{}, sp);
    else launch<128, 6, true, true, kEpiBf16Sq>(ta, tb, Cp, Rp, m, n, k, ldc, ldc, plan.splits, wsp, st,
                                                OwnerScatter{}, sp);
  }
  return slots;
}

FYB_BOUNDS_BINDER(bind_bounds_gemm)

}  // namespace fyb
