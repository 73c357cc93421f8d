// Chunkwise gated retention on tcgen05 (sm_100a): forward with an entering / leaving state, backward, and the
// one-token decode step. Replaces the chunkwise PyTorch + Triton path of the reference
// (yoco/models/decoder/kernel/gate_recurrent.py:10-98 state scan, :172-228 _gr_pre / _gr_post / inner_chunk,
// :253-264 recurrent decode).
//
// Per (batch, head) the sequence is cut into chunks of C = 128 positions. With k~ = k / sqrt(D), the chunk-local
// cumulative log decay gamma_i (reset to 0 before each chunk's first position) and Gamma = gamma of the chunk's last
// position:
//   O_c     = diag(e^gamma) Q_c S_c + tril(Q_c K~_c^T o E_c) V_c,          E_ij = e^(gamma_i - gamma_j)
//   S_{c+1} = e^Gamma S_c + K~_c^T diag(e^(Gamma - gamma)) V_c             (S_0 = entering state or 0)
// Every decay factor is e^(x) with x <= 0, so nothing overflows however negative the gates are, and the chunk-local
// cumsum keeps the exponent differences exact at any sequence length.
//
// Forward = three launches:
//   ret_outer_kernel (one CTA per chunk)   dS_c = K~_c^T diag(e^(Gamma - gamma)) V_c    (one 128^3 MMA, fp32 out)
//   ret_scan_kernel  (per head, 16 slices) S_c in bf16 for every chunk, S_{NC} in fp32 (the leaving state)
//   ret_fwd_kernel   (one CTA per chunk)   O_c: S = Q K^T and O = Q S_c (two MMAs into TMEM), O rows scaled by
//                                          e^gamma in TMEM, P = decayed causal S (bf16, shared memory), O += P V
// Backward = the same outer / scan pair on (Q, dO) in reverse (D_c = dL/dS_c = Q_c^T diag(e^gamma) dO_c +
// e^Gamma D_{c+1}), then ret_bwd_kernel per chunk:
//   S^T = K Q^T, dP^T = V dO^T; dV = diag(w) K~ D_{c+1} + P^T dO; dK = diag(w) V D_{c+1}^T + dS^T Q;
//   dQ = diag(e^gamma) dO S_c^T + dS K~   (w = e^(Gamma - gamma) / sqrt(D), dS = dP o E o tril / sqrt(D))
// with the row scalings applied to the TMEM accumulators between MMAs. The gate gradient needs no recurrence of its
// own: for the global cumsum G, dL/dG_i = dO_i . O_i - v_i . dv_i (+ <dS_out, S_out> at the last position). The
// chunk kernel evaluates it with the diagonal terms (which cancel) left out, from fp32 TMEM values:
// sum_{j<i} P_ij dP_ij + dO_i . O_state_i - sum_{t>i} P_ti dP_ti - v_i . dV_state_i, so strongly decaying gates
// (where the two dot products nearly cancel) keep their precision.
//
// Every wait is bounded (2 s) and records a status word instead of hanging; TMA loads read this GPU's memory only.
#include <ATen/ATen.h>

#include "common/host.h"
#include "common/ptx.cuh"

namespace fyb {
namespace {

constexpr int kD = 128;                  // head dim (Dk = Dv)
constexpr int kC = 128;                  // chunk length (= tile rows)
constexpr int kTile = kC * kD * 2;       // 32 KB bf16 tile: two 64-wide 128B-swizzle atoms, 16 KB apart
constexpr int kOuterThreads = 128;
constexpr int kChunkThreads = 320;       // producer, MMA issuer, 8 row warps
constexpr int kRowWarps = 8;

__device__ __forceinline__ uint32_t swz(int r, int c) {   // byte offset of 16-byte chunk c of row r in a tile
  return static_cast<uint32_t>((c >> 3) * 16384 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}
__device__ __forceinline__ uint64_t kdesc(uint32_t base, int k16) {       // K-major, K = 128 in two atoms
  return sw128_desc(base + (k16 >> 2) * 16384 + (k16 & 3) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t mdesc(uint32_t base, int k16) {       // MN-major, MN = 128 in two atoms
  return sw128_desc(base + k16 * 2048, 16384, 1024);
}

__device__ __forceinline__ void store_row32(uint8_t* tile, int r, int chunk0, const float* v) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4*>(tile + swz(r, chunk0 + j)) =
        make_uint4(pack_bf16(v[8 * j], v[8 * j + 1]), pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                   pack_bf16(v[8 * j + 4], v[8 * j + 5]), pack_bf16(v[8 * j + 6], v[8 * j + 7]));
}

// TMEM row r (lane), 64 fp32 columns from col: multiply by f in place
__device__ __forceinline__ void tmem_scale64(uint32_t taddr, float f) {
#pragma unroll
  for (int c = 0; c < 64; c += 32) {
    uint32_t v[32];
    tmem_ld32(taddr + c, v);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * f);
    tmem_st32(taddr + c, v);
  }
  tmem_st_wait();
}

// TMEM row r, 64 fp32 columns from taddr (feature columns c0..c0+63): multiply by f in place and return the dot
// product of the scaled values with row r, features c0..c0+63, of a bf16 tile in shared memory
__device__ __forceinline__ float tmem_scale64_dot(uint32_t taddr, float f, const uint8_t* tile, int r, int c0) {
  float dot = 0.f;
#pragma unroll
  for (int c = 0; c < 64; c += 32) {
    uint32_t v[32];
    tmem_ld32(taddr + c, v);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 u = *reinterpret_cast<const uint4*>(tile + swz(r, (c0 + c) / 8 + j));
      const uint32_t e[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 x = unpack_bf16(e[i]);
        const float a0 = __uint_as_float(v[8 * j + 2 * i]) * f, a1 = __uint_as_float(v[8 * j + 2 * i + 1]) * f;
        v[8 * j + 2 * i] = __float_as_uint(a0);
        v[8 * j + 2 * i + 1] = __float_as_uint(a1);
        dot = fmaf(a0, x.x, fmaf(a1, x.y, dot));
      }
    }
    tmem_st32(taddr + c, v);
  }
  tmem_st_wait();
  return dot;
}

struct RetParams {
  int B, L, H, NC;
  float scale;                 // 1 / sqrt(D)
  const float* gloc;           // [B, H, L] chunk-local cumsum of the log decays
  int* status;
};

__device__ __forceinline__ float chunk_total(const RetParams& p, int bh, int c) {
  return p.gloc[static_cast<int64_t>(bh) * p.L + min(c * kC + kC - 1, p.L - 1)];
}

// ============================================================================================ outer product per chunk
// out[bh, c] (fp32 [128 x 128], row = feature of X, column = feature of Y) = X_c^T diag(w) Y_c
//   MODE 0: X = K, Y = V,  w_j = e^(Gamma - gamma_j) / sqrt(D)   (the chunk's contribution to the leaving state)
//   MODE 1: X = Q, Y = dO, w_i = e^(gamma_i)                     (the chunk's contribution to dL/dS_c)
// Positions past L have w = 0 (their rows of Y are zeroed, and so are X's, whatever the tile read there).
template <int MODE>
__global__ void __launch_bounds__(kOuterThreads)
    ret_outer_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmY, RetParams p,
                     float* __restrict__ out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sX = smem;
  uint8_t* sY = smem + kTile;
  float* sW = reinterpret_cast<float*>(smem + 2 * kTile);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sW + kC);
  uint64_t* full = bars;
  uint64_t* done = bars + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x / p.NC, c = blockIdx.x % p.NC;
  const int b = bh / p.H, h = bh % p.H;
  const int pos0 = c * kC;
  const int nvalid = min(kC, p.L - pos0);

  if (threadIdx.x == 0) {
    mbar_init(full, 1);
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (threadIdx.x == 0) {
    const int row = b * p.L + pos0;
    mbar_arrive_expect_tx(full, 2 * kTile);
    tma_load_3d(sX, &tmX, full, 0, h, row);
    tma_load_3d(sX + 16384, &tmX, full, 64, h, row);
    tma_load_3d(sY, &tmY, full, 0, h, row);
    tma_load_3d(sY + 16384, &tmY, full, 64, h, row);
  }
  {
    const int r = threadIdx.x;                     // one weight per position of the chunk
    const float* g = p.gloc + static_cast<int64_t>(bh) * p.L + pos0;
    float w = 0.f;
    if (r < nvalid) {
      if (MODE == 0) w = __expf(fminf(g[nvalid - 1] - g[r], 0.f)) * p.scale;
      else w = __expf(fminf(g[r], 0.f));
    }
    sW[r] = w;
  }
  __syncthreads();
  bool ok = mbar_wait(full, 0, nullptr, p.status, 80);
  if (ok) {
    // scale row r of Y by w_r (and zero X's rows past L): warp w owns rows 32w..32w+31; per step 4 rows x 8
    // 16-byte chunks of one atom (512 contiguous bytes, no bank conflicts)
    const int sub = lane >> 3, ch = lane & 7;
#pragma unroll 1
    for (int rr = 0; rr < 32; rr += 4) {
      const int r = warp * 32 + rr + sub;
      const float w = sW[r];
#pragma unroll
      for (int atom = 0; atom < 2; ++atom) {
        uint4* py = reinterpret_cast<uint4*>(sY + atom * 16384 + r * 128 + ch * 16);
        uint4 u = *py;
        uint32_t* e = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = unpack_bf16(e[i]);
          e[i] = pack_bf16(f.x * w, f.y * w);
        }
        *py = u;
        if (r >= nvalid) *reinterpret_cast<uint4*>(sX + atom * 16384 + r * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
      }
    }
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (ok && threadIdx.x == 0) {
    tc_fence_after();
    constexpr uint32_t ID = idesc_bf16(128, 128, true, true);
    const uint32_t aX = smem_u32(sX), aY = smem_u32(sY);
#pragma unroll
    for (int k = 0; k < kC / 16; ++k) umma_bf16(tmem, mdesc(aX, k), mdesc(aY, k), ID, k > 0 ? 1u : 0u);
    umma_commit(done);
  }
  __syncwarp();
  const bool have = ok && mbar_wait(done, 0, nullptr, p.status, 81);
  if (have) tc_fence_after();
  float* orow = out + (static_cast<int64_t>(blockIdx.x) * kD + warp * 32 + lane) * kD;
#pragma unroll 1
  for (int cc = 0; cc < kD; cc += 32) {
    uint32_t v[32];
    if (have) {
      tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + cc, v);
      tmem_ld_wait();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = 0u;
    }
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<float4*>(orow + cc + j) = make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                                              __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// ====================================================================================================== state scan
// Forward (REVERSE = 0): S = state_in or 0; for c = 0..NC-1: states[bh, c] = bf16(S); S = e^Gamma_c S + part[c].
//   state_out (optional) = S.
// Backward (REVERSE = 1): D = dstate_out or 0; for c = NC-1..0: states[bh, c] = bf16(D) (dL/dS_{c+1}, what chunk c
//   needs); D = e^Gamma_c D + part[c]. state_out (optional) = D (= dL/dS_0).
// Grid (B*H, 16): each CTA owns 1024 of the 16384 state elements, 4 per thread; the next chunk's part is loaded
// before the current one is used.
constexpr int kScanSlices = 16;

template <int REVERSE>
__global__ void __launch_bounds__(256) ret_scan_kernel(const float* __restrict__ part, RetParams p,
                                                       const float* __restrict__ state_in,
                                                       __nv_bfloat16* __restrict__ states,
                                                       float* __restrict__ state_out) {
  const int bh = blockIdx.x;
  const int e = blockIdx.y * 1024 + threadIdx.x * 4;
  const int64_t base = static_cast<int64_t>(bh) * p.NC * (kD * kD) + e;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (state_in != nullptr) s = *reinterpret_cast<const float4*>(state_in + static_cast<int64_t>(bh) * kD * kD + e);
  const int first = REVERSE ? p.NC - 1 : 0;
  const int step = REVERSE ? -1 : 1;
  float4 nxt = *reinterpret_cast<const float4*>(part + base + static_cast<int64_t>(first) * kD * kD);
  for (int i = 0; i < p.NC; ++i) {
    const int c = first + step * i;
    const float4 cur = nxt;
    if (i + 1 < p.NC) nxt = *reinterpret_cast<const float4*>(part + base + static_cast<int64_t>(c + step) * kD * kD);
    *reinterpret_cast<uint2*>(states + base + static_cast<int64_t>(c) * kD * kD) =
        make_uint2(pack_bf16(s.x, s.y), pack_bf16(s.z, s.w));
    const float f = __expf(fminf(chunk_total(p, bh, c), 0.f));
    s = make_float4(fmaf(s.x, f, cur.x), fmaf(s.y, f, cur.y), fmaf(s.z, f, cur.z), fmaf(s.w, f, cur.w));
  }
  if (state_out != nullptr) *reinterpret_cast<float4*>(state_out + static_cast<int64_t>(bh) * kD * kD + e) = s;
}

// ================================================================================================ forward per chunk
struct FwdArgs {
  __nv_bfloat16* O;            // [B, L, H, D] contiguous
  int has_state0;              // chunk 0 has an entering state
};

__global__ void __launch_bounds__(kChunkThreads, 1)
    ret_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmS, RetParams p,
                   FwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kTile;
  uint8_t* sV = sK + kTile;
  uint8_t* sS = sV + kTile;
  uint8_t* sP = sS + kTile;
  float* sG = reinterpret_cast<float*>(sP + kTile);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sG + kC);
  uint64_t* qk_full = bars + 0;
  uint64_t* vs_full = bars + 1;
  uint64_t* s_full = bars + 2;
  uint64_t* os_full = bars + 3;
  uint64_t* p_full = bars + 4;     // kRowWarps arrivals
  uint64_t* o_full = bars + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x / p.NC, c = blockIdx.x % p.NC;
  const int b = bh / p.H, h = bh % p.H;
  const int pos0 = c * kC;
  const int nvalid = min(kC, p.L - pos0);
  const bool has_state = c > 0 || a.has_state0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 6; ++i) mbar_init(&bars[i], 1);
    mbar_init(p_full, kRowWarps);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;   // S @ 0, O @ 128

  if (warp == 0) {
    if (lane == 0) {
      const int row = b * p.L + pos0;
      mbar_arrive_expect_tx(qk_full, 2 * kTile);
      tma_load_3d(sQ, &tmQ, qk_full, 0, h, row);
      tma_load_3d(sQ + 16384, &tmQ, qk_full, 64, h, row);
      tma_load_3d(sK, &tmK, qk_full, 0, h, row);
      tma_load_3d(sK + 16384, &tmK, qk_full, 64, h, row);
      mbar_arrive_expect_tx(vs_full, (has_state ? 2 : 1) * kTile);
      tma_load_3d(sV, &tmV, vs_full, 0, h, row);
      tma_load_3d(sV + 16384, &tmV, vs_full, 64, h, row);
      if (has_state) {
        const int srow = (bh * p.NC + c) * kD;
        tma_load_2d(sS, &tmS, vs_full, 0, srow);
        tma_load_2d(sS + 16384, &tmS, vs_full, 64, srow);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16(128, 128, false, false);
      constexpr uint32_t ID_O = idesc_bf16(128, 128, false, true);
      const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV), aS = smem_u32(sS), aP = smem_u32(sP);
      bool ok = mbar_wait(qk_full, 0, abort_flag, p.status, 82);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16(tmem, kdesc(aQ, k), kdesc(aK, k), ID_S, k > 0 ? 1u : 0u);
        umma_commit(s_full);
        ok = mbar_wait(vs_full, 0, abort_flag, p.status, 83);
      }
      if (ok && has_state) {
        tc_fence_after();
        // O = Q S_c: B[n = dv][k = dk] read from S_c stored [dk rows, dv contiguous] (MN-major)
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16(tmem + 128, kdesc(aQ, k), mdesc(aS, k), ID_O, k > 0 ? 1u : 0u);
        umma_commit(os_full);
      }
      if (ok) ok = mbar_wait(p_full, 0, abort_flag, p.status, 84);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_bf16(tmem + 128, kdesc(aP, k), mdesc(aV, k), ID_O, (has_state || k > 0) ? 1u : 0u);
        umma_commit(o_full);
      }
      // drain: loads still in flight after an abort must land before the CTA ends
      if (!ok) {
        mbar_wait(qk_full, 0, nullptr, p.status, 85);
        mbar_wait(vs_full, 0, nullptr, p.status, 86);
      }
    }
  } else {
    // ------------------------------------------------------------------------------------------------- row warps
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;              // query row of the chunk
    const uint32_t trow = static_cast<uint32_t>(quad * 32) << 16;
    const int c0 = half * 64;                    // this thread's key columns of S / P and value columns of O
    const float* g = p.gloc + static_cast<int64_t>(bh) * p.L + pos0;
    if (half == 0) sG[r] = r < nvalid ? g[r] : 0.f;
    named_barrier(1, kRowWarps * 32);
    const float gq = sG[r];
    const bool rowvalid = r < nvalid;
    bool ok = true;
    if (has_state) {
      ok = mbar_wait(os_full, 0, abort_flag, p.status, 87);
      if (ok) {
        tc_fence_after();
        tmem_scale64(tmem + 128 + trow + c0, __expf(fminf(gq, 0.f)));
      }
    }
    if (ok) ok = mbar_wait(s_full, 0, abort_flag, p.status, 88);
    if (ok) {
      tc_fence_after();
      uint32_t va[2][32];
      tmem_ld32(tmem + trow + c0, va[0]);
      tmem_ld32(tmem + trow + c0 + 32, va[1]);
      tmem_ld_wait();
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float pv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int j = c0 + 32 * hh + i;                     // key position in the chunk
          const bool vis = rowvalid && j <= r;                // j <= r < nvalid
          pv[i] = vis ? __uint_as_float(va[hh][i]) * __expf(fminf(gq - sG[j], 0.f)) * p.scale : 0.f;
        }
        store_row32(sP, r, (c0 + 32 * hh) >> 3, pv);
      }
    }
    tc_fence_before();
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(p_full);
    const bool have = ok && mbar_wait(o_full, 0, abort_flag, p.status, 89);
    if (have) tc_fence_after();
    __nv_bfloat16* orow = a.O + ((static_cast<int64_t>(b) * p.L + pos0 + (rowvalid ? r : 0)) * p.H + h) * kD;
#pragma unroll
    for (int cc = c0; cc < c0 + 64; cc += 32) {
      uint32_t v[32];
      if (have) {
        tmem_ld32(tmem + 128 + trow + cc, v);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0u;
      }
      if (rowvalid) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(orow + cc + 8 * j) =
              make_uint4(pack_bf16(__uint_as_float(v[8 * j]), __uint_as_float(v[8 * j + 1])),
                         pack_bf16(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3])),
                         pack_bf16(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5])),
                         pack_bf16(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7])));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// =============================================================================================== backward per chunk
struct BwdArgs {
  __nv_bfloat16* dQ;           // [B, L, H, D] views (token strides ldq / ldk / ldv, head stride D)
  __nv_bfloat16* dK;
  __nv_bfloat16* dV;
  int64_t ldq, ldk, ldv;
  const __nv_bfloat16* rope_cos;   // non-null: dQ and dK leave through the conjugate rotation (q, k were rotated)
  const __nv_bfloat16* rope_sin;   // [L, D/2]
  int has_state0;              // chunk 0 has an entering state (S_0 != 0)
  int has_dlast;               // the last chunk has a leaving-state gradient (D_NC != 0)
  float* dG;                   // optional [B, H, L]: gate gradient w.r.t. the global cumsum
};

__device__ __forceinline__ void store_grad_row(__nv_bfloat16* dst, uint32_t taddr, bool have, bool valid, int pos,
                                               int col0, const __nv_bfloat16* cs, const __nv_bfloat16* sn) {
#pragma unroll
  for (int cc = 0; cc < 64; cc += 32) {
    uint32_t v[32];
    if (have) {
      tmem_ld32(taddr + cc, v);
      tmem_ld_wait();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = 0u;
    }
    if (!valid) continue;
    if (cs != nullptr) {
      // conjugate rotation of the interleaved pairs (2i, 2i+1) at position pos
      const __nv_bfloat16* cp = cs + static_cast<int64_t>(pos) * (kD / 2) + (col0 + cc) / 2;
      const __nv_bfloat16* sp = sn + static_cast<int64_t>(pos) * (kD / 2) + (col0 + cc) / 2;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float c = __bfloat162float(cp[i]), s = __bfloat162float(sp[i]);
        const float x0 = __uint_as_float(v[2 * i]), x1 = __uint_as_float(v[2 * i + 1]);
        v[2 * i] = __float_as_uint(x0 * c + x1 * s);
        v[2 * i + 1] = __float_as_uint(x1 * c - x0 * s);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4*>(dst + col0 + cc + 8 * j) =
          make_uint4(pack_bf16(__uint_as_float(v[8 * j]), __uint_as_float(v[8 * j + 1])),
                     pack_bf16(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3])),
                     pack_bf16(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5])),
                     pack_bf16(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7])));
  }
}

__global__ void __launch_bounds__(kChunkThreads, 1)
    ret_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                   const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmDn, RetParams p,
                   BwdArgs a) {
  // Shared memory: Q, K, V, dO, S_c, D_{c+1}, dS^T (7 tiles). P^T stays in TMEM (bf16 pairs written over the S^T
  // columns), the A operand of dV += P^T dO.
  // TMEM: S^T / P^T @ 0, dP^T / dQ @ 128, dV @ 256, dK @ 384.
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kTile;
  uint8_t* sV = sK + kTile;
  uint8_t* sdO = sV + kTile;
  uint8_t* sS = sdO + kTile;
  uint8_t* sDn = sS + kTile;
  uint8_t* sdST = sDn + kTile;
  float* sG = reinterpret_cast<float*>(sdST + kTile);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sG + kC);
  uint64_t* a_full = bars + 0;     // K, Q
  uint64_t* b_full = bars + 1;     // V, dO
  uint64_t* c_full = bars + 2;     // D_{c+1}, S_c
  uint64_t* s_full = bars + 3;
  uint64_t* dp_full = bars + 4;
  uint64_t* st_full = bars + 5;    // dV / dK state terms
  uint64_t* pt_full = bars + 6;    // kRowWarps: P^T in TMEM, state terms scaled
  uint64_t* dst_full = bars + 7;   // kRowWarps: dS^T in shared memory, dP^T drained
  uint64_t* dqs_full = bars + 8;
  uint64_t* dqs_done = bars + 9;   // kRowWarps: dQ state term scaled
  uint64_t* fin = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x / p.NC, c = blockIdx.x % p.NC;
  const int b = bh / p.H, h = bh % p.H;
  const int pos0 = c * kC;
  const int nvalid = min(kC, p.L - pos0);
  const bool has_state = c > 0 || a.has_state0;          // S_c != 0
  const bool has_dn = c < p.NC - 1 || a.has_dlast;       // D_{c+1} != 0
  constexpr uint32_t ID_KK = idesc_bf16(128, 128, false, false);
  constexpr uint32_t ID_KM = idesc_bf16(128, 128, false, true);
  constexpr uint32_t ID_MM = idesc_bf16(128, 128, true, true);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 11; ++i) mbar_init(&bars[i], 1);
    mbar_init(pt_full, kRowWarps);
    mbar_init(dst_full, kRowWarps);
    mbar_init(dqs_done, kRowWarps);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const int row = b * p.L + pos0;
      mbar_arrive_expect_tx(a_full, 2 * kTile);
      tma_load_3d(sK, &tmK, a_full, 0, h, row);
      tma_load_3d(sK + 16384, &tmK, a_full, 64, h, row);
      tma_load_3d(sQ, &tmQ, a_full, 0, h, row);
      tma_load_3d(sQ + 16384, &tmQ, a_full, 64, h, row);
      mbar_arrive_expect_tx(b_full, 2 * kTile);
      tma_load_3d(sV, &tmV, b_full, 0, h, row);
      tma_load_3d(sV + 16384, &tmV, b_full, 64, h, row);
      tma_load_3d(sdO, &tmdO, b_full, 0, h, row);
      tma_load_3d(sdO + 16384, &tmdO, b_full, 64, h, row);
      const int n_c = (has_dn ? 1 : 0) + (has_state ? 1 : 0);
      if (n_c > 0) {
        const int srow = (bh * p.NC + c) * kD;
        mbar_arrive_expect_tx(c_full, n_c * kTile);
        if (has_dn) {
          tma_load_2d(sDn, &tmDn, c_full, 0, srow);
          tma_load_2d(sDn + 16384, &tmDn, c_full, 64, srow);
        }
        if (has_state) {
          tma_load_2d(sS, &tmS, c_full, 0, srow);
          tma_load_2d(sS + 16384, &tmS, c_full, 64, srow);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV), adO = smem_u32(sdO);
      const uint32_t aS = smem_u32(sS), aDn = smem_u32(sDn), adST = smem_u32(sdST);
      const bool need_c = has_dn || has_state;
      bool ok = mbar_wait(a_full, 0, abort_flag, p.status, 90);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16(tmem + 0, kdesc(aK, k), kdesc(aQ, k), ID_KK, k > 0 ? 1u : 0u);
        umma_commit(s_full);
        ok = mbar_wait(b_full, 0, abort_flag, p.status, 91);
      }
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16(tmem + 128, kdesc(aV, k), kdesc(adO, k), ID_KK, k > 0 ? 1u : 0u);
        umma_commit(dp_full);
      }
      if (ok && need_c) ok = mbar_wait(c_full, 0, abort_flag, p.status, 92);
      if (ok && has_dn) {
        tc_fence_after();
        // dV_state = K D (B[n = dv][k = dk] from D stored [dk rows, dv contiguous]: MN-major);
        // dK_state = V D^T (B[n = dk][k = dv]: K-major view of the same tile)
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16(tmem + 256, kdesc(aK, k), mdesc(aDn, k), ID_KM, k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16(tmem + 384, kdesc(aV, k), kdesc(aDn, k), ID_KK, k > 0 ? 1u : 0u);
        umma_commit(st_full);
      }
      if (ok) ok = mbar_wait(pt_full, 0, abort_flag, p.status, 93);
      if (ok) {
        tc_fence_after();
        // dV += P^T dO, P^T (bf16 pairs) in TMEM: K step k = queries 16k..16k+15 in column half k / 4
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_bf16_ts(tmem + 256, tmem + (k >> 2) * 64 + (k & 3) * 8, mdesc(adO, k), ID_KM,
                       (has_dn || k > 0) ? 1u : 0u);
        ok = mbar_wait(dst_full, 0, abort_flag, p.status, 94);
      }
      if (ok) {
        tc_fence_after();
        // dK += dS^T Q
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_bf16(tmem + 384, kdesc(adST, k), mdesc(aQ, k), ID_KM, (has_dn || k > 0) ? 1u : 0u);
        if (has_state) {
          // dQ_state = dO S_c^T (B[n = dk][k = dv]: K-major view of S_c), scaled by e^gamma per query row next
#pragma unroll
          for (int k = 0; k < 8; ++k) umma_bf16(tmem + 128, kdesc(adO, k), kdesc(aS, k), ID_KK, k > 0 ? 1u : 0u);
          umma_commit(dqs_full);
          ok = mbar_wait(dqs_done, 0, abort_flag, p.status, 95);
          if (ok) tc_fence_after();
        }
      }
      if (ok) {
        // dQ += dS K~ (A = dS: MN-major view of dS^T; B[n = dk][k = key] from K stored [keys, dk]: MN-major)
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_bf16(tmem + 128, mdesc(adST, k), mdesc(aK, k), ID_MM, (has_state || k > 0) ? 1u : 0u);
        umma_commit(fin);
      }
      if (!ok) {
        mbar_wait(a_full, 0, nullptr, p.status, 96);
        mbar_wait(b_full, 0, nullptr, p.status, 97);
        if (need_c) mbar_wait(c_full, 0, nullptr, p.status, 98);
      }
    }
  } else {
    // ------------------------------------------------------------------------------------------------- row warps
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;            // key row (S^T, dP^T, dK, dV) / query row (dQ) of the chunk
    const uint32_t trow = static_cast<uint32_t>(quad * 32) << 16;
    const int c0 = half * 64;                  // this thread's query columns of S^T / dP^T, feature columns else
    const float* g = p.gloc + static_cast<int64_t>(bh) * p.L + pos0;
    if (half == 0) sG[r] = r < nvalid ? g[r] : 0.f;
    named_barrier(1, kRowWarps * 32);
    const bool rowvalid = r < nvalid;
    const float gr = sG[r];
    const float gend = sG[nvalid - 1];
    const float w = rowvalid ? __expf(fminf(gend - gr, 0.f)) * p.scale : 0.f;   // key row's state weight
    // Gate gradient (w.r.t. the global cumsum), without the cancellation of dO.O - v.dv: the diagonal terms
    // P_ii dP_ii cancel exactly, so dG_i = sum_{j<i} P_ij dP_ij + dO_i . O_state_i - sum_{t>i} P_ti dP_ti
    // - v_i . dV_state_i, every term from fp32 TMEM values. Scratch: the D_{c+1} tile, dead once the state MMAs
    // have completed (or never loaded).
    float* qpart = reinterpret_cast<float*>(sDn);         // [4 quads][128 queries]: column sums of M
    float* kpart = qpart + 4 * kC;                         // [2 halves][128 keys]: row sums of M + key state term
    float* qst = kpart + 2 * kC;                           // [2 halves][128 queries]: query state term
    float pk[64];                                          // this thread's fp32 P^T values (key r, 64 queries)
    float kst = 0.f;
    bool ok = mbar_wait(s_full, 0, abort_flag, p.status, 100);
    if (ok) {
      tc_fence_after();
      uint32_t va[2][32];
      tmem_ld32(tmem + trow + c0, va[0]);
      tmem_ld32(tmem + trow + c0 + 32, va[1]);
      tmem_ld_wait();
      uint32_t pp[32];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int q = c0 + 32 * hh + i;                    // query position in the chunk
          const bool vis = rowvalid && q >= r && q < nvalid;
          pk[32 * hh + i] = vis ? __uint_as_float(va[hh][i]) * __expf(fminf(sG[q] - gr, 0.f)) * p.scale : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) pp[16 * hh + i] = pack_bf16(pk[32 * hh + 2 * i], pk[32 * hh + 2 * i + 1]);
      }
      tmem_st32(tmem + trow + c0, pp);           // P^T row r, queries c0..c0+63 -> 32 packed columns at c0
      tmem_st_wait();
    }
    if (ok && has_dn) {
      ok = mbar_wait(st_full, 0, abort_flag, p.status, 101);
      if (ok) {
        tc_fence_after();
        kst = tmem_scale64_dot(tmem + 256 + trow + c0, w, sV, r, c0);      // v_r . dV_state_r (this half)
        tmem_scale64(tmem + 384 + trow + c0, w);
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(pt_full);
    if (ok) ok = mbar_wait(dp_full, 0, abort_flag, p.status, 102);
    float krow = 0.f;
    if (ok) {
      tc_fence_after();
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t da[32];
        tmem_ld32(tmem + 128 + trow + c0 + 32 * hh, da);
        tmem_ld_wait();
        float ds[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int q = c0 + 32 * hh + i;
          const bool vis = rowvalid && q >= r && q < nvalid;
          const float dp = __uint_as_float(da[i]);
          ds[i] = vis ? dp * __expf(fminf(sG[q] - gr, 0.f)) * p.scale : 0.f;
          const float m = q > r ? pk[32 * hh + i] * dp : 0.f;      // strictly causal pairs only
          pk[32 * hh + i] = m;
          krow += m;
        }
        store_row32(sdST, r, (c0 + 32 * hh) >> 3, ds);
      }
    }
    tc_fence_before();
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(dst_full);
    // column sums of M over this warp's 32 key rows: butterfly over the lanes, lane l ends with queries
    // c0 + 2l and c0 + 2l + 1
#pragma unroll
    for (int m = 16, n = 32; m >= 1; m >>= 1, n >>= 1) {
      const bool upper = (lane & m) != 0;
#pragma unroll
      for (int i = 0; i < n; ++i) {
        const float mine = upper ? pk[n + i] : pk[i];
        const float other = upper ? pk[i] : pk[n + i];
        pk[i] = mine + __shfl_xor_sync(0xffffffffu, other, m);
      }
    }
    qpart[quad * kC + c0 + 2 * lane] = pk[0];
    qpart[quad * kC + c0 + 2 * lane + 1] = pk[1];
    kpart[half * kC + r] = krow + kst;
    float qs = 0.f;
    if (has_state) {
      if (ok) ok = mbar_wait(dqs_full, 0, abort_flag, p.status, 103);
      if (ok) {
        tc_fence_after();
        // dQ row r = query r: scale the state term by e^gamma_r; e^gamma_r q_r . (dO_r S_c^T) = dO_r . O_state_r
        qs = tmem_scale64_dot(tmem + 128 + trow + c0, __expf(fminf(gr, 0.f)), sQ, r, c0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dqs_done);
    }
    qst[half * kC + r] = qs;
    named_barrier(2, kRowWarps * 32);
    if (a.dG != nullptr && half == 0 && rowvalid) {
      const float qside = qpart[r] + qpart[kC + r] + qpart[2 * kC + r] + qpart[3 * kC + r] + qst[r] + qst[kC + r];
      a.dG[static_cast<int64_t>(bh) * p.L + pos0 + r] = qside - (kpart[r] + kpart[kC + r]);
    }
    const bool have = ok && mbar_wait(fin, 0, abort_flag, p.status, 104);
    if (have) tc_fence_after();
    const int pos = pos0 + (rowvalid ? r : 0);
    const int64_t tok = static_cast<int64_t>(b) * p.L + pos;
    store_grad_row(a.dQ + tok * a.ldq + h * kD, tmem + 128 + trow + c0, have, rowvalid, pos, c0, a.rope_cos,
                   a.rope_sin);
    store_grad_row(a.dK + tok * a.ldk + h * kD, tmem + 384 + trow + c0, have, rowvalid, pos, c0, a.rope_cos,
                   a.rope_sin);
    store_grad_row(a.dV + tok * a.ldv + h * kD, tmem + 256 + trow + c0, have, rowvalid, pos, c0, nullptr, nullptr);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ====================================================================================================== decode step
// One token per sequence: S = e^g S + (k / sqrt(D))^T v (fp32 state, updated in place), o = q S.
// One CTA per (batch, head); thread t owns value column t % 128 of rows [64 (t / 128), 64 (t / 128) + 64).
__global__ void __launch_bounds__(256) ret_decode_kernel(const __nv_bfloat16* __restrict__ q,
                                                         const __nv_bfloat16* __restrict__ k,
                                                         const __nv_bfloat16* __restrict__ v,
                                                         const float* __restrict__ g, float* __restrict__ state,
                                                         __nv_bfloat16* __restrict__ o, int H, int64_t ldq,
                                                         int64_t ldk, int64_t ldv, int64_t ldo, float scale) {
  __shared__ float sq[kD], sk[kD], part[kD];
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  const int t = threadIdx.x;
  if (t < kD) {
    sq[t] = __bfloat162float(q[b * ldq + h * kD + t]);
    sk[t] = __bfloat162float(k[b * ldk + h * kD + t]) * scale;
  }
  __syncthreads();
  const int col = t & (kD - 1), r0 = (t >> 7) * 64;
  const float vc = __bfloat162float(v[b * ldv + h * kD + col]);
  const float f = __expf(fminf(g[bh], 0.f));
  float* S = state + static_cast<int64_t>(bh) * kD * kD;
  float acc = 0.f;
#pragma unroll 8
  for (int r = r0; r < r0 + 64; ++r) {
    const float s = fmaf(S[r * kD + col], f, sk[r] * vc);
    S[r * kD + col] = s;
    acc = fmaf(sq[r], s, acc);
  }
  if (t >= kD) part[col] = acc;
  __syncthreads();
  if (t < kD) o[b * ldo + h * kD + col] = __float2bfloat16_rn(acc + part[col]);
}

constexpr int kOuterSmem = 2 * kTile + kC * 4 + 64 + 1024;
constexpr int kFwdSmem = 5 * kTile + kC * 4 + 128 + 1024;
constexpr int kBwdSmem = 7 * kTile + kC * 4 + 128 + 1024;
static_assert(kBwdSmem <= 227 * 1024, "retention backward shared memory");

void check_heads(const at::Tensor& t, const char* name, int64_t B, int64_t L, int64_t H) {
  FYB_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 4 && t.size(0) == B && t.size(1) == L &&
                t.size(2) == H && t.size(3) == kD && t.stride(3) == 1 && t.stride(2) == kD,
            std::string(name) + ": bf16 [B, L, H, 128] with head stride 128 expected");
  FYB_CHECK(t.stride(0) == L * t.stride(1) || B == 1, std::string(name) + ": batch stride must be L x token stride");
  FYB_CHECK(t.stride(1) % 8 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
            std::string(name) + ": token stride must be a multiple of 8, base 16-byte aligned");
}

CUtensorMap tmap_tok(const at::Tensor& t) {
  return make_tmap_3d(t.data_ptr(), kD, t.size(2), t.size(0) * t.size(1), t.stride(2), t.stride(1), kC);
}

CUtensorMap tmap_states(const at::Tensor& s) {   // [B*H, NC, 128, 128] bf16 as [rows, 128]
  return make_tmap_2d(s.data_ptr(), s.numel() / kD, kD, kD, kD);
}

template <typename K>
void smem_attr(K kern, int bytes) {
  FYB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

RetParams make_params(int64_t B, int64_t L, int64_t H, const at::Tensor& gloc) {
  FYB_CHECK(gloc.is_cuda() && gloc.scalar_type() == at::kFloat && gloc.is_contiguous() && gloc.dim() == 3 &&
                gloc.size(0) == B && gloc.size(1) == H && gloc.size(2) == L,
            "retention: gloc must be contiguous fp32 [B, H, L] (chunk-local cumsum, chunk 128)");
  FYB_CHECK(B * H * L < (1ll << 31), "retention: problem too large");
  return RetParams{static_cast<int>(B), static_cast<int>(L), static_cast<int>(H),
                   static_cast<int>((L + kC - 1) / kC), static_cast<float>(1.0 / std::sqrt(static_cast<double>(kD))),
                   gloc.data_ptr<float>(), status_ptr()};
}

template <int MODE>
void launch_outer(const at::Tensor& x, const at::Tensor& y, const RetParams& p, at::Tensor& out) {
  static bool init = false;
  if (!init) {
    smem_attr(ret_outer_kernel<MODE>, kOuterSmem);
    init = true;
  }
  const CUtensorMap tx = tmap_tok(x), ty = tmap_tok(y);
  ret_outer_kernel<MODE><<<p.B * p.H * p.NC, kOuterThreads, kOuterSmem, cur_stream()>>>(tx, ty, p,
                                                                                       out.data_ptr<float>());
  check_launch(MODE == 0 ? "retention_chunk_state" : "retention_chunk_dstate");
}

}  // namespace

// -------------------------------------------------------------------------------------------------------- host API

// Chunk-local cumsum of the per-step log decays: gloc[b, h, t] = sum of g over [128 floor(t / 128), t].
// g: fp32 [B, H, L] contiguous.
at::Tensor retention_chunk_cumsum(const at::Tensor& g) {
  FYB_CHECK(g.is_cuda() && g.scalar_type() == at::kFloat && g.is_contiguous() && g.dim() == 3,
            "retention_chunk_cumsum: fp32 [B, H, L] expected");
  const int64_t L = g.size(2);
  const int64_t NC = (L + kC - 1) / kC;
  auto padded = at::constant_pad_nd(g, {0, NC * kC - L});
  return padded.view({g.size(0), g.size(1), NC, kC}).cumsum(-1).view({g.size(0), g.size(1), NC * kC})
      .narrow(2, 0, L).contiguous();
}

// Forward. q, k, v: bf16 [B, L, H, 128] (token-strided views allowed); gloc: chunk-local cumsum [B, H, L];
// state_in: optional fp32 [B, H, 128, 128]. Returns {o [B, L, H, 128], states (bf16 entering state of every chunk,
// needed by the backward), state_out (fp32 [B, H, 128, 128]) or an empty tensor}.
std::vector<at::Tensor> retention_chunk_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                            const at::Tensor& gloc, const c10::optional<at::Tensor>& state_in,
                                            bool want_state) {
  FYB_RANGE("fyb::retention_chunk_fwd");
  const int64_t B = q.size(0), L = q.size(1), H = q.size(2);
  check_heads(q, "q", B, L, H);
  check_heads(k, "k", B, L, H);
  check_heads(v, "v", B, L, H);
  c10::cuda::CUDAGuard guard(q.device());
  auto o = at::empty({B, L, H, kD}, q.options());
  const float* s_in = nullptr;
  if (state_in.has_value() && state_in->defined()) {
    FYB_CHECK(state_in->scalar_type() == at::kFloat && state_in->is_contiguous() && state_in->numel() == B * H * kD * kD,
              "retention_chunk_fwd: state_in must be contiguous fp32 [B, H, 128, 128]");
    s_in = state_in->data_ptr<float>();
  }
  at::Tensor state_out;
  if (want_state) state_out = at::empty({B, H, kD, kD}, q.options().dtype(at::kFloat));
  if (B == 0 || H == 0 || L == 0) {
    if (want_state) {
      if (s_in != nullptr) state_out.copy_(*state_in);
      else state_out.zero_();
    }
    return {o, at::empty({0}, q.options()), state_out};
  }
  const RetParams p = make_params(B, L, H, gloc);
  auto part = at::empty({B * H * p.NC, kD, kD}, q.options().dtype(at::kFloat));
  auto states = at::empty({B * H, p.NC, kD, kD}, q.options());
  launch_outer<0>(k, v, p, part);
  ret_scan_kernel<0><<<dim3(B * H, kScanSlices), 256, 0, cur_stream()>>>(
      part.data_ptr<float>(), p, s_in, reinterpret_cast<__nv_bfloat16*>(states.data_ptr()),
      want_state ? state_out.data_ptr<float>() : nullptr);
  check_launch("retention_chunk_scan");
  static bool init = false;
  if (!init) {
    smem_attr(ret_fwd_kernel, kFwdSmem);
    init = true;
  }
  const CUtensorMap tq = tmap_tok(q), tk = tmap_tok(k), tv = tmap_tok(v), ts = tmap_states(states);
  FwdArgs a{reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), s_in != nullptr ? 1 : 0};
  ret_fwd_kernel<<<B * H * p.NC, kChunkThreads, kFwdSmem, cur_stream()>>>(tq, tk, tv, ts, p, a);
  check_launch("retention_chunk_out");
  return {o, states, state_out};
}

// The leaving state only (no outputs): S_out = e^Gamma_total S_in + sum_j e^(G_last - G_j) k~_j^T v_j.
at::Tensor retention_chunk_state(const at::Tensor& k, const at::Tensor& v, const at::Tensor& gloc,
                                 const c10::optional<at::Tensor>& state_in) {
  FYB_RANGE("fyb::retention_chunk_state");
  const int64_t B = k.size(0), L = k.size(1), H = k.size(2);
  check_heads(k, "k", B, L, H);
  check_heads(v, "v", B, L, H);
  c10::cuda::CUDAGuard guard(k.device());
  const float* s_in = nullptr;
  if (state_in.has_value() && state_in->defined()) {
    FYB_CHECK(state_in->scalar_type() == at::kFloat && state_in->is_contiguous() && state_in->numel() == B * H * kD * kD,
              "retention_chunk_state: state_in must be contiguous fp32 [B, H, 128, 128]");
    s_in = state_in->data_ptr<float>();
  }
  auto state_out = at::empty({B, H, kD, kD}, k.options().dtype(at::kFloat));
  if (B == 0 || H == 0 || L == 0) {
    if (s_in != nullptr) state_out.copy_(*state_in);
    else state_out.zero_();
    return state_out;
  }
  const RetParams p = make_params(B, L, H, gloc);
  auto part = at::empty({B * H * p.NC, kD, kD}, k.options().dtype(at::kFloat));
  auto states = at::empty({B * H, p.NC, kD, kD}, k.options());
  launch_outer<0>(k, v, p, part);
  ret_scan_kernel<0><<<dim3(B * H, kScanSlices), 256, 0, cur_stream()>>>(
      part.data_ptr<float>(), p, s_in, reinterpret_cast<__nv_bfloat16*>(states.data_ptr()),
      state_out.data_ptr<float>());
  check_launch("retention_chunk_scan");
  return state_out;
}

// Backward. dout, q, k, v, gloc, states as in / from the forward; dstate_out: optional fp32 gradient of the leaving
// state; want_dstate_in: also return dL/dS_in. dq / dk / dv: optional output views (bf16 [B, L, H, 128], head
// stride 128). rope tables: dq and dk leave through the conjugate interleaved rotation.
// want_dgate: also return the gate gradient w.r.t. the global cumsum G, dL/dG_i = dO_i . O_i - v_i . dv_i, computed
// inside the chunk kernel from fp32 values with the cancelling diagonal terms left out (plus <dS_out, S_out> at
// the last position when dstate_out is given, which the caller adds). Returns {dq, dk, dv, dstate_in or empty,
// dG [B, H, L] or empty}.
std::vector<at::Tensor> retention_chunk_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                            const at::Tensor& v, const at::Tensor& gloc, const at::Tensor& states,
                                            const c10::optional<at::Tensor>& dstate_out, bool want_dstate_in,
                                            bool has_state_in, const c10::optional<at::Tensor>& dq_out,
                                            const c10::optional<at::Tensor>& dk_out,
                                            const c10::optional<at::Tensor>& dv_out,
                                            const c10::optional<at::Tensor>& rope_cos,
                                            const c10::optional<at::Tensor>& rope_sin, bool want_dgate) {
  FYB_RANGE("fyb::retention_chunk_bwd");
  const int64_t B = q.size(0), L = q.size(1), H = q.size(2);
  check_heads(q, "q", B, L, H);
  check_heads(k, "k", B, L, H);
  check_heads(v, "v", B, L, H);
  check_heads(dout, "dout", B, L, H);
  c10::cuda::CUDAGuard guard(q.device());
  auto view_or_new = [&](const c10::optional<at::Tensor>& t, const char* name) {
    if (t.has_value() && t->defined()) {
      check_heads(*t, name, B, L, H);
      return *t;
    }
    return at::empty({B, L, H, kD}, q.options());
  };
  auto dq = view_or_new(dq_out, "dq"), dk = view_or_new(dk_out, "dk"), dv = view_or_new(dv_out, "dv");
  at::Tensor dstate_in;
  if (want_dstate_in) dstate_in = at::empty({B, H, kD, kD}, q.options().dtype(at::kFloat));
  const float* d_out = nullptr;
  if (dstate_out.has_value() && dstate_out->defined()) {
    FYB_CHECK(dstate_out->scalar_type() == at::kFloat && dstate_out->is_contiguous() &&
                  dstate_out->numel() == B * H * kD * kD,
              "retention_chunk_bwd: dstate_out must be contiguous fp32 [B, H, 128, 128]");
    d_out = dstate_out->data_ptr<float>();
  }
  at::Tensor dg;
  if (want_dgate) dg = at::empty({B, H, L}, q.options().dtype(at::kFloat));
  if (B == 0 || H == 0 || L == 0) {
    if (want_dstate_in) {
      if (d_out != nullptr) dstate_in.copy_(*dstate_out);
      else dstate_in.zero_();
    }
    if (want_dgate) dg.zero_();
    return {dq, dk, dv, dstate_in, dg};
  }
  const RetParams p = make_params(B, L, H, gloc);
  FYB_CHECK(states.scalar_type() == at::kBFloat16 && states.is_contiguous() && states.numel() == B * H * p.NC * kD * kD,
            "retention_chunk_bwd: states must be the forward's bf16 [B*H, NC, 128, 128]");
  const __nv_bfloat16* rc = nullptr;
  const __nv_bfloat16* rs = nullptr;
  if (rope_cos.has_value() && rope_cos->defined()) {
    FYB_CHECK(rope_sin.has_value() && rope_cos->is_contiguous() && rope_sin->is_contiguous() &&
                  rope_cos->size(0) >= L && rope_cos->size(1) == kD / 2,
              "retention_chunk_bwd: rope tables [L, 64] expected");
    rc = reinterpret_cast<const __nv_bfloat16*>(rope_cos->data_ptr());
    rs = reinterpret_cast<const __nv_bfloat16*>(rope_sin->data_ptr());
  }
  auto part = at::empty({B * H * p.NC, kD, kD}, q.options().dtype(at::kFloat));
  auto dnext = at::empty({B * H, p.NC, kD, kD}, q.options());
  launch_outer<1>(q, dout, p, part);
  ret_scan_kernel<1><<<dim3(B * H, kScanSlices), 256, 0, cur_stream()>>>(
      part.data_ptr<float>(), p, d_out, reinterpret_cast<__nv_bfloat16*>(dnext.data_ptr()),
      want_dstate_in ? dstate_in.data_ptr<float>() : nullptr);
  check_launch("retention_chunk_dscan");
  static bool init = false;
  if (!init) {
    smem_attr(ret_bwd_kernel, kBwdSmem);
    init = true;
  }
  const CUtensorMap tq = tmap_tok(q), tk = tmap_tok(k), tv = tmap_tok(v), tdo = tmap_tok(dout);
  const CUtensorMap ts = tmap_states(states), tdn = tmap_states(dnext);
  BwdArgs a{reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dk.data_ptr()),
            reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()), dq.stride(1), dk.stride(1), dv.stride(1), rc, rs,
            has_state_in ? 1 : 0, d_out != nullptr ? 1 : 0, want_dgate ? dg.data_ptr<float>() : nullptr};
  ret_bwd_kernel<<<B * H * p.NC, kChunkThreads, kBwdSmem, cur_stream()>>>(tq, tk, tv, tdo, ts, tdn, p, a);
  check_launch("retention_chunk_grad");
  return {dq, dk, dv, dstate_in, dg};
}

// One decode step for every sequence: q, k, v: bf16 [B, H, 128] (token-major rows: strides [ld, 128, 1]); g: fp32
// [B, H] log decays; state: fp32 [B, H, 128, 128], updated in place. Returns o: bf16 [B, H, 128].
at::Tensor retention_decode(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                            at::Tensor& state) {
  FYB_RANGE("fyb::retention_decode");
  const int64_t B = q.size(0), H = q.size(1);
  for (const at::Tensor* t : {&q, &k, &v})
    FYB_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 3 && t->size(0) == B &&
                  t->size(1) == H && t->size(2) == kD && t->stride(2) == 1 && t->stride(1) == kD,
              "retention_decode: q / k / v must be bf16 [B, H, 128] with head stride 128");
  FYB_CHECK(g.scalar_type() == at::kFloat && g.is_contiguous() && g.numel() == B * H, "retention_decode: g fp32 [B, H]");
  FYB_CHECK(state.scalar_type() == at::kFloat && state.is_contiguous() && state.numel() == B * H * kD * kD,
            "retention_decode: state fp32 [B, H, 128, 128]");
  c10::cuda::CUDAGuard guard(q.device());
  auto o = at::empty({B, H, kD}, q.options());
  if (B * H == 0) return o;
  ret_decode_kernel<<<static_cast<int>(B * H), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), g.data_ptr<float>(), state.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), static_cast<int>(H), q.stride(0), k.stride(0), v.stride(0),
      o.stride(0), static_cast<float>(1.0 / std::sqrt(static_cast<double>(kD))));
  check_launch("retention_decode");
  return o;
}

}  // namespace fyb
