// Tiled attention on tcgen05 for sm_100a: causal / sliding-window softmax attention with GQA (the cross-decoder
// and the sliding-window self-decoder: flash_attn_func in yoco/models/decoder/cross_attention.py:42 and
// sliding_window_attention.py:65) and the parallel form of gated retention (gate_recurrent.py:266-276).
//
// One kernel family, two score transforms:
//   kSoftmax   : P = softmax(scale * Q K^T), online max with lazy rescaling: P is formed against a reference max
//                m_ref and O (in TMEM) and the row sum are rescaled only when the row max exceeds m_ref by more
//                than 2^8, so the common tile needs no O round trip
//   kRetention : P = (scale * Q K^T) * exp(G_q - G_k) (G = fp32 cumsum of the per-step log decays), causal. For a
//                key tile entirely before the query tile the decay factors into exp(G_q - G_e) * exp(G_e - G_k)
//                (G_e = last key of the tile; both factors <= 1): one exp per row plus a per-key column factor
//                staged in shared memory. Diagonal tiles use the exact per-element exp.
//
// Forward CTA (10 warps) = one (batch, head, 128-query tile):
//   warp 0     producer: Q once, K/V tiles (128 keys x 128 dims, 128B swizzle) in a 2-stage TMA ring, and the
//              retention gate tiles (G_k, column factors) into shared memory
//   warp 1     UMMA issuer: S = Q K^T into one of two TMEM S buffers; O += P V into one TMEM O accumulator, P
//              read from TMEM (A operand)
//   warps 2..9 two threads per query row (TMEM lane quadrant = warp % 4, column half = (warp - 2) / 4): read S
//              (tcgen05.ld), mask, exponentiate, write P as bf16 pairs into one of two TMEM P buffers (tcgen05.st),
//              so the softmax of tile j + 1 overlaps the PV MMA of tile j
//
// Backward CTA = one (batch, kv head, 128-key tile) looping over the query tiles that see this key tile, for ONE
// query head of the GQA group (fp32 dK / dV partial per head, summed in head order by a post pass) or,
// without GQA, for the head itself (dK / dV leave straight from TMEM). Per query tile: S^T = K Q^T and
// dP^T = V dO^T (TMEM); P^T goes back into the S^T columns as bf16 pairs and is the TMEM A operand of
// dV += P^T dO; dS^T (bf16, shared memory) feeds dK += dS^T Q and dQ_tile = dS K (TMEM, in the dP^T columns ->
// bulk tensor reductions into an fp32 dQ accumulator, staged per warp in the dS^T tile the dQ MMA has finished
// reading). The UMMA descriptors read the same swizzled dS^T tile as K-major (for dK)
// and as MN-major (for dQ). Q / dO are double-buffered, so the next tile's TMA load and S^T overlap this tile's
// dQ drain. The per-query values (lse and delta, or the gates) are staged in shared memory by the producer warp.
//
// Retention gate gradient, from dG_i = sum_j dP_ij P_ij - sum_k dP_ki P_ki:  dG_i = dO_i . O_i - V_i . dV_i
// (the two sums collapse into row dot products), computed by the small post kernel.
#include <ATen/ATen.h>

#include "common/host.h"
#include "common/ptx.cuh"

namespace fyb {
namespace {

constexpr int kD = 128;      // head dim
constexpr int kT = 128;      // tile rows (queries / keys)
constexpr int kTileBytes = kT * kD * 2;   // 32 KB: two 16 KB swizzle-atom columns (dims 0-63, 64-127)
constexpr int kAttnThreads = 320;         // producer, MMA issuer, 8 score warps
constexpr int kCompute = 8;               // score warps (mbarrier arrival count)
enum Mode : int { kSoftmax = 0, kRetention = 1 };

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;      // lazy rescale threshold (factor 256)

struct AttnParams {
  int B, Lq, Lk, Hq, Hk;
  int q_offset;          // absolute position of query 0 minus position of key 0 (causal alignment)
  int window;            // 0 = unlimited
  int causal;
  float scale;
  __nv_bfloat16* O;      // [B, Lq, Hq, D] contiguous
  float* lse;            // [B, Hq, Lq] (softmax)
  const float* gcum;     // [B, H, L] (retention)
  int* status;
};

// row r, 16-byte chunk c (0..15 over 128 bf16 values) of a [128 x 128] bf16 tile stored as two SW128 K-major atoms
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return static_cast<uint32_t>((c >> 3) * 16384 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// descriptors for a 128-wide K dimension split in two 64-wide swizzle atoms (K-major)
__device__ __forceinline__ uint64_t kmaj_desc(uint32_t base, int k16) {
  return sw128_desc(base + (k16 >> 2) * 16384 + (k16 & 3) * 32, 16, 1024);
}
// MN-major operand whose 128 MN values sit in two 64-wide atoms 16 KB apart; K advances 16 rows per step
__device__ __forceinline__ uint64_t mnmaj_desc(uint32_t base, int k16) {
  return sw128_desc(base + k16 * 2048, 16384, 1024);
}

struct Range {
  int j0, j1;
};

__device__ __forceinline__ Range kv_range(const AttnParams& p, int q0) {
  const int qa_lo = q0 + p.q_offset;
  const int qa_hi = min(q0 + kT, p.Lq) - 1 + p.q_offset;
  int kend = p.Lk;
  if (p.causal) kend = min(kend, qa_hi + 1);
  int kbeg = 0;
  if (p.window > 0) kbeg = max(0, qa_lo - p.window + 1);
  Range r;
  r.j0 = kbeg / kT;
  r.j1 = kend <= 0 ? r.j0 : (kend + kT - 1) / kT;
  if (r.j1 < r.j0) r.j1 = r.j0;
  return r;
}

template <typename P>
__device__ __forceinline__ bool key_valid(const P& p, int qa, int k) {
  if (k >= p.Lk) return false;
  if (p.causal && k > qa) return false;
  if (p.window > 0 && k <= qa - p.window) return false;
  return true;
}

// bit i set when key kbase + i is visible from absolute query position qa (causal / window / key-count bounds)
template <typename P>
__device__ __forceinline__ uint32_t key_mask32(const P& p, int qa, int kbase, bool rowvalid) {
  if (!rowvalid) return 0u;
  int hi = p.Lk - kbase;                                    // exclusive upper bound (relative)
  if (p.causal) hi = min(hi, qa + 1 - kbase);
  int lo = 0;
  if (p.window > 0) lo = max(0, qa - p.window + 1 - kbase);
  hi = min(max(hi, 0), 32);
  lo = min(lo, 32);
  if (hi <= lo) return 0u;
  const uint32_t up = hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u);
  const uint32_t dn = lo >= 32 ? 0xffffffffu : ((1u << lo) - 1u);
  return up & ~dn;
}

__device__ __forceinline__ void store_row8(uint8_t* tile, int r, int chunk0, const float* v) {
  // 32 consecutive values of row r starting at 16-byte chunk chunk0 -> 4 swizzled 16-byte stores
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4*>(tile + sw_off(r, chunk0 + j)) =
        make_uint4(pack_bf16(v[8 * j], v[8 * j + 1]), pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                   pack_bf16(v[8 * j + 4], v[8 * j + 5]), pack_bf16(v[8 * j + 6], v[8 * j + 7]));
}

// ======================================================================================================== forward

template <int MODE>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kTileBytes;             // 2 stages
  uint8_t* sV = sK + 2 * kTileBytes;         // 2 stages
  float* sG = reinterpret_cast<float*>(sV + 2 * kTileBytes);   // [2][128] key gates (retention)
  float* sCF = sG + 2 * kT;                                 // [2][128] column factors exp(G_e - G_k)
  float* sL = sCF + 2 * kT;                                 // [2][128] row-sum halves (softmax)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sL + 2 * kT);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [2]
  uint64_t* s_empty = bars + 11;  // [2]  (kCompute arrivals)
  uint64_t* p_full = bars + 13;   //      (kCompute arrivals)
  uint64_t* p_empty = bars + 14;
  uint64_t* o_full = bars + 15;
  uint64_t* g_full = bars + 16;   // [2]
  uint64_t* g_empty = bars + 18;  // [2]  (kCompute arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (p.Lq + kT - 1) / kT;
  // longest-first over the whole grid: every (batch, head) gets its last (heaviest causal) query tile before any
  // CTA starts a lighter tile, so the block scheduler packs the tail with short tiles
  const int units = p.B * p.Hq;
  const int qt = nq - 1 - static_cast<int>(blockIdx.x / units);
  const int bh = static_cast<int>(blockIdx.x % units);
  const int h = bh % p.Hq, b = bh / p.Hq;
  const int hk = h / (p.Hq / p.Hk);
  const int q0 = qt * kT;
  const Range rg = kv_range(p, q0);
  const int n = rg.j1 - rg.j0;
  const float* gbase = MODE == kRetention ? p.gcum + (static_cast<int64_t>(b) * p.Hq + h) * p.Lq : nullptr;
  constexpr uint32_t IDESC_S = idesc_bf16(128, 128, false, false);
  constexpr uint32_t IDESC_O = idesc_bf16(128, 128, false, true);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 20; ++i) mbar_init(&bars[i], 1);
    mbar_init(&s_empty[0], kCompute);
    mbar_init(&s_empty[1], kCompute);
    mbar_init(p_full, kCompute);
    mbar_init(&g_empty[0], kCompute);
    mbar_init(&g_empty[1], kCompute);
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
  // S[0] @ col 0, S[1] @ 128, O @ 256, P[0] @ 384, P[1] @ 448 (P: bf16 pairs, 64 columns per 128 keys)
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------------------------------------- producer
    if (n > 0) {
      if (lane == 0) {
        const int rowq = b * p.Lq + q0;
        mbar_arrive_expect_tx(q_full, kTileBytes);
        tma_load_3d(sQ, &tmQ, q_full, 0, h, rowq);
        tma_load_3d(sQ + 16384, &tmQ, q_full, 64, h, rowq);
      }
      for (int it = 0; it < n; ++it) {
        const int st = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        const int k0 = (rg.j0 + it) * kT;
        int ok = 1;
        if (lane == 0) {
          const int rowk = b * p.Lk + k0;
          ok = mbar_wait(&k_empty[st], ph ^ 1u, abort_flag, p.status, 20);
          if (ok) {
            mbar_arrive_expect_tx(&k_full[st], kTileBytes);
            tma_load_3d(sK + st * kTileBytes, &tmK, &k_full[st], 0, hk, rowk);
            tma_load_3d(sK + st * kTileBytes + 16384, &tmK, &k_full[st], 64, hk, rowk);
            ok = mbar_wait(&v_empty[st], ph ^ 1u, abort_flag, p.status, 21);
          }
          if (ok) {
            mbar_arrive_expect_tx(&v_full[st], kTileBytes);
            tma_load_3d(sV + st * kTileBytes, &tmV, &v_full[st], 0, hk, rowk);
            tma_load_3d(sV + st * kTileBytes + 16384, &tmV, &v_full[st], 64, hk, rowk);
          }
          if (ok && MODE == kRetention) ok = mbar_wait(&g_empty[st], ph ^ 1u, abort_flag, p.status, 22);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (MODE == kRetention) {
          const float ge = gbase[min(k0 + kT, p.Lk) - 1];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = lane * 4 + j;
            const int kk = k0 + c;
            const float g = kk < p.Lk ? gbase[kk] : 0.f;
            sG[st * kT + c] = g;
            sCF[st * kT + c] = kk < p.Lk ? __expf(ge - g) : 0.f;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&g_full[st]);
        }
      }
      if (lane == 0) {   // drain the ring before exit
        for (int it = n; it < n + 2; ++it) {
          const int st = it & 1;
          const uint32_t ph = (it >> 1) & 1;
          mbar_wait(&k_empty[st], ph ^ 1u, nullptr, p.status, 23);
          mbar_wait(&v_empty[st], ph ^ 1u, nullptr, p.status, 24);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------------------------------------- UMMA issuer
    if (lane == 0 && n > 0) {
      const uint32_t aQ = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, 25);
      auto issue_s = [&](int it) -> bool {
        const int st = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (!mbar_wait(&k_full[st], ph, abort_flag, p.status, 26)) return false;
        if (!mbar_wait(&s_empty[st], ph ^ 1u, abort_flag, p.status, 27)) return false;
        tc_fence_after();
        const uint32_t aK = smem_u32(sK + st * kTileBytes);
#pragma unroll
        for (int k = 0; k < kD / 16; ++k)
          umma_bf16(tmem + st * 128, kmaj_desc(aQ, k), kmaj_desc(aK, k), IDESC_S, k > 0 ? 1u : 0u);
        umma_commit(&s_full[st]);
        umma_commit(&k_empty[st]);
        return true;
      };
      auto issue_pv = [&](int it) -> bool {
        const int st = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (!mbar_wait(p_full, it & 1, abort_flag, p.status, 28)) return false;
        if (!mbar_wait(&v_full[st], ph, abort_flag, p.status, 29)) return false;
        tc_fence_after();
        const uint32_t aV = smem_u32(sV + st * kTileBytes);
        // O += P V with P (bf16 pairs) in TMEM: K step k = keys 16k..16k+15 of column half k / 4
#pragma unroll
        for (int k = 0; k < kT / 16; ++k)
          umma_bf16_ts(tmem + 256, tmem + 384 + st * 64 + (k >> 2) * 32 + (k & 3) * 8, mnmaj_desc(aV, k), IDESC_O,
                       (it > 0 || k > 0) ? 1u : 0u);
        umma_commit(p_empty);
        umma_commit(&v_empty[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int it = 0; ok && it < n; ++it) {
        if (it + 1 < n) ok = issue_s(it + 1);
        if (ok) ok = issue_pv(it);
      }
      if (ok) umma_commit(o_full);
    }
  } else {
    // -------------------------------------------------------------------------------------------- score warps
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;                 // query row within the tile
    const int qrow = q0 + r;
    const bool rowvalid = qrow < p.Lq;
    const int qa = qrow + p.q_offset;               // absolute query position
    const uint32_t trow = static_cast<uint32_t>(quad * 32) << 16;
    const int c0 = half * 64;                       // this thread's columns of S / P / O
    const float sl2 = p.scale * kLog2e;
    float m_ref = -INFINITY, l_part = 0.f;
    const float gq = (MODE == kRetention && rowvalid) ? gbase[qrow] : 0.f;
    bool ok = true;
    for (int it = 0; ok && it < n; ++it) {
      const int st = it & 1;
      const uint32_t ph = (it >> 1) & 1;
      const int k0 = (rg.j0 + it) * kT;
      const bool full_tile = rowvalid ? ((k0 + kT <= p.Lk) && (!p.causal || k0 + kT - 1 <= q0 + p.q_offset) &&
                                         (p.window <= 0 || k0 > min(q0 + kT, p.Lq) - 1 + p.q_offset - p.window))
                                      : false;
      if (MODE == kRetention && !(ok = mbar_wait(&g_full[st], ph, abort_flag, p.status, 30))) break;
      if (!(ok = mbar_wait(&s_full[st], ph, abort_flag, p.status, 31))) break;
      tc_fence_after();
      if (MODE == kSoftmax) {
        // full-row max (both threads of the row compute the same value, so their decisions agree)
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < kT; c += 64) {
          uint32_t v[32], w[32];
          tmem_ld32(tmem + st * 128 + trow + c, v);
          tmem_ld32(tmem + st * 128 + trow + c + 32, w);
          tmem_ld_wait();
          const uint32_t mv = full_tile ? 0xffffffffu : key_mask32(p, qa, k0 + c, rowvalid);
          const uint32_t mw = full_tile ? 0xffffffffu : key_mask32(p, qa, k0 + c + 32, rowvalid);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            mx = fmaxf(mx, ((mv >> i) & 1u) ? __uint_as_float(v[i]) : -INFINITY);
            mx = fmaxf(mx, ((mw >> i) & 1u) ? __uint_as_float(w[i]) : -INFINITY);
          }
        }
        const float m_cand = fmaxf(m_ref, mx * sl2);
        const bool need = m_cand > m_ref + kRescaleLog2;
        const bool scale_o = need && m_ref != -INFINITY;
        if (__any_sync(0xffffffffu, scale_o)) {
          // O may be touched only after PV(it-1) has completed. PV(it-2) is complete (S(it), whose commit this
          // thread waited for, was issued after it) and PV(it) is not issued yet, so the parity of phase it - 1
          // names exactly one phase
          if (!(ok = mbar_wait(p_empty, (it & 1) ^ 1u, abort_flag, p.status, 32))) break;
          const float f = scale_o ? fast_exp2(m_ref - m_cand) : 1.0f;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 64; c += 32) {
            uint32_t v[32];
            tmem_ld32(tmem + 256 + trow + c0 + c, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * f);
            tmem_st32(tmem + 256 + trow + c0 + c, v);
          }
          tmem_st_wait();
          if (scale_o) l_part *= f;
        }
        if (need) m_ref = m_cand;
      }
      const bool diag = k0 + kT - 1 >= q0 + p.q_offset;   // retention: tile reaches the query tile
      const float rf = (MODE == kRetention && !diag) ? __expf(gq - sG[st * kT + kT - 1]) * p.scale : 0.f;
      const float mref = m_ref == -INFINITY ? 0.f : m_ref;
      {
        uint32_t va[2][32];
        uint32_t pp[32];
        tmem_ld32(tmem + st * 128 + trow + c0, va[0]);
        tmem_ld32(tmem + st * 128 + trow + c0 + 32, va[1]);
        tmem_ld_wait();
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int c = c0 + 32 * hh;
          const uint32_t m = full_tile ? 0xffffffffu : key_mask32(p, qa, k0 + c, rowvalid);
          float pv[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const bool valid = (m >> i) & 1u;
            float x;
            if (MODE == kSoftmax) {
              x = fast_exp2(__uint_as_float(va[hh][i]) * sl2 - mref);
              x = valid ? x : 0.f;
              l_part += x;
            } else {
              const float decay = diag ? __expf(gq - sG[st * kT + c + i]) * p.scale : rf * sCF[st * kT + c + i];
              x = valid ? __uint_as_float(va[hh][i]) * decay : 0.f;
            }
            pv[i] = x;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) pp[16 * hh + i] = pack_bf16(pv[2 * i], pv[2 * i + 1]);
        }
        // P row r, keys c0..c0+63 -> 32 packed columns of P[st]. PV(it-2), the last reader of P[st], was issued
        // before S(it) and so has completed
        tmem_st32(tmem + 384 + st * 64 + trow + half * 32, pp);
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_empty[st]);
        mbar_arrive(p_full);
        if (MODE == kRetention) mbar_arrive(&g_empty[st]);
      }
    }
    // ---------------------------------------------------------------------------------------------- epilogue
    const bool have = ok && n > 0 && mbar_wait(o_full, 0, abort_flag, p.status, 33);
    if (have) tc_fence_after();
    float inv = 1.f;
    if (MODE == kSoftmax) {
      sL[half * kT + r] = l_part;
      named_barrier(1, kCompute * 32);
      const float l_tot = sL[r] + sL[kT + r];
      inv = l_tot > 0.f ? 1.0f / l_tot : 0.f;
      if (half == 0 && rowvalid)
        p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.Lq + qrow] =
            l_tot > 0.f ? (m_ref + __log2f(l_tot)) * 0.6931471805599453f : -INFINITY;
    }
    __nv_bfloat16* orow = p.O + ((static_cast<int64_t>(b) * p.Lq + (rowvalid ? qrow : 0)) * p.Hq + h) * kD;
#pragma unroll
    for (int c = c0; c < c0 + 64; c += 32) {
      uint32_t v[32];
      if (have) {
        tmem_ld32(tmem + 256 + trow + c, v);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0u;
      }
      if (rowvalid) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(orow + c + 8 * j) =
              make_uint4(pack_bf16(__uint_as_float(v[8 * j]) * inv, __uint_as_float(v[8 * j + 1]) * inv),
                         pack_bf16(__uint_as_float(v[8 * j + 2]) * inv, __uint_as_float(v[8 * j + 3]) * inv),
                         pack_bf16(__uint_as_float(v[8 * j + 4]) * inv, __uint_as_float(v[8 * j + 5]) * inv),
                         pack_bf16(__uint_as_float(v[8 * j + 6]) * inv, __uint_as_float(v[8 * j + 7]) * inv));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ====================================================================================== forward, two CTAs per SM
// Softmax attention forward sized so that two CTAs share an SM (the tensor core works on one CTA's MMAs while the
// other's softmax runs): one query tile per CTA, 6 warps (producer, MMA issuer, 4 softmax warps with one thread per
// query row), single-buffered K / V (96 KB of shared memory), 256 TMEM columns: S @ 0 with P written back over its
// first 64 columns as bf16 pairs (the A operand of O += P V), O @ 128. The next key tile's S MMA is issued after the
// PV MMA that reads P from the same columns (one CTA's MMAs run in issue order). Lazy rescaling as in attn_fwd_kernel.
constexpr int kFwd2Threads = 192;
constexpr int kSoftWarps = 4;

__global__ void __launch_bounds__(kFwd2Threads, 2)
    attn_fwd2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kTileBytes;
  uint8_t* sV = sK + kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 2;
  uint64_t* v_full = bars + 3;
  uint64_t* v_empty = bars + 4;
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 6;    // kSoftWarps arrivals
  uint64_t* pv_done = bars + 7;
  uint64_t* o_full = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (p.Lq + kT - 1) / kT;
  const int units = p.B * p.Hq;
  const int qt = nq - 1 - static_cast<int>(blockIdx.x / units);      // longest first
  const int bh = static_cast<int>(blockIdx.x % units);
  const int h = bh % p.Hq, b = bh / p.Hq;
  const int hk = h / (p.Hq / p.Hk);
  const int q0 = qt * kT;
  const Range rg = kv_range(p, q0);
  const int n = rg.j1 - rg.j0;
  constexpr uint32_t IDESC_S = idesc_bf16(128, 128, false, false);
  constexpr uint32_t IDESC_O = idesc_bf16(128, 128, false, true);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 9; ++i) mbar_init(&bars[i], 1);
    mbar_init(p_full, kSoftWarps);
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
  const uint32_t tmem = *tmem_slot;   // S / P @ 0, O @ 128

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------------ producer
    if (lane == 0 && n > 0) {
      const int rowq = b * p.Lq + q0;
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_3d(sQ, &tmQ, q_full, 0, h, rowq);
      tma_load_3d(sQ + 16384, &tmQ, q_full, 64, h, rowq);
      int issued_k = 0, issued_v = 0;
      for (int it = 0; it < n; ++it) {
        const uint32_t ph = it & 1;
        const int rowk = b * p.Lk + (rg.j0 + it) * kT;
        if (!mbar_wait(k_empty, ph ^ 1u, abort_flag, p.status, 60)) break;
        mbar_arrive_expect_tx(k_full, kTileBytes);
        tma_load_3d(sK, &tmK, k_full, 0, hk, rowk);
        tma_load_3d(sK + 16384, &tmK, k_full, 64, hk, rowk);
        issued_k = it + 1;
        if (!mbar_wait(v_empty, ph ^ 1u, abort_flag, p.status, 61)) break;
        mbar_arrive_expect_tx(v_full, kTileBytes);
        tma_load_3d(sV, &tmV, v_full, 0, hk, rowk);
        tma_load_3d(sV + 16384, &tmV, v_full, 64, hk, rowk);
        issued_v = it + 1;
      }
      // drain: the last loads must have landed before the CTA ends
      if (issued_k > 0) mbar_wait(k_full, (issued_k - 1) & 1, nullptr, p.status, 62);
      if (issued_v > 0) mbar_wait(v_full, (issued_v - 1) & 1, nullptr, p.status, 63);
      mbar_wait(q_full, 0, nullptr, p.status, 64);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------------ MMA issuer
    if (lane == 0 && n > 0) {
      const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, 65);
      for (int it = 0; ok && it < n; ++it) {
        const uint32_t ph = it & 1;
        if (!(ok = mbar_wait(k_full, ph, abort_flag, p.status, 66))) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kD / 16; ++k)
          umma_bf16(tmem, kmaj_desc(aQ, k), kmaj_desc(aK, k), IDESC_S, k > 0 ? 1u : 0u);
        umma_commit(s_full);
        umma_commit(k_empty);
        if (!(ok = mbar_wait(p_full, ph, abort_flag, p.status, 67))) break;
        if (!(ok = mbar_wait(v_full, ph, abort_flag, p.status, 68))) break;
        tc_fence_after();
        // O += P V, P (bf16 pairs) in TMEM columns 0..63: K step k = keys 16k..16k+15 in columns 8k..8k+7
#pragma unroll
        for (int k = 0; k < kT / 16; ++k)
          umma_bf16_ts(tmem + 128, tmem + k * 8, mnmaj_desc(aV, k), IDESC_O, (it > 0 || k > 0) ? 1u : 0u);
        umma_commit(pv_done);
        umma_commit(v_empty);
      }
      if (ok) umma_commit(o_full);
    }
  } else {
    // ------------------------------------------------------------------------------------------ softmax warps
    const int quad = warp & 3;
    const int r = quad * 32 + lane;                 // query row within the tile
    const int qrow = q0 + r;
    const bool rowvalid = qrow < p.Lq;
    const int qa = qrow + p.q_offset;
    const uint32_t trow = static_cast<uint32_t>(quad * 32) << 16;
    const float sl2 = p.scale * kLog2e;
    float m_ref = -INFINITY, l_sum = 0.f;
    bool ok = true;
    for (int it = 0; ok && it < n; ++it) {
      const uint32_t ph = it & 1;
      const int k0 = (rg.j0 + it) * kT;
      const bool full_tile = rowvalid && (k0 + kT <= p.Lk) && (!p.causal || k0 + kT - 1 <= q0 + p.q_offset) &&
                             (p.window <= 0 || k0 > min(q0 + kT, p.Lq) - 1 + p.q_offset - p.window);
      if (!(ok = mbar_wait(s_full, ph, abort_flag, p.status, 69))) break;
      tc_fence_after();
      // row max over the tile (this thread owns the whole row)
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kT; c += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + trow + c, v);
        tmem_ld_wait();
        const uint32_t mk = full_tile ? 0xffffffffu : key_mask32(p, qa, k0 + c, rowvalid);
#pragma unroll
        for (int i = 0; i < 32; ++i) mx = fmaxf(mx, ((mk >> i) & 1u) ? __uint_as_float(v[i]) : -INFINITY);
      }
      const float m_cand = fmaxf(m_ref, mx * sl2);
      const bool need = m_cand > m_ref + kRescaleLog2;
      const bool scale_o = need && m_ref != -INFINITY;
      if (__any_sync(0xffffffffu, scale_o)) {
        // O may be touched only after PV(it-1): PV(it-2) completed before S(it) was issued and PV(it) is not issued
        // yet, so the parity of phase it - 1 names exactly one phase
        if (!(ok = mbar_wait(pv_done, ph ^ 1u, abort_flag, p.status, 70))) break;
        tc_fence_after();
        const float f = scale_o ? fast_exp2(m_ref - m_cand) : 1.0f;
#pragma unroll
        for (int c = 0; c < kD; c += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + 128 + trow + c, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * f);
          tmem_st32(tmem + 128 + trow + c, v);
        }
        tmem_st_wait();
        if (scale_o) l_sum *= f;
      }
      if (need) m_ref = m_cand;
      const float mref = m_ref == -INFINITY ? 0.f : m_ref;
      // P = exp2(S * scale * log2 e - m) as bf16 pairs over S's first 64 columns: the packed chunk of S columns
      // c .. c + 31 lands in columns c / 2 .. c / 2 + 15, all of which this thread has already read
#pragma unroll
      for (int c = 0; c < kT; c += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + trow + c, v);
        tmem_ld_wait();
        const uint32_t mk = full_tile ? 0xffffffffu : key_mask32(p, qa, k0 + c, rowvalid);
        uint32_t pp[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float x0 = fast_exp2(__uint_as_float(v[2 * i]) * sl2 - mref);
          float x1 = fast_exp2(__uint_as_float(v[2 * i + 1]) * sl2 - mref);
          x0 = ((mk >> (2 * i)) & 1u) ? x0 : 0.f;
          x1 = ((mk >> (2 * i + 1)) & 1u) ? x1 : 0.f;
          l_sum += x0 + x1;
          pp[i] = pack_bf16(x0, x1);
        }
        tmem_st16(tmem + trow + c / 2, pp);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // ------------------------------------------------------------------------------------------------ epilogue
    const bool have = ok && n > 0 && mbar_wait(o_full, 0, abort_flag, p.status, 71);
    if (have) tc_fence_after();
    const float inv = l_sum > 0.f ? 1.0f / l_sum : 0.f;
    if (rowvalid)
      p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.Lq + qrow] =
          l_sum > 0.f ? (m_ref + __log2f(l_sum)) * 0.6931471805599453f : -INFINITY;
    __nv_bfloat16* orow = p.O + ((static_cast<int64_t>(b) * p.Lq + (rowvalid ? qrow : 0)) * p.Hq + h) * kD;
#pragma unroll 1
    for (int c = 0; c < kD; c += 32) {
      uint32_t v[32];
      if (have) {
        tmem_ld32(tmem + 128 + trow + c, v);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0u;
      }
      if (rowvalid) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(orow + c + 8 * j) =
              make_uint4(pack_bf16(__uint_as_float(v[8 * j]) * inv, __uint_as_float(v[8 * j + 1]) * inv),
                         pack_bf16(__uint_as_float(v[8 * j + 2]) * inv, __uint_as_float(v[8 * j + 3]) * inv),
                         pack_bf16(__uint_as_float(v[8 * j + 4]) * inv, __uint_as_float(v[8 * j + 5]) * inv),
                         pack_bf16(__uint_as_float(v[8 * j + 6]) * inv, __uint_as_float(v[8 * j + 7]) * inv));
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

// ======================================================================================================= backward

struct AttnBwdParams {
  int B, Lq, Lk, Hq, Hk;
  int q_offset, window, causal;
  float scale;
  const float* lse;      // softmax: [B, Hq, Lq]
  const float* delta;    // softmax: [B, Hq, Lq] rowsum(dO * O)
  const float* gcum;     // retention: [B, H, L]
  float* dq_acc;         // [B, Lq, Hq, D] fp32
  float* dk_acc;         // split mode: [G][B, Lk, Hk, D] fp32 partials, one slice per query head of the group
  float* dv_acc;         //   (summed in head order by the post pass: deterministic)
  int split;             // 1: one CTA per (key tile, query head); 0: a CTA loops over the GQA group's heads
  __nv_bfloat16* dK;     // [B, Lk, Hk, D] view: token stride dk_ld, head stride D
  __nv_bfloat16* dV;     // [B, Lk, Hk, D] view: token stride dv_ld
  int64_t dk_ld, dv_ld;
  const __nv_bfloat16* rope_cos;   // non-null: dK leaves through the conjugate rotation (keys were rotated)
  const __nv_bfloat16* rope_sin;   // [Lk, D/2] tables
  int* status;
};

template <int MODE>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                    const __grid_constant__ CUtensorMap tmdQ, AttnBwdParams p) {
  // Shared memory: K, V (once), Q / dO double-buffered (the next query tile loads while this one computes),
  // dS^T (bf16, read by the dK MMA as K-major and by the dQ MMA as MN-major). P^T never touches shared memory:
  // the score warps store it (bf16 pairs) into the TMEM columns of S^T they have just read, and the dV MMA takes
  // its A operand from there.
  // TMEM: S^T / P^T @ 0, dP^T / dQ @ 128, dV @ 256, dK @ 384.
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + kTileBytes;
  uint8_t* sQ = sV + kTileBytes;            // [2]
  uint8_t* sdO = sQ + 2 * kTileBytes;       // [2]
  uint8_t* sdST = sdO + 2 * kTileBytes;
  float* sQA = reinterpret_cast<float*>(sdST + kTileBytes);   // softmax: lse * log2(e); retention: G_q
  float* sQB = sQA + kT;                                      // softmax: delta; retention: exp(G_q - G_e)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sQB + kT);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;    // [2]
  uint64_t* qdo_empty = bars + 3;   // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* dp_full = bars + 6;
  uint64_t* pt_full = bars + 7;     // kCompute
  uint64_t* dst_full = bars + 8;    // kCompute
  uint64_t* ds_empty = bars + 9;
  uint64_t* dq_full = bars + 10;
  uint64_t* dq_empty = bars + 11;   // kCompute
  uint64_t* fin = bars + 12;
  uint64_t* qv_full = bars + 13;
  uint64_t* qv_empty = bars + 14;   // kCompute
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (p.Lq + kT - 1) / kT;
  const int G = p.Hq / p.Hk;
  const int S = p.split ? G : 1;                     // CTAs per (batch, kv head, key tile)
  const int units = p.B * p.Hk * S;
  // longest-first over the whole grid: under a causal mask the early key tiles see the most query tiles
  const int kt = static_cast<int>(blockIdx.x / units);
  const int unit = static_cast<int>(blockIdx.x % units);
  const int bh = unit / S;
  const int hk = bh % p.Hk, b = bh / p.Hk;
  const int h_first = hk * G + (p.split ? unit % S : 0);
  const int n_heads = p.split ? 1 : G;
  const int k0 = kt * kT;
  const int k_hi = min(k0 + kT, p.Lk) - 1;
  int i_lo = 0, i_hi = nq;
  if (p.causal) i_lo = max(0, k0 - p.q_offset) / kT;
  if (p.window > 0) i_hi = min(nq, max(0, k_hi + p.window - 1 - p.q_offset) / kT + 1);
  const int per_h = max(0, i_hi - i_lo);
  const int n_it = n_heads * per_h;
  constexpr uint32_t ID_KK = idesc_bf16(128, 128, false, false);
  constexpr uint32_t ID_KM = idesc_bf16(128, 128, false, true);
  constexpr uint32_t ID_MM = idesc_bf16(128, 128, true, true);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 15; ++i) mbar_init(&bars[i], 1);
    mbar_init(pt_full, kCompute);
    mbar_init(dst_full, kCompute);
    mbar_init(dq_empty, kCompute);
    mbar_init(qv_empty, kCompute);
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
  const float g_end = (MODE == kRetention) ? p.gcum[(static_cast<int64_t>(b) * p.Hk + hk) * p.Lk + k_hi] : 0.f;

  if (warp == 0) {
    if (n_it > 0) {
      if (lane == 0) {
        const int rowk = b * p.Lk + k0;
        mbar_arrive_expect_tx(kv_full, 2 * kTileBytes);
        tma_load_3d(sK, &tmK, kv_full, 0, hk, rowk);
        tma_load_3d(sK + 16384, &tmK, kv_full, 64, hk, rowk);
        tma_load_3d(sV, &tmV, kv_full, 0, hk, rowk);
        tma_load_3d(sV + 16384, &tmV, kv_full, 64, hk, rowk);
      }
      // iteration it: Q / dO tile of `it` into buffer it & 1, then the per-query values of `it` (single buffer,
      // refilled once the score warps are done with the previous tile's values)
      int it = 0, issued = 0;
      for (; it < n_it; ++it) {
        const int buf = it & 1;
        const int h = h_first + it / per_h;
        const int q0 = (i_lo + it % per_h) * kT;
        const int64_t hq_base = (static_cast<int64_t>(b) * p.Hq + h) * p.Lq;
        int ok = 1;
        if (lane == 0) {
          ok = mbar_wait(&qdo_empty[buf], ((it >> 1) & 1) ^ 1u, abort_flag, p.status, 40);
          if (ok) {
            const int rowq = b * p.Lq + q0;
            uint8_t* q_dst = sQ + buf * kTileBytes;
            uint8_t* do_dst = sdO + buf * kTileBytes;
            mbar_arrive_expect_tx(&qdo_full[buf], 2 * kTileBytes);
            tma_load_3d(q_dst, &tmQ, &qdo_full[buf], 0, h, rowq);
            tma_load_3d(q_dst + 16384, &tmQ, &qdo_full[buf], 64, h, rowq);
            tma_load_3d(do_dst, &tmdO, &qdo_full[buf], 0, h, rowq);
            tma_load_3d(do_dst + 16384, &tmdO, &qdo_full[buf], 64, h, rowq);
            issued = it + 1;
            ok = mbar_wait(qv_empty, (it & 1) ^ 1u, abort_flag, p.status, 41);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = lane * 4 + j;
          const int q = q0 + c;
          if (MODE == kSoftmax) {
            sQA[c] = q < p.Lq ? p.lse[hq_base + q] * kLog2e : INFINITY;
            sQB[c] = q < p.Lq ? p.delta[hq_base + q] : 0.f;
          } else {
            const float g = q < p.Lq ? p.gcum[hq_base + q] : 0.f;
            sQA[c] = g;
            sQB[c] = q < p.Lq ? __expf(fminf(g - g_end, 0.f)) : 0.f;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(qv_full);
      }
      // drain: the last one or two tile loads must have landed before the CTA can end (normally the MMA warp has
      // consumed them already; after an abort they may still be in flight)
      if (lane == 0) {
        for (int j = max(0, issued - 2); j < issued; ++j)
          mbar_wait(&qdo_full[j & 1], (j >> 1) & 1, nullptr, p.status, 42);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_it > 0) {
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), adST = smem_u32(sdST);
      bool ok = mbar_wait(kv_full, 0, abort_flag, p.status, 43);
      for (int it = 0; ok && it < n_it; ++it) {
        const uint32_t ph = it & 1;
        const int buf = it & 1;
        const uint32_t aQ = smem_u32(sQ + buf * kTileBytes), adO = smem_u32(sdO + buf * kTileBytes);
        if (!(ok = mbar_wait(&qdo_full[buf], (it >> 1) & 1, abort_flag, p.status, 44))) break;
        tc_fence_after();
        // S^T = K Q^T: its columns were last read by the score warps for P^T(it - 1), which they finished before
        // arriving at pt_full(it - 1) -- waited for below in the previous iteration
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16(tmem + 0, kmaj_desc(aK, k), kmaj_desc(aQ, k), ID_KK, k > 0);
        umma_commit(s_full);
        // dP^T = V dO^T into the dQ columns: dQ(it - 1) must have been drained
        if (it > 0 && !(ok = mbar_wait(dq_empty, ph ^ 1u, abort_flag, p.status, 45))) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16(tmem + 128, kmaj_desc(aV, k), kmaj_desc(adO, k), ID_KK, k > 0);
        umma_commit(dp_full);
        // dV += P^T dO, P^T (bf16 pairs) in TMEM: K step k = queries 16k..16k+15 of column half k / 4
        if (!(ok = mbar_wait(pt_full, ph, abort_flag, p.status, 46))) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_bf16_ts(tmem + 256, tmem + (k >> 2) * 64 + (k & 3) * 8, mnmaj_desc(adO, k), ID_KM,
                       (it > 0 || k > 0) ? 1u : 0u);
        if (!(ok = mbar_wait(dst_full, ph, abort_flag, p.status, 47))) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_bf16(tmem + 384, kmaj_desc(adST, k), mnmaj_desc(aQ, k), ID_KM, (it > 0 || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16(tmem + 128, mnmaj_desc(adST, k), mnmaj_desc(aK, k), ID_MM, k > 0);
        umma_commit(dq_full);
        umma_commit(&qdo_empty[buf]);
        umma_commit(ds_empty);
      }
      if (ok) umma_commit(fin);
    }
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;          // key row (S^T, dP^T, dK, dV) / query row (dQ) within the tile
    const int kpos = k0 + r;
    const uint32_t trow = static_cast<uint32_t>(quad * 32) << 16;
    const int c0 = half * 64;                // this thread's query columns of S^T / dP^T and d columns of dQ/dK/dV
    const float sl2 = p.scale * kLog2e;
    const float gk = (MODE == kRetention && kpos < p.Lk)
                         ? p.gcum[(static_cast<int64_t>(b) * p.Hk + hk) * p.Lk + kpos] : 0.f;
    const float rfk = (MODE == kRetention && kpos < p.Lk) ? __expf(g_end - gk) * p.scale : 0.f;
    bool ok = true;
    for (int it = 0; ok && it < n_it; ++it) {
      const uint32_t ph = it & 1;
      const int h = h_first + it / per_h;
      const int q0 = (i_lo + it % per_h) * kT;
      const bool full_tile = (q0 + kT <= p.Lq) && (kpos < p.Lk) && (!p.causal || q0 + p.q_offset >= k0 + kT - 1) &&
                             (p.window <= 0 || q0 + kT - 1 + p.q_offset < k0 + p.window);
      const bool offdiag = q0 + p.q_offset > k_hi;
      if (!(ok = mbar_wait(qv_full, ph, abort_flag, p.status, 48))) break;
      if (!(ok = mbar_wait(s_full, ph, abort_flag, p.status, 49))) break;
      tc_fence_after();
      // visibility of this key from the 32-query chunks: query q sees key kpos iff kpos <= qa (causal) and
      // kpos > qa - window, i.e. qa in [kpos, kpos + window - 1]; qa = q + q_offset, q < Lq
      uint32_t qm[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int qb = q0 + c0 + 32 * hh;          // first query of the chunk
        if (full_tile) {
          qm[hh] = 0xffffffffu;
        } else if (kpos >= p.Lk) {
          qm[hh] = 0u;
        } else {
          int lo = 0, hi = min(32, p.Lq - qb);
          if (p.causal) lo = max(lo, kpos - p.q_offset - qb);
          if (p.window > 0) hi = min(hi, kpos + p.window - p.q_offset - qb);
          lo = max(lo, 0);
          hi = min(hi, 32);
          qm[hh] = hi <= lo ? 0u : ((hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u)) & ~(lo >= 32 ? 0xffffffffu : ((1u << lo) - 1u)));
        }
      }
      float pk[64];
      {
        uint32_t va[2][32];
        tmem_ld32(tmem + 0 + trow + c0, va[0]);
        tmem_ld32(tmem + 0 + trow + c0 + 32, va[1]);
        tmem_ld_wait();
        uint32_t pp[32];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int cc = c0 + 32 * hh + i;
            float x;
            if (MODE == kSoftmax) x = fast_exp2(__uint_as_float(va[hh][i]) * sl2 - sQA[cc]);
            else x = __uint_as_float(va[hh][i]) * (offdiag ? rfk * sQB[cc] : __expf(sQA[cc] - gk) * p.scale);
            pk[32 * hh + i] = ((qm[hh] >> i) & 1u) ? x : 0.f;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) pp[16 * hh + i] = pack_bf16(pk[32 * hh + 2 * i], pk[32 * hh + 2 * i + 1]);
        }
        // P^T row r, queries c0..c0+63 -> 32 packed columns starting at this half's first S^T column
        tmem_st32(tmem + 0 + trow + c0, pp);
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pt_full);
      if (!(ok = mbar_wait(dp_full, ph, abort_flag, p.status, 53))) break;
      if (!(ok = mbar_wait(ds_empty, ph ^ 1u, abort_flag, p.status, 50))) break;
      tc_fence_after();
      // this warp's slice of dS^T (rows quad*32.., columns c0..) is the 4 KB block it staged dQ in last iteration:
      // the bulk reduction must have read it
      if (lane == 0) bulk_wait_read0();
      __syncwarp();
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t da[32];
        tmem_ld32(tmem + 128 + trow + c0 + 32 * hh, da);
        tmem_ld_wait();
        float ds[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int cc = c0 + 32 * hh + i;
          float x;
          if (MODE == kSoftmax) {
            x = pk[32 * hh + i] * (__uint_as_float(da[i]) - sQB[cc]) * p.scale;
          } else {
            x = __uint_as_float(da[i]) * (offdiag ? rfk * sQB[cc] : __expf(sQA[cc] - gk) * p.scale);
            x = ((qm[hh] >> i) & 1u) ? x : 0.f;
          }
          ds[i] = x;
        }
        store_row8(sdST, r, (c0 + 32 * hh) >> 3, ds);
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(dst_full);
        mbar_arrive(qv_empty);
      }
      // dQ tile (TMEM lane = query row, columns 128..255) -> fp32 bulk tensor reductions: each warp stages its
      // 32 rows x 32 columns (4 KB, 128-byte swizzle) in its own slice of the dS^T tile, which the dK / dQ MMAs of
      // this iteration have finished reading (dq_full), and one lane reduces it into dq_acc
      if (!(ok = mbar_wait(dq_full, ph, abort_flag, p.status, 51))) break;
      tc_fence_after();
      const int qrow = q0 + r;
      uint8_t* stage = sdST + half * 16384 + quad * 4096;
#pragma unroll
      for (int c = 0; c < 64; c += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + 128 + trow + c0 + c, v);
        tmem_ld_wait();
        if (c > 0) {                        // the first chunk's reduction must have read the staging block
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
        }
        const bool live = qrow < p.Lq;      // rows past Lq belong to the next sequence: add zeros there
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float4*>(stage + lane * 128 + ((j ^ (lane & 7)) << 4)) =
              live ? make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                 __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_3d(&tmdQ, stage, c0 + c, h, b * p.Lq + q0 + quad * 32);
          bulk_commit_group();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_empty);
    }
    // the last dQ reductions complete before the CTA ends (their shared-memory source included)
    if (lane == 0) bulk_wait0();
    __syncwarp();
    // ---- dK, dV
    const bool have = ok && n_it > 0 && mbar_wait(fin, 0, abort_flag, p.status, 52);
    if (have) tc_fence_after();
    const int64_t tok = static_cast<int64_t>(b) * p.Lk + min(kpos, p.Lk - 1);
    if (p.dk_acc != nullptr) {
      // split mode: this query head's share into its fp32 partial slice (rotation applied by the post pass).
      // tcgen05.ld is warp-collective (.sync.aligned): it runs under the warp-uniform `have` only, and the
      // lane-dependent key bound guards the stores
      const int64_t slice = static_cast<int64_t>(h_first - hk * G) * p.B * p.Lk * p.Hk * kD;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        float* acc = (which == 0 ? p.dk_acc : p.dv_acc) + slice + (tok * p.Hk + hk) * kD + c0;
        const uint32_t col = which == 0 ? 384u : 256u;
#pragma unroll
        for (int c = 0; c < 64; c += 32) {
          uint32_t v[32];
          if (have) {
            tmem_ld32(tmem + col + trow + c0 + c, v);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0u;
          }
          if (kpos < p.Lk) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(acc + c + j) =
                  make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                              __uint_as_float(v[j + 3]));
          }
        }
      }
    } else {
#pragma unroll 1
    for (int which = 0; which < 2; ++which) {
      __nv_bfloat16* dst = which == 0 ? p.dK + tok * p.dk_ld + hk * kD + c0 : p.dV + tok * p.dv_ld + hk * kD + c0;
      const uint32_t col = which == 0 ? 384u : 256u;
#pragma unroll
      for (int c = 0; c < 64; c += 32) {
        uint32_t v[32];
        if (have) {
          tmem_ld32(tmem + col + trow + c0 + c, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0u;
        }
        if (which == 0 && p.rope_cos != nullptr && kpos < p.Lk) {
          // conjugate rotation of interleaved pairs (2i, 2i+1) at position kpos
          const __nv_bfloat16* cp = p.rope_cos + static_cast<int64_t>(kpos) * (kD / 2) + (c0 + c) / 2;
          const __nv_bfloat16* sp = p.rope_sin + static_cast<int64_t>(kpos) * (kD / 2) + (c0 + c) / 2;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float cs = __bfloat162float(cp[i]), sn = __bfloat162float(sp[i]);
            const float x0 = __uint_as_float(v[2 * i]), x1 = __uint_as_float(v[2 * i + 1]);
            v[2 * i] = __float_as_uint(x0 * cs + x1 * sn);
            v[2 * i + 1] = __float_as_uint(x1 * cs - x0 * sn);
          }
        }
        if (kpos < p.Lk) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(dst + c + 8 * j) =
                make_uint4(pack_bf16(__uint_as_float(v[8 * j]), __uint_as_float(v[8 * j + 1])),
                           pack_bf16(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3])),
                           pack_bf16(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5])),
                           pack_bf16(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7])));
        }
      }
    }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// rowdot[b, h, t] = sum_d X[b, t, h, d] * Y[b, t, h, d] (fp32); one warp per (b, t, h)
__global__ void rowdot_kernel(const __nv_bfloat16* __restrict__ X, const __nv_bfloat16* __restrict__ Y,
                              float* __restrict__ out, int B, int L, int H, float* __restrict__ sub_from,
                              int64_t ldx = -1, int64_t ldy = -1) {
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= static_cast<int64_t>(B) * L * H) return;
  const int h = static_cast<int>(wid % H);
  const int64_t bt = wid / H;
  const int t = static_cast<int>(bt % L);
  const int b = static_cast<int>(bt / L);
  const int64_t tok = static_cast<int64_t>(b) * L + t;
  const int64_t xo = (ldx < 0 ? wid * kD : tok * ldx + h * kD) + lane * 4;
  const int64_t yo = (ldy < 0 ? wid * kD : tok * ldy + h * kD) + lane * 4;
  const uint2 xu = *reinterpret_cast<const uint2*>(X + xo);
  const uint2 yu = *reinterpret_cast<const uint2*>(Y + yo);
  const float2 x0 = unpack_bf16(xu.x), x1 = unpack_bf16(xu.y), y0 = unpack_bf16(yu.x), y1 = unpack_bf16(yu.y);
  float s = x0.x * y0.x + x0.y * y0.y + x1.x * y1.x + x1.y * y1.y;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    const int64_t idx = (static_cast<int64_t>(b) * H + h) * L + t;
    out[idx] = sub_from != nullptr ? sub_from[idx] - s : s;
  }
}

// out[b, t, h, :] (token stride ld) = bf16(conj_rope(sum_g acc[g][b, t, h, :])), the nparts slices of acc
// (contiguous [B, L, H, D] fp32 each) added in slice order
__global__ void dq_out_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ out, int64_t ld, int B,
                              int L, int H, const __nv_bfloat16* __restrict__ cos_t,
                              const __nv_bfloat16* __restrict__ sin_t, int nparts = 1) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;   // one thread per 4 values
  const int64_t total = static_cast<int64_t>(B) * L * H * (kD / 4);
  if (i >= total) return;
  const int c = static_cast<int>(i % (kD / 4)) * 4;
  const int64_t bth = i / (kD / 4);
  const int h = static_cast<int>(bth % H);
  const int64_t bt = bth / H;
  const int t = static_cast<int>(bt % L);
  float4 v = *reinterpret_cast<const float4*>(acc + bth * kD + c);
  for (int g = 1; g < nparts; ++g) {
    const float4 u = *reinterpret_cast<const float4*>(acc + g * total * 4 + bth * kD + c);
    v = make_float4(v.x + u.x, v.y + u.y, v.z + u.z, v.w + u.w);
  }
  if (cos_t != nullptr) {
    const float c0 = __bfloat162float(cos_t[static_cast<int64_t>(t) * (kD / 2) + c / 2]);
    const float s0 = __bfloat162float(sin_t[static_cast<int64_t>(t) * (kD / 2) + c / 2]);
    const float c1 = __bfloat162float(cos_t[static_cast<int64_t>(t) * (kD / 2) + c / 2 + 1]);
    const float s1 = __bfloat162float(sin_t[static_cast<int64_t>(t) * (kD / 2) + c / 2 + 1]);
    const float x0 = v.x, x1 = v.y, x2 = v.z, x3 = v.w;
    v = make_float4(x0 * c0 + x1 * s0, x1 * c0 - x0 * s0, x2 * c1 + x3 * s1, x3 * c1 - x2 * s1);
  }
  *reinterpret_cast<uint2*>(out + bt * ld + h * kD + c) = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
}

constexpr int kFwdSmem = 5 * kTileBytes + 6 * kT * 4 + 256 + 1024;
constexpr int kFwd2Smem = 3 * kTileBytes + 128 + 1024;
constexpr int kBwdSmem = 7 * kTileBytes + 2 * kT * 4 + 256 + 1024;
static_assert(kBwdSmem <= 227 * 1024, "attention backward shared memory");

void check_qkv(const at::Tensor& t, const char* name) {
  FYB_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 4 && t.size(3) == kD && t.stride(3) == 1,
            std::string(name) + ": bf16 [B, L, H, 128] with contiguous last dim expected");
  FYB_CHECK(t.stride(0) == t.size(1) * t.stride(1) || t.size(0) == 1,
            std::string(name) + ": batch stride must equal L x token stride");
  FYB_CHECK(t.stride(1) % 8 == 0 && t.stride(2) % 8 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
            std::string(name) + ": strides must be multiples of 8 elements, base 16-byte aligned");
}

// dQ accumulator [B, L, H, 128] fp32 (contiguous) as {128, H, B * L} with 32 x 1 x 32 boxes
CUtensorMap tmap_dq(const at::Tensor& acc) {
  return make_tmap_3d_f32(acc.data_ptr(), kD, acc.size(2), acc.size(0) * acc.size(1), kD, acc.size(2) * kD, 32);
}

CUtensorMap tmap_heads(const at::Tensor& t) {
  return make_tmap_3d(t.data_ptr(), kD, t.size(2), t.size(0) * t.size(1), t.stride(2), t.stride(1), kT);
}

template <typename K>
void set_smem(K kern, int bytes) {
  FYB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

}  // namespace

// -------------------------------------------------------------------------------------------------------- host API

std::vector<at::Tensor> attention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, bool causal,
                                      int64_t window, double scale) {
  FYB_RANGE("fyb::attention_fwd");
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  const int B = (int)q.size(0), Lq = (int)q.size(1), Hq = (int)q.size(2), Lk = (int)k.size(1), Hk = (int)k.size(2);
  FYB_CHECK(k.size(0) == B && v.size(0) == B && v.size(1) == Lk && v.size(2) == Hk && Hq % Hk == 0,
            "attention_fwd: shape mismatch");
  c10::cuda::CUDAGuard guard(q.device());
  auto o = at::empty({B, Lq, Hq, kD}, q.options());
  auto lse = at::empty({B, Hq, Lq}, q.options().dtype(at::kFloat));
  if (B == 0 || Lq == 0) return {o, lse};
  AttnParams p{B, Lq, Lk, Hq, Hk, Lk - Lq, (int)window, causal ? 1 : 0, (float)scale,
               reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), lse.data_ptr<float>(), nullptr, status_ptr()};
  const CUtensorMap tq = tmap_heads(q), tk = tmap_heads(k), tv = tmap_heads(v);
  static bool init = false;
  if (!init) {
    set_smem(attn_fwd2_kernel, kFwd2Smem);
    FYB_CUDA(cudaFuncSetAttribute(attn_fwd2_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    init = true;
  }
  const int grid = B * Hq * ((Lq + kT - 1) / kT);
  attn_fwd2_kernel<<<grid, kFwd2Threads, kFwd2Smem, cur_stream()>>>(tq, tk, tv, p);
  check_launch("attn_fwd");
  return {o, lse};
}

at::Tensor out_view(const c10::optional<at::Tensor>& opt, int B, int L, int H, const at::TensorOptions& o,
                    const char* name) {
  if (opt.has_value() && opt->defined()) {
    const at::Tensor& t = *opt;
    FYB_CHECK(t.dim() == 4 && t.size(0) == B && t.size(1) == L && t.size(2) == H && t.size(3) == kD &&
                  t.stride(3) == 1 && t.stride(2) == kD && (t.stride(0) == L * t.stride(1) || B == 1) &&
                  t.stride(1) % 8 == 0 && t.scalar_type() == at::kBFloat16,
              std::string(name) + ": output view must be bf16 [B, L, H, 128] with head stride 128");
    return t;
  }
  return at::empty({B, L, H, kD}, o);
}

std::vector<at::Tensor> attention_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                      const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse, bool causal,
                                      int64_t window, double scale, const c10::optional<at::Tensor>& dq_out,
                                      const c10::optional<at::Tensor>& dk_out, const c10::optional<at::Tensor>& dv_out,
                                      const c10::optional<at::Tensor>& rope_cos,
                                      const c10::optional<at::Tensor>& rope_sin, bool rope_q, bool rope_k) {
  FYB_RANGE("fyb::attention_bwd");
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  FYB_CHECK(dout.is_contiguous() && o.is_contiguous() && dout.sizes() == q.sizes(), "attention_bwd: dout/o");
  const int B = (int)q.size(0), Lq = (int)q.size(1), Hq = (int)q.size(2), Lk = (int)k.size(1), Hk = (int)k.size(2);
  c10::cuda::CUDAGuard guard(q.device());
  auto delta = at::empty({B, Hq, Lq}, q.options().dtype(at::kFloat));
  auto dq_acc = at::zeros({B, Lq, Hq, kD}, q.options().dtype(at::kFloat));
  auto dk = out_view(dk_out, B, Lk, Hk, q.options(), "attention_bwd dk");
  auto dv = out_view(dv_out, B, Lk, Hk, q.options(), "attention_bwd dv");
  auto dq = out_view(dq_out, B, Lq, Hq, q.options(), "attention_bwd dq");
  const __nv_bfloat16* rc = nullptr;
  const __nv_bfloat16* rs = nullptr;
  if (rope_cos.has_value() && rope_cos->defined()) {
    FYB_CHECK(rope_sin.has_value() && rope_cos->is_contiguous() && rope_sin->is_contiguous() &&
                  rope_cos->size(0) >= std::max(Lq, Lk) && rope_cos->size(1) == kD / 2,
              "attention_bwd: rope tables [L, 64] expected");
    rc = reinterpret_cast<const __nv_bfloat16*>(rope_cos->data_ptr());
    rs = reinterpret_cast<const __nv_bfloat16*>(rope_sin->data_ptr());
  }
  if (B == 0 || Lq == 0) return {dq.zero_(), dk.zero_(), dv.zero_()};
  const int64_t rows = (int64_t)B * Lq * Hq;
  rowdot_kernel<<<(rows * 32 + 255) / 256, 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()),
      delta.data_ptr<float>(), B, Lq, Hq, nullptr);
  check_launch("attn_bwd_delta");
  // GQA: one CTA per (key tile, query head) with fp32 dK / dV accumulators, so the grid is G times larger and the
  // longest CTA walks one head's query tiles instead of the whole group's
  const int G = Hq / Hk;
  const bool split = G > 1;
  at::Tensor dk_acc, dv_acc;
  if (split) {
    dk_acc = at::empty({G, B, Lk, Hk, kD}, q.options().dtype(at::kFloat));
    dv_acc = at::empty({G, B, Lk, Hk, kD}, q.options().dtype(at::kFloat));
  }
  AttnBwdParams p{B, Lq, Lk, Hq, Hk, Lk - Lq, (int)window, causal ? 1 : 0, (float)scale, lse.data_ptr<float>(),
                  delta.data_ptr<float>(), nullptr, dq_acc.data_ptr<float>(),
                  split ? dk_acc.data_ptr<float>() : nullptr, split ? dv_acc.data_ptr<float>() : nullptr,
                  split ? 1 : 0,
                  reinterpret_cast<__nv_bfloat16*>(dk.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()),
                  dk.stride(1), dv.stride(1), rope_k ? rc : nullptr, rope_k ? rs : nullptr, status_ptr()};
  const CUtensorMap tq = tmap_heads(q), tk = tmap_heads(k), tv = tmap_heads(v), tdo = tmap_heads(dout);
  const CUtensorMap tdq = tmap_dq(dq_acc);
  static bool init = false;
  if (!init) {
    set_smem(attn_bwd_kernel<kSoftmax>, kBwdSmem);
    init = true;
  }
  const int grid = B * Hk * (split ? G : 1) * ((Lk + kT - 1) / kT);
  attn_bwd_kernel<kSoftmax><<<grid, kAttnThreads, kBwdSmem, cur_stream()>>>(tq, tk, tv, tdo, tdq, p);
  check_launch("attn_bwd");
  if (split) {
    const int64_t nk4 = static_cast<int64_t>(B) * Lk * Hk * (kD / 4);
    dq_out_kernel<<<static_cast<int>((nk4 + 255) / 256), 256, 0, cur_stream()>>>(
        dk_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dk.data_ptr()), dk.stride(1), B, Lk, Hk,
        rope_k ? rc : nullptr, rope_k ? rs : nullptr, G);
    check_launch("attn_bwd_dk");
    dq_out_kernel<<<static_cast<int>((nk4 + 255) / 256), 256, 0, cur_stream()>>>(
        dv_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()), dv.stride(1), B, Lk, Hk,
        nullptr, nullptr, G);
    check_launch("attn_bwd_dv");
  }
  const int64_t nq4 = static_cast<int64_t>(B) * Lq * Hq * (kD / 4);
  dq_out_kernel<<<static_cast<int>((nq4 + 255) / 256), 256, 0, cur_stream()>>>(
      dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), dq.stride(1), B, Lq, Hq,
      rope_q ? rc : nullptr, rope_q ? rs : nullptr);
  check_launch("attn_bwd_dq");
  return {dq, dk, dv};
}

at::Tensor retention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& gcum) {
  FYB_RANGE("fyb::retention_fwd");
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  const int B = (int)q.size(0), L = (int)q.size(1), H = (int)q.size(2);
  FYB_CHECK(k.sizes() == q.sizes() && v.sizes() == q.sizes(), "retention_fwd: q/k/v shapes differ");
  FYB_CHECK(gcum.scalar_type() == at::kFloat && gcum.is_contiguous() && gcum.dim() == 3 && gcum.size(0) == B &&
                gcum.size(1) == H && gcum.size(2) == L,
            "retention_fwd: gcum must be contiguous fp32 [B, H, L]");
  c10::cuda::CUDAGuard guard(q.device());
  auto o = at::empty({B, L, H, kD}, q.options());
  if (B == 0 || L == 0) return o;
  AttnParams p{B, L, L, H, H, 0, 0, 1, (float)(1.0 / std::sqrt((double)kD)),
               reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), nullptr, gcum.data_ptr<float>(), status_ptr()};
  const CUtensorMap tq = tmap_heads(q), tk = tmap_heads(k), tv = tmap_heads(v);
  static bool init = false;
  if (!init) {
    set_smem(attn_fwd_kernel<kRetention>, kFwdSmem);
    init = true;
  }
  const int grid = B * H * ((L + kT - 1) / kT);
  attn_fwd_kernel<kRetention><<<grid, kAttnThreads, kFwdSmem, cur_stream()>>>(tq, tk, tv, p);
  check_launch("retention_fwd");
  return o;
}

std::vector<at::Tensor> retention_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                      const at::Tensor& v, const at::Tensor& gcum, const at::Tensor& o,
                                      const c10::optional<at::Tensor>& dq_out, const c10::optional<at::Tensor>& dk_out,
                                      const c10::optional<at::Tensor>& dv_out,
                                      const c10::optional<at::Tensor>& rope_cos,
                                      const c10::optional<at::Tensor>& rope_sin) {
  FYB_RANGE("fyb::retention_bwd");
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  FYB_CHECK(dout.is_contiguous() && o.is_contiguous() && dout.sizes() == q.sizes(), "retention_bwd: dout/o");
  const int B = (int)q.size(0), L = (int)q.size(1), H = (int)q.size(2);
  c10::cuda::CUDAGuard guard(q.device());
  auto dgo = at::empty({B, H, L}, q.options().dtype(at::kFloat));
  auto dg = at::empty({B, H, L}, q.options().dtype(at::kFloat));
  auto dq_acc = at::zeros({B, L, H, kD}, q.options().dtype(at::kFloat));
  auto dk = out_view(dk_out, B, L, H, q.options(), "retention_bwd dk");
  auto dv = out_view(dv_out, B, L, H, q.options(), "retention_bwd dv");
  auto dq = out_view(dq_out, B, L, H, q.options(), "retention_bwd dq");
  const __nv_bfloat16* rc = nullptr;
  const __nv_bfloat16* rs = nullptr;
  if (rope_cos.has_value() && rope_cos->defined()) {
    FYB_CHECK(rope_sin.has_value() && rope_cos->is_contiguous() && rope_sin->is_contiguous() &&
                  rope_cos->size(0) >= L && rope_cos->size(1) == kD / 2,
              "retention_bwd: rope tables [L, 64] expected");
    rc = reinterpret_cast<const __nv_bfloat16*>(rope_cos->data_ptr());
    rs = reinterpret_cast<const __nv_bfloat16*>(rope_sin->data_ptr());
  }
  if (B == 0 || L == 0) return {dq.zero_(), dk.zero_(), dv.zero_(), dg.zero_()};
  const int64_t rows = (int64_t)B * L * H;
  rowdot_kernel<<<(rows * 32 + 255) / 256, 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()),
      dgo.data_ptr<float>(), B, L, H, nullptr);
  check_launch("retention_bwd_dot");
  AttnBwdParams p{B, L, L, H, H, 0, 0, 1, (float)(1.0 / std::sqrt((double)kD)), nullptr, nullptr,
                  gcum.data_ptr<float>(), dq_acc.data_ptr<float>(), nullptr, nullptr, 0,
                  reinterpret_cast<__nv_bfloat16*>(dk.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()),
                  dk.stride(1), dv.stride(1), rc, rs, status_ptr()};
  const CUtensorMap tq = tmap_heads(q), tk = tmap_heads(k), tv = tmap_heads(v), tdo = tmap_heads(dout);
  const CUtensorMap tdq = tmap_dq(dq_acc);
  static bool init = false;
  if (!init) {
    set_smem(attn_bwd_kernel<kRetention>, kBwdSmem);
    init = true;
  }
  const int grid = B * H * ((L + kT - 1) / kT);
  attn_bwd_kernel<kRetention><<<grid, kAttnThreads, kBwdSmem, cur_stream()>>>(tq, tk, tv, tdo, tdq, p);
  check_launch("retention_bwd");
  // dG = dO.O - V.dV (both operands may be token-strided views)
  rowdot_kernel<<<(rows * 32 + 255) / 256, 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dv.data_ptr()),
      dg.data_ptr<float>(), B, L, H, dgo.data_ptr<float>(), v.stride(1), dv.stride(1));
  check_launch("retention_bwd_dg");
  const int64_t nq4 = static_cast<int64_t>(B) * L * H * (kD / 4);
  dq_out_kernel<<<static_cast<int>((nq4 + 255) / 256), 256, 0, cur_stream()>>>(
      dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), dq.stride(1), B, L, H, rc, rs);
  check_launch("retention_bwd_dq");
  return {dq, dk, dv, dg};
}

}  // namespace fyb
