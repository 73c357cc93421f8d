// Memory-bound kernels: SwiGLU, rotary embedding, scaled embedding gather / scatter-sum, cross-entropy over the
// vocabulary, the sharded Adam step and the gradient sum of squares.
//
// References: SwiGLU kernel/swiglu.py:4-17 (silu of the first operand); rotary kernel/rotary.py:20-141
// (interleaved pairs, fp32 math, conjugate rotation for the backward); fused CE tasks/fused_ce.py:23-59 (online
// log-sum-exp over bf16 logits, bf16 gradient (softmax - onehot) * g, 0 for padding targets); fused Adam
// tasks/fused_adam_cast.py:19-45 (apex AdamFunctor: fma for m and v, IEEE division and square root, host bias
// corrections, bf16 copy of the new master); owner embedding gradient models/decoder/layer_graphs.py:68-105.
#include <ATen/ATen.h>
#include <c10/util/Optional.h>

#include "common/host.h"
#include "common/ptx.cuh"
#include "common/bounds.cuh"
#include "common/zero_map.cuh"

namespace fyb {
namespace {

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = unpack_bf16(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  *reinterpret_cast<uint4*>(p) =
      make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]), pack_bf16(f[6], f[7]));
}


// ------------------------------------------------------------------------------------------------------------------
// SwiGLU on [M, N] views with row strides (N % 8 == 0)

// grid: (rows, column blocks of 8 x blockDim values); no integer division per thread
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ y,
                                  int64_t ldy, __nv_bfloat16* __restrict__ out, int64_t M, int N) {
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (c >= N) return;
  const int64_t r = blockIdx.x;
  float a[8], b[8], o[8];
  load8(x + r * ldx + c, a);
  load8(y + r * ldy + c, b);
#pragma unroll
  for (int k = 0; k < 8; ++k) o[k] = swiglu_val(a[k], b[k]);
  store8(out + r * N + c, o);
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ y,
                                  int64_t ldy, const __nv_bfloat16* __restrict__ g, __nv_bfloat16* __restrict__ dx,
                                  __nv_bfloat16* __restrict__ dy, int64_t M, int N, int64_t lddx, int64_t lddy) {
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (c >= N) return;
  const int64_t r = blockIdx.x;
  float a[8], b[8], gg[8], da[8], db[8];
  load8(x + r * ldx + c, a);
  load8(y + r * ldy + c, b);
  load8(g + r * N + c, gg);
#pragma unroll
  for (int k = 0; k < 8; ++k) swiglu_grad(a[k], b[k], gg[k], da[k], db[k]);
  store8(dx + r * lddx + c, da);
  store8(dy + r * lddy + c, db);
}

// ------------------------------------------------------------------------------------------------------------------
// rotary embedding, interleaved pairs. x: [B, L, H, D] strided (last dim contiguous); out contiguous.

// one block per token (b * L + l); its threads walk the (head, 8-value chunk) items; per = D / 8 is a power of two
__global__ void rope_kernel(const __nv_bfloat16* __restrict__ x, int64_t sb, int64_t sl, int64_t sh,
                            const __nv_bfloat16* __restrict__ cos_t, const __nv_bfloat16* __restrict__ sin_t,
                            __nv_bfloat16* __restrict__ out, int B, int L, int H, int D, float sign) {
  const int per = D / 8;
  const int l = static_cast<int>(blockIdx.x % static_cast<unsigned>(L));
  const int b = static_cast<int>(blockIdx.x / static_cast<unsigned>(L));
  for (int j = threadIdx.x; j < H * per; j += blockDim.x) {
    const int c8 = (j & (per - 1)) * 8;
    const int h = j / per;
    float f[8], o[8];
    load8(x + b * sb + l * sl + h * sh + c8, f);
    const __nv_bfloat16* cp = cos_t + static_cast<int64_t>(l) * (D / 2) + c8 / 2;
    const __nv_bfloat16* spp = sin_t + static_cast<int64_t>(l) * (D / 2) + c8 / 2;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float cs = __bfloat162float(cp[k]);
      const float sn = sign * __bfloat162float(spp[k]);
      rope_rot(f[2 * k], f[2 * k + 1], cs, sn, o[2 * k], o[2 * k + 1]);
    }
    store8(out + ((static_cast<int64_t>(b) * L + l) * H + h) * D + c8, o);
  }
}

// NeoX / non-interleaved rotary: pairs (x[i], x[i + D/2]); each thread rotates 8 pairs.
__global__ void rope_neox_kernel(const __nv_bfloat16* __restrict__ x, int64_t sb, int64_t sl, int64_t sh,
                                 const __nv_bfloat16* __restrict__ cos_t, const __nv_bfloat16* __restrict__ sin_t,
                                 __nv_bfloat16* __restrict__ out, int B, int L, int H, int D, float sign) {
  const int half = D / 2;
  const int per = half / 8;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(B) * L * H * per;
  if (i >= total) return;
  const int c8 = static_cast<int>(i % per) * 8;
  int64_t rest = i / per;
  const int h = static_cast<int>(rest % H);
  rest /= H;
  const int l = static_cast<int>(rest % L);
  const int b = static_cast<int>(rest / L);
  float a[8], bb[8], oa[8], ob[8];
  const __nv_bfloat16* src = x + b * sb + l * sl + h * sh;
  load8(src + c8, a);
  load8(src + half + c8, bb);
  const __nv_bfloat16* cp = cos_t + static_cast<int64_t>(l) * half + c8;
  const __nv_bfloat16* spp = sin_t + static_cast<int64_t>(l) * half + c8;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float cs = __bfloat162float(cp[k]);
    const float sn = sign * __bfloat162float(spp[k]);
    oa[k] = a[k] * cs - bb[k] * sn;
    ob[k] = a[k] * sn + bb[k] * cs;
  }
  __nv_bfloat16* dst = out + ((static_cast<int64_t>(b) * L + l) * H + h) * D;
  store8(dst + c8, oa);
  store8(dst + half + c8, ob);
}

// ------------------------------------------------------------------------------------------------------------------
// embedding: out[i] = bf16(w[tok[i]] * scale)

__global__ void embed_fwd_kernel(const int64_t* __restrict__ tok, const __nv_bfloat16* __restrict__ w,
                                 __nv_bfloat16* __restrict__ out, int64_t M, int N, float scale, int64_t V,
                                 int* status) {
  const int per = N / 8;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= M * per) return;
  const int64_t r = i / per;
  const int c = static_cast<int>(i % per) * 8;
  int64_t t = tok[r];
  if (t < 0 || t >= V) {
    record_status(status, kBounds, 100);
    t = 0;
  }
  float f[8];
  load8(w + t * N + c, f);
#pragma unroll
  for (int k = 0; k < 8; ++k) f[k] *= scale;
  store8(out + r * N + c, f);
}

// Deterministic embedding gradient: block j handles the FIRST occurrence of token tok[j] and sums, in position
// order, bf16(dy[i] * scale) over every position i with the same token (fp32 accumulation). Rows of tokens that do
// not occur must be zero beforehand.
// Deterministic embedding gradient: positions sorted by token (stable, so equal tokens keep ascending position
// order); the CTA at the first sorted position of each token sums that token's rows of dy in position order and
// writes the row of dw once. Rows of dw that no position touches stay zero (memset before).
__global__ void embed_bwd_kernel(const int64_t* __restrict__ sorted_tok, const int64_t* __restrict__ order,
                                 const __nv_bfloat16* __restrict__ dy, __nv_bfloat16* __restrict__ dw, int64_t M,
                                 int N, float scale, int64_t V) {
  const int64_t j = blockIdx.x;
  const int64_t t = sorted_tok[j];
  if (!FYB_IN_BOUNDS(t, V, 503) || t < 0 || t >= V) return;
  if (j > 0 && sorted_tok[j - 1] == t) return;      // not the first position of this token
  int64_t end = j + 1;
  while (end < M && sorted_tok[end] == t) ++end;
  for (int c = threadIdx.x * 8; c < N; c += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t i = j; i < end; ++i) {
      float f[8];
      load8(dy + order[i] * N + c, f);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += bf16_round(f[k] * scale);
    }
    store8(dw + t * N + c, acc);
  }
}

// Embedding backward fused with the ZeRO reduce-scatter: the same per-token sums as embed_bwd_kernel, each row of
// the weight gradient stored at its owners (OwnerScatter: this rank's slot or the owner's staging slot) instead of
// locally. Only the rows of tokens in the batch are stored: the owners keep the rest of their staging slots zero.
__global__ void embed_bwd_scatter_kernel(const int64_t* __restrict__ sorted_tok, const int64_t* __restrict__ order,
                                         const __nv_bfloat16* __restrict__ dy, int64_t M, int N, float scale,
                                         int64_t V, const OwnerScatter sc) {
  const int64_t j = blockIdx.x;
  const int64_t t = sorted_tok[j];
  if (!FYB_IN_BOUNDS(t, V, 504) || t < 0 || t >= V) return;
  if (j > 0 && sorted_tok[j - 1] == t) return;      // not the first position of this token
  int64_t end = j + 1;
  while (end < M && sorted_tok[end] == t) ++end;
  for (int c = threadIdx.x * 8; c < N; c += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t i = j; i < end; ++i) {
      float f[8];
      load8(dy + order[i] * N + c, f);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += bf16_round(f[k] * scale);
    }
    if (__nv_bfloat16* d = owner_dst(sc, sc.x0 + t * N + c)) store8(d, acc);
  }
}

// ------------------------------------------------------------------------------------------------------------------
// cross-entropy over bf16 logits [M, V] (row stride ld), one CTA per row

constexpr int kCeThreads = 512;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}

__global__ void __launch_bounds__(kCeThreads) ce_fwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld,
                                                            const int64_t* __restrict__ tgt, float* __restrict__ loss,
                                                            float* __restrict__ lse_out, int V, int64_t ignore) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * ld;
  float m = -INFINITY, s = 0.f;
  const bool vec = (V % 8 == 0) && (ld % 8 == 0);
  if (vec) {
    for (int c = threadIdx.x * 8; c < V; c += kCeThreads * 8) {
      float f[8];
      load8(xr + c, f);
      float mx = f[0];
#pragma unroll
      for (int k = 1; k < 8; ++k) mx = fmaxf(mx, f[k]);
      const float mn = fmaxf(m, mx);
      float acc = s * __expf(m - mn);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc += __expf(f[k] - mn);
      s = acc;
      m = mn;
    }
  } else {
    for (int c = threadIdx.x; c < V; c += kCeThreads) {
      const float f = __bfloat162float(xr[c]);
      const float mn = fmaxf(m, f);
      s = s * __expf(m - mn) + __expf(f - mn);
      m = mn;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  __shared__ float sm[32], ss[32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sm[w] = m;
    ss[w] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M_ = sm[0], S_ = ss[0];
    for (int i = 1; i < kCeThreads / 32; ++i) online_merge(M_, S_, sm[i], ss[i]);
    const float lse = M_ + logf(S_);
    const int64_t t = tgt[row];
    lse_out[row] = lse;
    const bool valid = t != ignore && FYB_IN_BOUNDS(t, V, 502) && t >= 0 && t < V;
    loss[row] = valid ? lse - __bfloat162float(xr[t]) : 0.f;
  }
}

__global__ void __launch_bounds__(kCeThreads) ce_bwd_kernel(const __nv_bfloat16* x, int64_t ld,
                                                            const int64_t* __restrict__ tgt,
                                                            const float* __restrict__ lse_in,
                                                            const float* __restrict__ grad, __nv_bfloat16* dx,
                                                            int64_t ldd, int V, int64_t ignore) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * ld;
  __nv_bfloat16* dr = dx + row * ldd;
  const int64_t t = tgt[row];
  const float lse = lse_in[row];
  const float g = (t == ignore) ? 0.f : grad[0];
  const bool vec = (V % 8 == 0) && (ld % 8 == 0) && (ldd % 8 == 0);
  if (vec) {
    for (int c = threadIdx.x * 8; c < V; c += kCeThreads * 8) {
      float f[8];
      load8(xr + c, f);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float p = __expf(f[k] - lse);
        if (c + k == t) p -= 1.0f;
        f[k] = p * g;
      }
      store8(dr + c, f);
    }
  } else {
    for (int c = threadIdx.x; c < V; c += kCeThreads) {
      float p = __expf(__bfloat162float(xr[c]) - lse);
      if (c == t) p -= 1.0f;
      dr[c] = __float2bfloat16_rn(p * g);
    }
  }
}

// ------------------------------------------------------------------------------------------------------------------
// Adam (apex AdamFunctor expression), 4 elements per thread. hyper = [lr, bias_corr1, bias_corr2, step].

__device__ __forceinline__ void adam_elem(float& p, float& m, float& v, float g, float lr, float b1, float b2,
                                          float eps, float wd, float bc1, float bc2, bool adamw) {
  if (!adamw) g = g + wd * p;
  m = fmaf(b1, m, (1.0f - b1) * g);
  v = fmaf(b2, v, ((1.0f - b2) * g) * g);
  const float mh = __fdiv_rn(m, bc1);
  const float vh = __fdiv_rn(v, bc2);
  const float denom = __fadd_rn(__fsqrt_rn(vh), eps);
  float upd = __fdiv_rn(mh, denom);
  if (adamw) upd = upd + wd * p;
  p = p - lr * upd;
}

__global__ void adam_kernel(float* __restrict__ p32, const __nv_bfloat16* __restrict__ g16, float* __restrict__ m,
                            float* __restrict__ v, __nv_bfloat16* __restrict__ p16, const float* __restrict__ hyper,
                            const float* __restrict__ factor, int64_t n, float b1, float b2, float eps, float wd,
                            bool adamw, const ZeroMap z) {
  const float lr = hyper[0], bc1 = hyper[1], bc2 = hyper[2];
  const float f = factor[0];
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 4;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < n; i += stride) {
    if (i + 4 <= n) {
      const int64_t x = zero_flat(z, i);   // the bf16 gradient / parameter of local element i (4 in one chunk)
      // every byte is touched once per update: streaming loads / stores (evict-first) keep the L2 for the rest
      float4 P = __ldcs(reinterpret_cast<const float4*>(p32 + i));
      float4 Mv = __ldcs(reinterpret_cast<const float4*>(m + i));
      float4 Vv = __ldcs(reinterpret_cast<const float4*>(v + i));
      const uint2 gu = __ldcs(reinterpret_cast<const uint2*>(g16 + x));
      const float2 g01 = unpack_bf16(gu.x), g23 = unpack_bf16(gu.y);
      adam_elem(P.x, Mv.x, Vv.x, g01.x * f, lr, b1, b2, eps, wd, bc1, bc2, adamw);
      adam_elem(P.y, Mv.y, Vv.y, g01.y * f, lr, b1, b2, eps, wd, bc1, bc2, adamw);
      adam_elem(P.z, Mv.z, Vv.z, g23.x * f, lr, b1, b2, eps, wd, bc1, bc2, adamw);
      adam_elem(P.w, Mv.w, Vv.w, g23.y * f, lr, b1, b2, eps, wd, bc1, bc2, adamw);
      __stcs(reinterpret_cast<float4*>(p32 + i), P);
      __stcs(reinterpret_cast<float4*>(m + i), Mv);
      __stcs(reinterpret_cast<float4*>(v + i), Vv);
      __stcs(reinterpret_cast<uint2*>(p16 + x), make_uint2(pack_bf16(P.x, P.y), pack_bf16(P.z, P.w)));
    } else {
      for (int64_t j = i; j < n; ++j) {
        const int64_t x = zero_flat(z, j);
        float P = p32[j], Mv = m[j], Vv = v[j];
        adam_elem(P, Mv, Vv, __bfloat162float(g16[x]) * f, lr, b1, b2, eps, wd, bc1, bc2, adamw);
        p32[j] = P;
        m[j] = Mv;
        v[j] = Vv;
        p16[x] = __float2bfloat16_rn(P);
      }
    }
  }
}

// Adam fused with the ZeRO parameter all-gather: the owner updates its segment (the expression of adam_kernel,
// 8 elements per thread) and stores each 16-byte group of new bf16 parameters into its own flat buffer AND into every
// peer's flat buffer at the same offset (remote stores over NVLink into CUDA-IPC mapped memory), so the exchange
// streams out while the HBM-bound update runs instead of after it. A flag barrier after the kernel publishes the
// stores; the system fence at the end orders them before it.
struct PushTargets {
  void* p[8];
};

__global__ void adam_push_kernel(float* __restrict__ p32, const __nv_bfloat16* __restrict__ g16,
                                 float* __restrict__ m, float* __restrict__ v, __nv_bfloat16* __restrict__ p16,
                                 const float* __restrict__ hyper, const float* __restrict__ factor, int64_t n,
                                 float b1, float b2, float eps, float wd, bool adamw, PushTargets peers,
                                 int64_t peer_off, int world, int rank, int64_t chunk) {
  const float lr = hyper[0], bc1 = hyper[1], bc2 = hyper[2];
  const float f = factor[0];
  const ZeroMap z{chunk, world, rank};
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 8;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < n; i += stride) {
    if (i + 8 <= n) {
      const int64_t x = zero_flat(z, i);   // 8 local elements lie in one chunk
      float P[8], Mv[8], Vv[8], G[8];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float4 a = *reinterpret_cast<const float4*>(p32 + i + 4 * h);
        const float4 b = *reinterpret_cast<const float4*>(m + i + 4 * h);
        const float4 c = *reinterpret_cast<const float4*>(v + i + 4 * h);
        P[4 * h] = a.x, P[4 * h + 1] = a.y, P[4 * h + 2] = a.z, P[4 * h + 3] = a.w;
        Mv[4 * h] = b.x, Mv[4 * h + 1] = b.y, Mv[4 * h + 2] = b.z, Mv[4 * h + 3] = b.w;
        Vv[4 * h] = c.x, Vv[4 * h + 1] = c.y, Vv[4 * h + 2] = c.z, Vv[4 * h + 3] = c.w;
      }
      {
        const uint4 gu = *reinterpret_cast<const uint4*>(g16 + x);
        const uint32_t gw[4] = {gu.x, gu.y, gu.z, gu.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 t = unpack_bf16(gw[k]);
          G[2 * k] = t.x;
          G[2 * k + 1] = t.y;
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) adam_elem(P[k], Mv[k], Vv[k], G[k] * f, lr, b1, b2, eps, wd, bc1, bc2, adamw);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        *reinterpret_cast<float4*>(p32 + i + 4 * h) = make_float4(P[4 * h], P[4 * h + 1], P[4 * h + 2], P[4 * h + 3]);
        *reinterpret_cast<float4*>(m + i + 4 * h) = make_float4(Mv[4 * h], Mv[4 * h + 1], Mv[4 * h + 2], Mv[4 * h + 3]);
        *reinterpret_cast<float4*>(v + i + 4 * h) = make_float4(Vv[4 * h], Vv[4 * h + 1], Vv[4 * h + 2], Vv[4 * h + 3]);
      }
      const uint4 out = make_uint4(pack_bf16(P[0], P[1]), pack_bf16(P[2], P[3]), pack_bf16(P[4], P[5]),
                                   pack_bf16(P[6], P[7]));
      *reinterpret_cast<uint4*>(p16 + x) = out;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (q < world && q != rank)
          *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(peers.p[q]) + peer_off + x) = out;
    } else {
      for (int64_t j = i; j < n; ++j) {
        const int64_t xj = zero_flat(z, j);
        float P = p32[j], Mv = m[j], Vv = v[j];
        adam_elem(P, Mv, Vv, __bfloat162float(g16[xj]) * f, lr, b1, b2, eps, wd, bc1, bc2, adamw);
        p32[j] = P;
        m[j] = Mv;
        v[j] = Vv;
        const __nv_bfloat16 o = __float2bfloat16_rn(P);
        p16[xj] = o;
        for (int q = 0; q < world; ++q)
          if (q != rank) reinterpret_cast<__nv_bfloat16*>(peers.p[q])[peer_off + xj] = o;
      }
    }
  }
  __threadfence_system();
}

// ------------------------------------------------------------------------------------------------------------------
// sum of squares of a bf16 vector: per-CTA fp32 partials, then one CTA sums them in a fixed order

constexpr int kSqThreads = 512;

__global__ void sq_partial_kernel(const __nv_bfloat16* __restrict__ x, int64_t n, float* __restrict__ part) {
  float s = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 8;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < n; i += stride) {
    if (i + 8 <= n) {
      float f[8];
      load8(x + i, f);
#pragma unroll
      for (int k = 0; k < 8; ++k) s += f[k] * f[k];
    } else {
      for (int64_t j = i; j < n; ++j) {
        const float f = __bfloat162float(x[j]);
        s += f * f;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < kSqThreads / 32; ++i) t += red[i];
    part[blockIdx.x] = t;
  }
}

// Sum of squares over many ranges of one bf16 buffer in one launch: block i sums chunk i ([start, start + len),
// len <= 65,536, any alignment) into part[i]; the caller sums the partials in order (deterministic).
__global__ void sq_ranges_kernel(const __nv_bfloat16* __restrict__ x, const int64_t* __restrict__ chunks,
                                 float* __restrict__ part) {
  const int64_t start = chunks[2 * blockIdx.x], len = chunks[2 * blockIdx.x + 1];
  const __nv_bfloat16* p = x + start;
  // scalar head up to a 16-byte boundary, then 8-wide loads, then a scalar tail
  const int64_t mis = static_cast<int64_t>(((16 - (reinterpret_cast<uintptr_t>(p) & 15)) & 15) / 2);
  const int64_t head = len < mis ? len : mis;
  float s = 0.f;
  for (int64_t j = threadIdx.x; j < head; j += blockDim.x) {
    const float f = __bfloat162float(p[j]);
    s += f * f;
  }
  const int64_t nvec = (len - head) / 8;
  for (int64_t v = threadIdx.x; v < nvec; v += blockDim.x) {
    float f[8];
    load8(p + head + 8 * v, f);
#pragma unroll
    for (int k = 0; k < 8; ++k) s += f[k] * f[k];
  }
  for (int64_t j = head + 8 * nvec + threadIdx.x; j < len; j += blockDim.x) {
    const float f = __bfloat162float(p[j]);
    s += f * f;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    part[blockIdx.x] = t;
  }
}

__global__ void sq_final_kernel(const float* __restrict__ part, int P, float* __restrict__ out) {
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

// ------------------------------------------------------------------------------------------------------------------
// retention gates: gcum[b, h, t] = sum_{s<=t} logsigmoid(y[b*L+s, h]) / normalizer (fp32), one warp per (b, h);
// backward: dy[b*L+t, h] = sigmoid(-y) / normalizer * sum_{s>=t} dgcum[b, h, s]

__device__ __forceinline__ float logsigmoidf_(float x) { return fminf(x, 0.f) - log1pf(__expf(-fabsf(x))); }

// One CTA (1024 threads) per (b, h); each thread owns a contiguous run of positions: local sums, a block-wide
// exclusive scan of the run totals (warp shuffles + one shared-memory level), then the run is rewritten.
constexpr int kScanThreads = 1024;

__device__ __forceinline__ float block_exclusive_scan(float v, float* sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float u = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += u;
  }
  if (lane == 31) sh[w] = inc;
  __syncthreads();
  if (w == 0) {
    float t = lane < (kScanThreads >> 5) ? sh[lane] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float u = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += u;
    }
    sh[lane] = t;   // inclusive prefix of warp totals
  }
  __syncthreads();
  const float before_warp = w > 0 ? sh[w - 1] : 0.f;
  __syncthreads();
  return before_warp + inc - v;
}

__global__ void __launch_bounds__(kScanThreads) gate_cumsum_fwd_kernel(const __nv_bfloat16* __restrict__ y,
                                                                      int64_t ldy, float* __restrict__ gcum, int B,
                                                                      int L, int H, float inv_norm) {
  __shared__ float sh[32];
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  const int per = (L + kScanThreads - 1) / kScanThreads;
  const int t0 = threadIdx.x * per, t1 = min(L, t0 + per);
  float local = 0.f;
  for (int t = t0; t < t1; ++t)
    // F.logsigmoid on bf16 rounds its output to bf16; the division by the normaliser (a power of two) is exact
    local += bf16_round(logsigmoidf_(__bfloat162float(y[(static_cast<int64_t>(b) * L + t) * ldy + h]))) * inv_norm;
  float run = block_exclusive_scan(local, sh);
  float* out = gcum + static_cast<int64_t>(bh) * L;
  for (int t = t0; t < t1; ++t) {
    run += bf16_round(logsigmoidf_(__bfloat162float(y[(static_cast<int64_t>(b) * L + t) * ldy + h]))) * inv_norm;
    out[t] = run;
  }
}

// Chunk-local variant (chunkwise retention): the cumsum restarts at every multiple of 128 positions. One warp per
// (b, h, chunk), four positions per lane, a warp scan of the lane totals.
__global__ void __launch_bounds__(256) gate_cumsum_chunk_kernel(const __nv_bfloat16* __restrict__ y, int64_t ldy,
                                                                float* __restrict__ gcum, int B, int L, int H,
                                                                float inv_norm) {
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nc = (L + 127) / 128;
  if (wid >= static_cast<int64_t>(B) * H * nc) return;
  const int c = static_cast<int>(wid % nc);
  const int bh = static_cast<int>(wid / nc);
  const int b = bh / H, h = bh % H;
  const int t0 = c * 128 + lane * 4;
  float v[4];
  float run = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + i;
    const float x = t < L ? bf16_round(logsigmoidf_(__bfloat162float(y[(static_cast<int64_t>(b) * L + t) * ldy + h])))
                                * inv_norm : 0.f;
    run += x;
    v[i] = run;
  }
  float inc = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float u = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += u;
  }
  const float excl = inc - run;
  float* out = gcum + static_cast<int64_t>(bh) * L;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (t0 + i < L) out[t0 + i] = excl + v[i];
}

// dy[b*L+t, h] = sigmoid(-y) / normalizer * sum_{s>=t} dg[b, h, s]  (reverse scan: thread i owns run i from the end)
__global__ void __launch_bounds__(kScanThreads) gate_cumsum_bwd_kernel(const float* __restrict__ dg,
                                                                      const __nv_bfloat16* __restrict__ y,
                                                                      int64_t ldy, __nv_bfloat16* __restrict__ dy,
                                                                      int64_t lddy, int B, int L, int H,
                                                                      float inv_norm) {
  __shared__ float sh[32];
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  const float* src = dg + static_cast<int64_t>(bh) * L;
  const int per = (L + kScanThreads - 1) / kScanThreads;
  // run i covers positions [L - (i+1)*per, L - i*per)
  const int t1 = L - threadIdx.x * per, t0 = max(0, t1 - per);
  float local = 0.f;
  for (int t = t0; t < t1; ++t) local += src[t];
  float run = block_exclusive_scan(local, sh);   // sum over positions after this run
  for (int t = t1 - 1; t >= t0; --t) {
    run += src[t];
    const int64_t row = static_cast<int64_t>(b) * L + t;
    const float x = __bfloat162float(y[row * ldy + h]);
    dy[row * lddy + h] = __float2bfloat16_rn(run * inv_norm / (1.0f + __expf(x)));
  }
}

}  // namespace

// ------------------------------------------------------------------------------------------------------------------
// host entry points

at::Tensor gate_cumsum_fwd(const at::Tensor& y, int64_t B, int64_t L, double normalizer, bool chunk_local) {
  FYB_RANGE("fyb::gate_cumsum_fwd");
  FYB_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.dim() == 2 && y.stride(1) == 1 && y.size(0) == B * L,
            "gate_cumsum_fwd: bf16 [B*L, H] view expected");
  c10::cuda::CUDAGuard guard(y.device());
  const int H = static_cast<int>(y.size(1));
  auto g = at::empty({B, H, L}, y.options().dtype(at::kFloat));
  if (chunk_local) {
    const int64_t warps = B * H * ((L + 127) / 128);
    if (warps > 0)
      gate_cumsum_chunk_kernel<<<static_cast<int>((warps * 32 + 255) / 256), 256, 0, cur_stream()>>>(
          reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), y.stride(0), g.data_ptr<float>(), (int)B, (int)L, H,
          static_cast<float>(1.0 / normalizer));
    check_launch("gate_cumsum_chunk");
    return g;
  }
  const int blocks = static_cast<int>(B) * H;
  if (blocks > 0)
    gate_cumsum_fwd_kernel<<<blocks, kScanThreads, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), y.stride(0), g.data_ptr<float>(), (int)B, (int)L, H,
        static_cast<float>(1.0 / normalizer));
  check_launch("gate_cumsum_fwd");
  return g;
}

void gate_cumsum_bwd(const at::Tensor& dg, const at::Tensor& y, at::Tensor& dy, double normalizer) {
  FYB_RANGE("fyb::gate_cumsum_bwd");
  const int64_t B = dg.size(0), H = dg.size(1), L = dg.size(2);
  FYB_CHECK(dg.is_contiguous() && dg.scalar_type() == at::kFloat, "gate_cumsum_bwd: dg fp32 [B, H, L]");
  FYB_CHECK(dy.stride(1) == 1 && dy.size(0) == B * L && dy.size(1) == H, "gate_cumsum_bwd: dy view [B*L, H]");
  c10::cuda::CUDAGuard guard(y.device());
  const int blocks = static_cast<int>(B * H);
  if (blocks > 0)
    gate_cumsum_bwd_kernel<<<blocks, kScanThreads, 0, cur_stream()>>>(
        dg.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), y.stride(0),
        reinterpret_cast<__nv_bfloat16*>(dy.data_ptr()), dy.stride(0), (int)B, (int)L, (int)H,
        static_cast<float>(1.0 / normalizer));
  check_launch("gate_cumsum_bwd");
}

at::Tensor swiglu_fwd(const at::Tensor& x, const at::Tensor& y) {
  FYB_RANGE("fyb::swiglu_fwd");
  FYB_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16 && x.dim() == 2 &&
                x.sizes() == y.sizes() && x.stride(1) == 1 && y.stride(1) == 1,
            "swiglu_fwd: bf16 [M, N] views with contiguous rows expected");
  const int64_t M = x.size(0), N = x.size(1);
  FYB_CHECK(N % 8 == 0 && x.stride(0) % 8 == 0 && y.stride(0) % 8 == 0, "swiglu_fwd: alignment");
  c10::cuda::CUDAGuard guard(x.device());
  auto out = at::empty({M, N}, x.options());
  const int64_t n = M * (N / 8);
  if (n > 0)
    swiglu_fwd_kernel<<<dim3(static_cast<unsigned>(M), static_cast<unsigned>((N / 8 + 127) / 128)), 128, 0,
                        cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), y.stride(0),
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), M, (int)N);
  check_launch("swiglu_fwd");
  return out;
}

std::vector<at::Tensor> swiglu_bwd(const at::Tensor& x, const at::Tensor& y, const at::Tensor& g,
                                   const c10::optional<at::Tensor>& dx_out, const c10::optional<at::Tensor>& dy_out) {
  FYB_RANGE("fyb::swiglu_bwd");
  const int64_t M = x.size(0), N = x.size(1);
  FYB_CHECK(g.is_contiguous() && g.size(0) == M && g.size(1) == N, "swiglu_bwd: grad");
  c10::cuda::CUDAGuard guard(x.device());
  auto pick = [&](const c10::optional<at::Tensor>& o) {
    if (o.has_value() && o->defined()) {
      FYB_CHECK(o->size(0) == M && o->size(1) == N && o->stride(1) == 1 && o->stride(0) % 8 == 0,
                "swiglu_bwd: output view");
      return *o;
    }
    return at::empty({M, N}, x.options());
  };
  auto dx = pick(dx_out);
  auto dy = pick(dy_out);
  const int64_t n = M * (N / 8);
  if (n > 0)
    swiglu_bwd_kernel<<<dim3(static_cast<unsigned>(M), static_cast<unsigned>((N / 8 + 127) / 128)), 128, 0,
                        cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), y.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(dy.data_ptr()), M, (int)N, dx.stride(0), dy.stride(0));
  check_launch("swiglu_bwd");
  return {dx, dy};
}

at::Tensor rope_fwd(const at::Tensor& x, const at::Tensor& cos_t, const at::Tensor& sin_t, bool conj, bool neox) {
  FYB_RANGE("fyb::rope_fwd");
  FYB_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 4 && x.stride(3) == 1,
            "rope: bf16 [B, L, H, D] with contiguous last dim expected");
  const int B = (int)x.size(0), L = (int)x.size(1), H = (int)x.size(2), D = (int)x.size(3);
  FYB_CHECK(D % 8 == 0 && x.stride(0) % 8 == 0 && x.stride(1) % 8 == 0 && x.stride(2) % 8 == 0,
            "rope: alignment (strides multiple of 8 elements)");
  FYB_CHECK(cos_t.is_contiguous() && sin_t.is_contiguous() && cos_t.size(0) >= L && cos_t.size(1) == D / 2 &&
                cos_t.scalar_type() == at::kBFloat16 && sin_t.scalar_type() == at::kBFloat16,
            "rope: cos/sin must be contiguous bf16 [L, D/2]");
  c10::cuda::CUDAGuard guard(x.device());
  auto out = at::empty({B, L, H, D}, x.options());
  if (neox) {
    FYB_CHECK(D % 16 == 0, "rope (neox): head dim must be a multiple of 16");
    const int64_t n = static_cast<int64_t>(B) * L * H * (D / 16);
    if (n > 0)
      rope_neox_kernel<<<(n + 255) / 256, 256, 0, cur_stream()>>>(
          reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), x.stride(1), x.stride(2),
          reinterpret_cast<const __nv_bfloat16*>(cos_t.data_ptr()),
          reinterpret_cast<const __nv_bfloat16*>(sin_t.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
          B, L, H, D, conj ? -1.f : 1.f);
    check_launch("rope_neox");
    return out;
  }
  FYB_CHECK(((D / 8) & (D / 8 - 1)) == 0, "rope: head dim / 8 must be a power of two");
  const int64_t n = static_cast<int64_t>(B) * L;
  if (n > 0 && H > 0)
    rope_kernel<<<static_cast<unsigned>(n), 128, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), x.stride(1), x.stride(2),
        reinterpret_cast<const __nv_bfloat16*>(cos_t.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(sin_t.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), B, L, H, D, conj ? -1.f : 1.f);
  check_launch("rope");
  return out;
}

at::Tensor embedding_fwd(const at::Tensor& tok, const at::Tensor& w, double scale) {
  FYB_RANGE("fyb::embedding_fwd");
  FYB_CHECK(tok.is_cuda() && tok.scalar_type() == at::kLong && tok.dim() == 1 && tok.is_contiguous(),
            "embedding_fwd: int64 token vector expected");
  FYB_CHECK(w.scalar_type() == at::kBFloat16 && w.dim() == 2 && w.is_contiguous() && w.size(1) % 8 == 0,
            "embedding_fwd: contiguous bf16 [V, N] with N % 8 == 0");
  c10::cuda::CUDAGuard guard(w.device());
  const int64_t M = tok.size(0), N = w.size(1);
  auto out = at::empty({M, N}, w.options());
  const int64_t n = M * (N / 8);
  if (n > 0)
    embed_fwd_kernel<<<(n + 255) / 256, 256, 0, cur_stream()>>>(
        tok.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), M, (int)N, (float)scale, w.size(0), status_ptr());
  check_launch("embedding_fwd");
  return out;
}

at::Tensor embedding_bwd(const at::Tensor& tok, const at::Tensor& dy, int64_t V, double scale,
                         const c10::optional<at::Tensor>& out_opt) {
  FYB_RANGE("fyb::embedding_bwd");
  FYB_CHECK(dy.is_contiguous() && dy.dim() == 2 && dy.size(1) % 8 == 0 && dy.size(0) == tok.size(0),
            "embedding_bwd: dy");
  const int64_t M = tok.size(0), N = dy.size(1);
  FYB_CHECK(M < (1ll << 31), "embedding_bwd: too many positions");
  c10::cuda::CUDAGuard guard(dy.device());
  at::Tensor dw;
  if (out_opt.has_value() && out_opt->defined()) {
    dw = *out_opt;
    FYB_CHECK(dw.is_contiguous() && dw.size(0) == V && dw.size(1) == N && dw.scalar_type() == at::kBFloat16,
              "embedding_bwd: out");
  } else {
    dw = at::empty({V, N}, dy.options());
  }
  FYB_CUDA(cudaMemsetAsync(dw.data_ptr(), 0, dw.numel() * 2, cur_stream()));
  if (M > 0) {
    // a stable sort of the (few thousand) token ids groups equal tokens, in position order
    auto sorted = at::sort(tok, /*stable=*/true, /*dim=*/0, /*descending=*/false);
    const at::Tensor& stok = std::get<0>(sorted);
    const at::Tensor& order = std::get<1>(sorted);
    embed_bwd_kernel<<<static_cast<unsigned>(M), 128, 0, cur_stream()>>>(
        stok.data_ptr<int64_t>(), order.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(dw.data_ptr()), M, (int)N, (float)scale, V);
  }
  check_launch("embedding_bwd");
  return dw;
}

// Weight gradient of the embedding stored at its ZeRO owners (embed_bwd_scatter_kernel): slot is the weight's
// [V, N] slot inside grad_flat; its local copy is zeroed (the rows this rank owns and no token touched stay zero),
// the touched rows go to their owners. bases: int64 [world] device tensor of every rank's staging buffer.
void embedding_bwd_scatter(const at::Tensor& tok, const at::Tensor& dy, double scale, at::Tensor& slot,
                           const at::Tensor& grad_flat, const at::Tensor& bases, int64_t seg, int64_t rank,
                           int64_t chunk) {
  FYB_RANGE("fyb::embedding_bwd_scatter");
  FYB_CHECK(dy.is_cuda() && dy.is_contiguous() && dy.dim() == 2 && dy.size(1) % 8 == 0 && dy.size(0) == tok.size(0),
            "embedding_bwd_scatter: dy");
  FYB_CHECK(slot.is_contiguous() && slot.dim() == 2 && slot.size(1) == dy.size(1) &&
                slot.scalar_type() == at::kBFloat16 && grad_flat.scalar_type() == at::kBFloat16,
            "embedding_bwd_scatter: slot must be a contiguous bf16 [V, N] slot of grad_flat");
  FYB_CHECK(bases.is_cuda() && bases.scalar_type() == at::kLong && bases.dim() == 1 && rank >= 0 &&
                rank < bases.size(0),
            "embedding_bwd_scatter: bases must be int64 [world]");
  const auto base = reinterpret_cast<uintptr_t>(grad_flat.data_ptr());
  const auto sp = reinterpret_cast<uintptr_t>(slot.data_ptr());
  FYB_CHECK(sp >= base && sp + slot.numel() * 2 <= base + grad_flat.numel() * 2,
            "embedding_bwd_scatter: slot must lie inside grad_flat");
  const int64_t x0 = static_cast<int64_t>((sp - base) / 2);
  FYB_CHECK(seg > 0 && seg % 8 == 0 && chunk % 8 == 0 && x0 % 8 == 0 && (chunk == 0 || seg % chunk == 0) &&
                x0 + slot.numel() <= bases.size(0) * seg,
            "embedding_bwd_scatter: seg / chunk / slot offset must be multiples of 8 inside the owners' range");
  const int64_t M = tok.size(0), N = dy.size(1), V = slot.size(0);
  FYB_CHECK(M < (1ll << 31), "embedding_bwd_scatter: too many positions");
  c10::cuda::CUDAGuard guard(dy.device());
  FYB_CUDA(cudaMemsetAsync(slot.data_ptr(), 0, slot.numel() * 2, cur_stream()));
  if (M > 0) {
    OwnerScatter sc;
    sc.bases = reinterpret_cast<const unsigned long long*>(bases.data_ptr<int64_t>());
    sc.own = reinterpret_cast<__nv_bfloat16*>(grad_flat.data_ptr());
    sc.x0 = x0;
    sc.seg = seg;
    sc.chunk = chunk;
    sc.rank = static_cast<int>(rank);
    sc.world = static_cast<int>(bases.size(0));
    auto sorted = at::sort(tok, /*stable=*/true, /*dim=*/0, /*descending=*/false);
    const at::Tensor& stok = std::get<0>(sorted);
    const at::Tensor& order = std::get<1>(sorted);
    embed_bwd_scatter_kernel<<<static_cast<unsigned>(M), 128, 0, cur_stream()>>>(
        stok.data_ptr<int64_t>(), order.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
        M, (int)N, (float)scale, V, sc);
  }
  check_launch("embedding_bwd_scatter");
}

std::vector<at::Tensor> ce_fwd(const at::Tensor& logits, const at::Tensor& target, int64_t ignore) {
  FYB_RANGE("fyb::ce_fwd");
  FYB_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1,
            "ce_fwd: bf16 [M, V] logits with contiguous rows expected");
  FYB_CHECK(target.scalar_type() == at::kLong && target.is_contiguous() && target.numel() == logits.size(0),
            "ce_fwd: int64 target [M]");
  c10::cuda::CUDAGuard guard(logits.device());
  const int64_t M = logits.size(0), V = logits.size(1);
  auto loss = at::empty({M}, logits.options().dtype(at::kFloat));
  auto lse = at::empty({M}, logits.options().dtype(at::kFloat));
  if (M > 0)
    ce_fwd_kernel<<<M, kCeThreads, 0, cur_stream()>>>(reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()),
                                                      logits.stride(0), target.data_ptr<int64_t>(),
                                                      loss.data_ptr<float>(), lse.data_ptr<float>(), (int)V, ignore);
  check_launch("ce_fwd");
  return {loss, lse};
}

at::Tensor ce_bwd(const at::Tensor& logits, const at::Tensor& target, const at::Tensor& lse, const at::Tensor& grad,
                  int64_t ignore, const c10::optional<at::Tensor>& out_opt) {
  FYB_RANGE("fyb::ce_bwd");
  c10::cuda::CUDAGuard guard(logits.device());
  const int64_t M = logits.size(0), V = logits.size(1);
  at::Tensor dx = (out_opt.has_value() && out_opt->defined()) ? *out_opt : at::empty_like(logits);
  FYB_CHECK(dx.sizes() == logits.sizes() && dx.stride(1) == 1 && dx.scalar_type() == at::kBFloat16, "ce_bwd: out");
  FYB_CHECK(grad.scalar_type() == at::kFloat && grad.numel() == 1, "ce_bwd: grad must be one fp32 value");
  if (M > 0)
    ce_bwd_kernel<<<M, kCeThreads, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0), target.data_ptr<int64_t>(),
        lse.data_ptr<float>(), grad.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), dx.stride(0),
        (int)V, ignore);
  check_launch("ce_bwd");
  return dx;
}

// chunk > 0 (block-cyclic ZeRO layout): g16 / p16 are the whole flat buffers and local element c of this owner is
// flat element ((c / chunk) * world + rank) * chunk + c % chunk; chunk == 0: g16 / p16 are this owner's segment.
void check_zero_map(const char* what, int64_t n, const at::Tensor& g16, const at::Tensor& p16, int64_t chunk,
                    int64_t world, int64_t rank) {
  if (chunk == 0) {
    FYB_CHECK(g16.numel() == n && p16.numel() == n, std::string(what) + ": segment views of the state's size expected");
    return;
  }
  FYB_CHECK(chunk % 8 == 0 && n % chunk == 0 && world >= 1 && rank >= 0 && rank < world,
            std::string(what) + ": chunk must be a multiple of 8 dividing the owned size");
  FYB_CHECK(g16.numel() == n * world && p16.numel() == n * world,
            std::string(what) + ": block-cyclic layout needs the whole flat buffers (world x owned size)");
}

void adam_step(at::Tensor& p32, const at::Tensor& g16, at::Tensor& m, at::Tensor& v, at::Tensor& p16,
               const at::Tensor& hyper, const at::Tensor& factor, double b1, double b2, double eps, double wd,
               bool adamw, int64_t chunk, int64_t world, int64_t rank) {
  FYB_RANGE("fyb::adam_step");
  const int64_t n = p32.numel();
  FYB_CHECK(p32.is_contiguous() && m.is_contiguous() && v.is_contiguous() && g16.is_contiguous() &&
                p16.is_contiguous() && m.numel() == n && v.numel() == n,
            "adam_step: contiguous tensors of equal size expected");
  check_zero_map("adam_step", n, g16, p16, chunk, world, rank);
  FYB_CHECK(p32.scalar_type() == at::kFloat && g16.scalar_type() == at::kBFloat16 &&
                p16.scalar_type() == at::kBFloat16,
            "adam_step: fp32 master / bf16 grad / bf16 param");
  FYB_CHECK(reinterpret_cast<uintptr_t>(g16.data_ptr()) % 8 == 0 && reinterpret_cast<uintptr_t>(p16.data_ptr()) % 8 == 0,
            "adam_step: bf16 buffers must be 8-byte aligned");
  c10::cuda::CUDAGuard guard(p32.device());
  if (n == 0) return;
  const int blocks = static_cast<int>(std::min<int64_t>((n / 4 + 255) / 256 + 1, num_sms() * 8));
  adam_kernel<<<blocks, 256, 0, cur_stream()>>>(
      p32.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(g16.data_ptr()), m.data_ptr<float>(),
      v.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(p16.data_ptr()), hyper.data_ptr<float>(),
      factor.data_ptr<float>(), n, (float)b1, (float)b2, (float)eps, (float)wd, adamw,
      ZeroMap{chunk, static_cast<int>(world), static_cast<int>(rank)});
  check_launch("adam");
}

void adam_push(at::Tensor& p32, const at::Tensor& g16, at::Tensor& m, at::Tensor& v, at::Tensor& p16,
               const at::Tensor& hyper, const at::Tensor& factor, double b1, double b2, double eps, double wd,
               bool adamw, const std::vector<int64_t>& peer_params, int64_t peer_off, int64_t rank, int64_t chunk) {
  FYB_RANGE("fyb::adam_push");
  const int64_t n = p32.numel();
  const int world = static_cast<int>(peer_params.size());
  FYB_CHECK(world >= 1 && world <= 8 && rank >= 0 && rank < world, "adam_push: 1..8 ranks");
  FYB_CHECK(p32.is_contiguous() && m.is_contiguous() && v.is_contiguous() && g16.is_contiguous() &&
                p16.is_contiguous() && m.numel() == n && v.numel() == n,
            "adam_push: contiguous tensors of equal size expected");
  check_zero_map("adam_push", n, g16, p16, chunk, world, rank);
  FYB_CHECK(chunk == 0 || peer_off == 0, "adam_push: the block-cyclic layout addresses peers from their buffer start");
  FYB_CHECK(p32.scalar_type() == at::kFloat && g16.scalar_type() == at::kBFloat16 &&
                p16.scalar_type() == at::kBFloat16,
            "adam_push: fp32 master / bf16 grad / bf16 param");
  FYB_CHECK(reinterpret_cast<uintptr_t>(g16.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(p16.data_ptr()) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(p32.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(m.data_ptr()) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(v.data_ptr()) % 16 == 0 && peer_off % 8 == 0,
            "adam_push: 16-byte aligned buffers and a segment offset that is a multiple of 8 elements");
  PushTargets t{};
  for (int q = 0; q < world; ++q) {
    FYB_CHECK(peer_params[q] % 16 == 0, "adam_push: peer buffers must be 16-byte aligned");
    t.p[q] = reinterpret_cast<void*>(peer_params[q]);
  }
  c10::cuda::CUDAGuard guard(p32.device());
  if (n == 0) return;
  const int blocks = static_cast<int>(std::min<int64_t>((n / 8 + 255) / 256 + 1, num_sms() * 8));
  adam_push_kernel<<<blocks, 256, 0, cur_stream()>>>(
      p32.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(g16.data_ptr()), m.data_ptr<float>(),
      v.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(p16.data_ptr()), hyper.data_ptr<float>(),
      factor.data_ptr<float>(), n, (float)b1, (float)b2, (float)eps, (float)wd, adamw, t, peer_off,
      world, static_cast<int>(rank), chunk);
  check_launch("adam_push");
}

int sq_norm_ctas(int64_t n) { return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + 4095) / 4096, 1024))); }

void sq_norm_into(const at::Tensor& x, float* part, int P, float* out) {
  sq_partial_kernel<<<P, kSqThreads, 0, cur_stream()>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                                                        x.numel(), part);
  check_launch("sq_partial");
  sq_final_kernel<<<1, 1024, 0, cur_stream()>>>(part, P, out);
  check_launch("sq_final");
}

// Sum of squares of x over the chunks [n, 2] (start, length <= 65,536) of a bf16 buffer: one launch for the partials
// and one for their ordered sum. Returns fp32 [1].
at::Tensor sq_norm_ranges(const at::Tensor& x, const at::Tensor& chunks) {
  FYB_RANGE("fyb::sq_norm_ranges");
  FYB_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "sq_norm_ranges: bf16 buffer");
  FYB_CHECK(chunks.is_cuda() && chunks.scalar_type() == at::kLong && chunks.is_contiguous() && chunks.dim() == 2 &&
                chunks.size(1) == 2,
            "sq_norm_ranges: chunks must be int64 [n, 2] on the device");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t n = chunks.size(0);
  auto out = at::zeros({1}, x.options().dtype(at::kFloat));
  if (n == 0) return out;
  FYB_CHECK(n < (1ll << 31), "sq_norm_ranges: too many chunks");
  auto part = at::empty({n}, x.options().dtype(at::kFloat));
  sq_ranges_kernel<<<static_cast<unsigned>(n), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), chunks.data_ptr<int64_t>(), part.data_ptr<float>());
  check_launch("sq_ranges");
  sq_final_kernel<<<1, 1024, 0, cur_stream()>>>(part.data_ptr<float>(), static_cast<int>(n), out.data_ptr<float>());
  check_launch("sq_final");
  return out;
}

at::Tensor sq_norm(const at::Tensor& x) {
  FYB_RANGE("fyb::sq_norm");
  FYB_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() &&
                reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
            "sq_norm: contiguous 16-byte aligned bf16 expected");
  c10::cuda::CUDAGuard guard(x.device());
  const int P = sq_norm_ctas(x.numel());
  auto part = at::empty({P}, x.options().dtype(at::kFloat));
  auto out = at::empty({1}, x.options().dtype(at::kFloat));
  sq_norm_into(x, part.data_ptr<float>(), P, out.data_ptr<float>());
  return out;
}

FYB_BOUNDS_BINDER(bind_bounds_elementwise)

}  // namespace fyb
