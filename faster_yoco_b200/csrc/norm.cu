// RMSNorm forward / backward and the per-head weightless RMSNorm fused with the retention output gate.
//
// Numerics follow the reference's RMSNorm (yoco/models/decoder/rms_norm.py:34-46): statistics in fp32,
// n = bf16(x * rsqrt(mean(x^2) + eps)), y = bf16(n * w) -- two bf16 roundings, as the upstream expression and its
// Triton port (yoco/models/decoder/rms_triton.py:19-63) produce. The weight gradient is reduced deterministically
// from per-CTA fp32 partials (no atomics), like the Triton kernel's per-program partials (:102).
//
// subln_swiglu: the retention output o [T, H*D] is normalised per head without weight (n16 = bf16(o * rstd_h)),
// then gated: out = bf16(g * n16 * sigmoid(g)) (gate_retention.py:101-107 with kernel/swiglu.py:4-9).
#include <ATen/ATen.h>
#include <c10/util/Optional.h>

#include <mutex>

#include "common/host.h"
#include "common/ptx.cuh"
#include "noalloc.h"

namespace fyb {
namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

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

// one CTA per row; N % 8 == 0
__global__ void rms_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                               __nv_bfloat16* __restrict__ y, float* __restrict__ rstd, int N, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * N;
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < N; c += blockDim.x * 8) {
    float f[8];
    load8(xr + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / static_cast<float>(N) + eps);
  if (threadIdx.x == 0) rstd[row] = r;
  for (int c = threadIdx.x * 8; c < N; c += blockDim.x * 8) {
    float f[8], o[8];
    load8(xr + c, f);
    if (w != nullptr) {
      float wf[8];
      load8(w + c, wf);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = bf16_round(f[i] * r) * wf[i];
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = f[i] * r;
    }
    store8(y + row * N + c, o);
  }
}

// rows [row0, row1) per CTA; dx per row; dw partial (fp32) per CTA in part[blockIdx.x, N]
__global__ void rms_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                               const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                               __nv_bfloat16* __restrict__ dx, float* __restrict__ part, int M, int N,
                               int rows_per_cta, const __nv_bfloat16* __restrict__ dres = nullptr) {
  __shared__ float red[32];
  extern __shared__ float dw_acc[];   // N floats (only when w != nullptr)
  if (w != nullptr)
    for (int c = threadIdx.x; c < N; c += blockDim.x) dw_acc[c] = 0.f;
  __syncthreads();
  const int row0 = blockIdx.x * rows_per_cta;
  const int row1 = min(M, row0 + rows_per_cta);
  for (int row = row0; row < row1; ++row) {
    const int64_t off = static_cast<int64_t>(row) * N;
    const float r = rstd[row];
    float dot = 0.f;
    for (int c = threadIdx.x * 8; c < N; c += blockDim.x * 8) {
      float g[8], f[8];
      load8(dy + off + c, g);
      load8(x + off + c, f);
      if (w != nullptr) {
        float wf[8];
        load8(w + c, wf);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float n = f[i] * r;
          const float dn = bf16_round(g[i] * wf[i]);
          dot += dn * n;
          dw_acc[c + i] += g[i] * bf16_round(n);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) dot += g[i] * f[i] * r;
      }
    }
    dot = block_sum(dot, red) / static_cast<float>(N);
    for (int c = threadIdx.x * 8; c < N; c += blockDim.x * 8) {
      float g[8], f[8], o[8];
      load8(dy + off + c, g);
      load8(x + off + c, f);
      if (w != nullptr) {
        float wf[8];
        load8(w + c, wf);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = r * (bf16_round(g[i] * wf[i]) - f[i] * r * dot);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = r * (g[i] - f[i] * r * dot);
      }
      if (dres != nullptr) {
        // gradient reaching x through the residual branch: bf16(dx_norm) + dres, as autograd's bf16 sum
        float rr[8];
        load8(dres + off + c, rr);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = bf16_round(o[i]) + rr[i];
      }
      store8(dx + off + c, o);
    }
  }
  if (w != nullptr) {
    __syncthreads();
    for (int c = threadIdx.x; c < N; c += blockDim.x) part[static_cast<int64_t>(blockIdx.x) * N + c] = dw_acc[c];
  }
}

// Register-resident RMSNorm backward for N <= 8192: one thread per 8 columns (blockDim = N/8 rounded up to a warp),
// so each row's dy / x values are read once and kept in registers between the row-dot reduction and the dx store,
// and the thread's 8 weight-gradient partials stay in registers over all rows of the CTA. The next row is loaded
// before the current row's reduction so its global loads overlap the barrier.
__global__ void rms_bwd_reg_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                   const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                                   __nv_bfloat16* __restrict__ dx, float* __restrict__ part, int M, int N,
                                   int rows_per_cta, const __nv_bfloat16* __restrict__ dres) {
  __shared__ float red[32];
  const int c = threadIdx.x * 8;
  const bool act = c < N;
  const int row0 = blockIdx.x * rows_per_cta;
  const int row1 = min(M, row0 + rows_per_cta);
  float wf[8], dw[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    wf[i] = 1.f;
    dw[i] = 0.f;
  }
  if (act && w != nullptr) load8(w + c, wf);
  uint4 gu = make_uint4(0, 0, 0, 0), xu = make_uint4(0, 0, 0, 0);
  if (act && row0 < row1) {
    gu = *reinterpret_cast<const uint4*>(dy + static_cast<int64_t>(row0) * N + c);
    xu = *reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row0) * N + c);
  }
  for (int row = row0; row < row1; ++row) {
    const int64_t off = static_cast<int64_t>(row) * N;
    float g[8], f[8];
    {
      const uint32_t gw[4] = {gu.x, gu.y, gu.z, gu.w}, xw[4] = {xu.x, xu.y, xu.z, xu.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = unpack_bf16(gw[i]), b = unpack_bf16(xw[i]);
        g[2 * i] = a.x;
        g[2 * i + 1] = a.y;
        f[2 * i] = b.x;
        f[2 * i + 1] = b.y;
      }
    }
    if (act && row + 1 < row1) {             // prefetch the next row
      gu = *reinterpret_cast<const uint4*>(dy + off + N + c);
      xu = *reinterpret_cast<const uint4*>(x + off + N + c);
    }
    const float r = rstd[row];
    float dot = 0.f;
    if (act) {
      if (w != nullptr) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float n = f[i] * r;
          dot += bf16_round(g[i] * wf[i]) * n;
          dw[i] += g[i] * bf16_round(n);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) dot += g[i] * f[i] * r;
      }
    }
    dot = block_sum(dot, red) / static_cast<float>(N);
    if (act) {
      float o[8];
      if (w != nullptr) {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = r * (bf16_round(g[i] * wf[i]) - f[i] * r * dot);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = r * (g[i] - f[i] * r * dot);
      }
      if (dres != nullptr) {
        float rr[8];
        load8(dres + off + c, rr);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = bf16_round(o[i]) + rr[i];
      }
      store8(dx + off + c, o);
    }
  }
  if (w != nullptr && act) {
    float* pp = part + static_cast<int64_t>(blockIdx.x) * N + c;
    *reinterpret_cast<float4*>(pp) = make_float4(dw[0], dw[1], dw[2], dw[3]);
    *reinterpret_cast<float4*>(pp + 4) = make_float4(dw[4], dw[5], dw[6], dw[7]);
  }
}

// dw[c] = bf16(sum_p part[p, c]): 32 columns x 8 row groups per CTA, each group sums rows p = g (mod 8) in order,
// then the 8 group sums are added in group order (a fixed order, independent of timing)
__global__ void col_sum8_kernel(const float* __restrict__ part, __nv_bfloat16* __restrict__ dw, int P, int N) {
  __shared__ float acc[8][33];
  const int col = blockIdx.x * 32 + (threadIdx.x & 31);
  const int grp = threadIdx.x >> 5;
  float s = 0.f;
  if (col < N)
    for (int p = grp; p < P; p += 8) s += part[static_cast<int64_t>(p) * N + col];
  acc[grp][threadIdx.x & 31] = s;
  __syncthreads();
  if (grp == 0 && col < N) {
    float t = 0.f;
#pragma unroll
    for (int g2 = 0; g2 < 8; ++g2) t += acc[g2][threadIdx.x];
    dw[col] = __float2bfloat16_rn(t);
  }
}

// dw[c] = bf16(sum_p part[p, c]) in a fixed order
__global__ void col_sum_kernel(const float* __restrict__ part, __nv_bfloat16* __restrict__ dw, int P, int N) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= N) return;
  float s = 0.f;
  for (int p = 0; p < P; ++p) s += part[static_cast<int64_t>(p) * N + c];
  dw[c] = __float2bfloat16_rn(s);
}

// ------------------------------------------------------------------------------------------------------------------
// subln (per-head RMSNorm, no weight) + swiglu(g, .)
// D/8 threads per (token, head) row; each thread 8 contiguous elements.

template <int D>
__global__ void subln_swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ g,
                                        int64_t ldg, __nv_bfloat16* __restrict__ out, float* __restrict__ rstd,
                                        int T, int H, float eps) {
  constexpr int TPR = D / 8;   // threads per head row
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t hrow = gid / TPR;   // (t, h) flattened
  const int sub = static_cast<int>(gid % TPR);
  const bool valid = hrow < static_cast<int64_t>(T) * H;
  const int64_t t = valid ? hrow / H : 0;
  const int h = valid ? static_cast<int>(hrow % H) : 0;
  float f[8];
  float ss = 0.f;
  if (valid) {
    load8(o + t * (static_cast<int64_t>(H) * D) + h * D + sub * 8, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
#pragma unroll
  for (int s = TPR / 2; s > 0; s >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, s);
  if (!valid) return;
  const float r = rsqrtf(ss / static_cast<float>(D) + eps);
  if (sub == 0) rstd[hrow] = r;
  float gv[8], res[8];
  load8(g + t * ldg + h * D + sub * 8, gv);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float n16 = bf16_round(f[i] * r);
    res[i] = gv[i] * n16 / (1.0f + __expf(-gv[i]));
  }
  store8(out + t * (static_cast<int64_t>(H) * D) + h * D + sub * 8, res);
}

template <int D>
__global__ void subln_swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ o,
                                        const __nv_bfloat16* __restrict__ g, int64_t ldg,
                                        const float* __restrict__ rstd, __nv_bfloat16* __restrict__ d_o,
                                        __nv_bfloat16* __restrict__ dg, int T, int H, int64_t lddg) {
  constexpr int TPR = D / 8;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t hrow = gid / TPR;
  const int sub = static_cast<int>(gid % TPR);
  const bool valid = hrow < static_cast<int64_t>(T) * H;
  const int64_t t = valid ? hrow / H : 0;
  const int h = valid ? static_cast<int>(hrow % H) : 0;
  const int64_t ooff = t * (static_cast<int64_t>(H) * D) + h * D + sub * 8;   // o, dout, d_o, dg: contiguous
  const int64_t goff = t * ldg + h * D + sub * 8;                              // g: strided view
  float f[8], gv[8], dv[8], dn[8];
  float dot = 0.f;
  float r = 0.f;
  if (valid) {
    r = rstd[hrow];
    load8(o + ooff, f);
    load8(g + goff, gv);
    load8(dout + ooff, dv);
    float dgo[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float n16 = bf16_round(f[i] * r);
      const float s = 1.0f / (1.0f + __expf(-gv[i]));
      dgo[i] = s * (1.0f + gv[i] * (1.0f - s)) * dv[i] * n16;
      dn[i] = bf16_round(gv[i] * s * dv[i]);
      dot += dn[i] * f[i] * r;
    }
    store8(dg + t * lddg + h * D + sub * 8, dgo);
  }
#pragma unroll
  for (int s = TPR / 2; s > 0; s >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, s);
  if (!valid) return;
  dot /= static_cast<float>(D);
  float res[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) res[i] = r * (dn[i] - f[i] * r * dot);
  store8(d_o + ooff, res);
}

}  // namespace

std::vector<at::Tensor> rms_norm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& w, double eps) {
  FYB_RANGE("fyb::rms_norm_fwd");
  FYB_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(),
            "rms_norm_fwd: contiguous bf16 [M, N] expected");
  const int64_t M = x.size(0), N = x.size(1);
  FYB_CHECK(N % 8 == 0, "rms_norm_fwd: N must be a multiple of 8");
  const __nv_bfloat16* wp = nullptr;
  if (w.has_value() && w->defined()) {
    FYB_CHECK(w->scalar_type() == at::kBFloat16 && w->numel() == N && w->is_contiguous(), "rms_norm_fwd: weight");
    wp = reinterpret_cast<const __nv_bfloat16*>(w->data_ptr());
  }
  c10::cuda::CUDAGuard guard(x.device());
  auto y = at::empty_like(x);
  auto rstd = at::empty({M}, x.options().dtype(at::kFloat));
  if (M > 0)
    rms_fwd_kernel<<<M, N >= 2048 ? kNormThreads : 128, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), wp, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()),
        rstd.data_ptr<float>(), static_cast<int>(N), static_cast<float>(eps));
  check_launch("rms_fwd");
  return {y, rstd};
}

// Gradient of RMSNorm. The weight gradient's per-CTA partials live in `part` (P x N fp32); pass an empty tensor to
// have it allocated here.
std::vector<at::Tensor> rms_norm_bwd_impl(const at::Tensor& dy, const at::Tensor& x, const c10::optional<at::Tensor>& w,
                                          const at::Tensor& rstd, float* part, int P,
                                          const __nv_bfloat16* dres = nullptr) {
  const int64_t M = x.size(0), N = x.size(1);
  const bool has_w = w.has_value() && w->defined();
  auto dx = at::empty_like(x);
  at::Tensor dw;
  if (has_w) dw = at::empty({N}, x.options());
  if (M == 0) {
    if (has_w) dw.zero_();
    return {dx, has_w ? dw : at::Tensor()};
  }
  const int rows_per = static_cast<int>((M + P - 1) / P);
  const int grid = static_cast<int>((M + rows_per - 1) / rows_per);
  if (N <= 8192) {
    const int threads = static_cast<int>((N / 8 + 31) / 32 * 32);
    rms_bwd_reg_kernel<<<grid, threads, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
        has_w ? reinterpret_cast<const __nv_bfloat16*>(w->data_ptr()) : nullptr, rstd.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), part, static_cast<int>(M), static_cast<int>(N), rows_per,
        dres);
    check_launch("rms_bwd_reg");
    if (has_w) {
      col_sum8_kernel<<<static_cast<int>((N + 31) / 32), 256, 0, cur_stream()>>>(
          part, reinterpret_cast<__nv_bfloat16*>(dw.data_ptr()), grid, static_cast<int>(N));
      check_launch("rms_bwd_colsum8");
    }
    return {dx, has_w ? dw : at::Tensor()};
  }
  const size_t shm = has_w ? N * sizeof(float) : 0;
  auto kern = rms_bwd_kernel;
  if (shm > 48 * 1024) FYB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)shm));
  kern<<<grid, kNormThreads, shm, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
      has_w ? reinterpret_cast<const __nv_bfloat16*>(w->data_ptr()) : nullptr, rstd.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), part, static_cast<int>(M), static_cast<int>(N), rows_per,
      dres);
  check_launch("rms_bwd");
  if (has_w) {
    col_sum_kernel<<<(N + 255) / 256, 256, 0, cur_stream()>>>(part, reinterpret_cast<__nv_bfloat16*>(dw.data_ptr()),
                                                             grid, static_cast<int>(N));
    check_launch("rms_bwd_colsum");
  }
  return {dx, has_w ? dw : at::Tensor()};
}

int rms_bwd_ctas(int64_t M) { return static_cast<int>(std::min<int64_t>(M, 2 * num_sms())); }

std::vector<at::Tensor> rms_norm_bwd(const at::Tensor& dy, const at::Tensor& x, const c10::optional<at::Tensor>& w,
                                     const at::Tensor& rstd, const c10::optional<at::Tensor>& dres) {
  FYB_RANGE("fyb::rms_norm_bwd");
  FYB_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous() &&
                dy.is_contiguous() && dy.sizes() == x.sizes() && dy.scalar_type() == at::kBFloat16,
            "rms_norm_bwd: contiguous bf16 [M, N] expected");
  FYB_CHECK(x.size(1) % 8 == 0, "rms_norm_bwd: N must be a multiple of 8");
  c10::cuda::CUDAGuard guard(x.device());
  const int P = std::max(rms_bwd_ctas(x.size(0)), 1);
  const bool has_w = w.has_value() && w->defined();
  at::Tensor part;
  if (has_w) part = at::empty({P, x.size(1)}, x.options().dtype(at::kFloat));
  const __nv_bfloat16* dr = nullptr;
  if (dres.has_value() && dres->defined()) {
    FYB_CHECK(dres->is_contiguous() && dres->sizes() == x.sizes() && dres->scalar_type() == at::kBFloat16,
              "rms_norm_bwd: dres must be contiguous bf16 like x");
    dr = reinterpret_cast<const __nv_bfloat16*>(dres->data_ptr());
  }
  return rms_norm_bwd_impl(dy, x, w, rstd, has_w ? part.data_ptr<float>() : nullptr, P, dr);
}

std::vector<at::Tensor> subln_swiglu_fwd(const at::Tensor& o, const at::Tensor& g, double eps, int64_t D) {
  FYB_RANGE("fyb::subln_swiglu_fwd");
  FYB_CHECK(o.is_cuda() && o.scalar_type() == at::kBFloat16 && o.dim() == 2 && o.is_contiguous(),
            "subln_swiglu_fwd: o must be contiguous bf16 [T, H*D]");
  FYB_CHECK(g.scalar_type() == at::kBFloat16 && g.dim() == 2 && g.stride(1) == 1 && g.sizes() == o.sizes() &&
                g.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(g.data_ptr()) % 16 == 0,
            "subln_swiglu_fwd: g must be bf16 [T, H*D] with 16-byte aligned rows");
  const int64_t T = o.size(0), HD = o.size(1);
  FYB_CHECK(D == 64 || D == 128, "subln_swiglu: head_dim 64 or 128");
  const int H = static_cast<int>(HD / D);
  c10::cuda::CUDAGuard guard(o.device());
  auto out = at::empty_like(o);
  auto rstd = at::empty({T, H}, o.options().dtype(at::kFloat));
  const int64_t threads = T * H * (D / 8);
  const int blocks = static_cast<int>((threads + 255) / 256);
  if (T > 0) {
    if (D == 128)
      subln_swiglu_fwd_kernel<128><<<blocks, 256, 0, cur_stream()>>>(
          reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()),
          g.stride(0), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rstd.data_ptr<float>(), (int)T, H, (float)eps);
    else
      subln_swiglu_fwd_kernel<64><<<blocks, 256, 0, cur_stream()>>>(
          reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()),
          g.stride(0), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rstd.data_ptr<float>(), (int)T, H, (float)eps);
  }
  check_launch("subln_swiglu_fwd");
  return {out, rstd};
}

std::vector<at::Tensor> subln_swiglu_bwd(const at::Tensor& dout, const at::Tensor& o, const at::Tensor& g,
                                         const at::Tensor& rstd, int64_t D, const c10::optional<at::Tensor>& dg_out) {
  FYB_RANGE("fyb::subln_swiglu_bwd");
  FYB_CHECK(dout.is_contiguous() && dout.sizes() == o.sizes(), "subln_swiglu_bwd: dout");
  const int64_t T = o.size(0), HD = o.size(1);
  const int H = static_cast<int>(HD / D);
  c10::cuda::CUDAGuard guard(o.device());
  auto d_o = at::empty_like(o);
  at::Tensor dg;
  if (dg_out.has_value() && dg_out->defined()) {
    dg = *dg_out;
    FYB_CHECK(dg.sizes() == o.sizes() && dg.stride(1) == 1 && dg.stride(0) % 8 == 0, "subln_swiglu_bwd: dg_out");
  } else {
    dg = at::empty({T, HD}, o.options());
  }
  const int64_t threads = T * H * (D / 8);
  const int blocks = static_cast<int>((threads + 255) / 256);
  if (T > 0) {
    if (D == 128)
      subln_swiglu_bwd_kernel<128><<<blocks, 256, 0, cur_stream()>>>(
          reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
          reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()),
          g.stride(0), rstd.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(d_o.data_ptr()),
          reinterpret_cast<__nv_bfloat16*>(dg.data_ptr()), (int)T, H, dg.stride(0));
    else
      subln_swiglu_bwd_kernel<64><<<blocks, 256, 0, cur_stream()>>>(
          reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
          reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()),
          g.stride(0), rstd.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(d_o.data_ptr()),
          reinterpret_cast<__nv_bfloat16*>(dg.data_ptr()), (int)T, H, dg.stride(0));
  }
  check_launch("subln_swiglu_bwd");
  return {d_o, dg};
}

}  // namespace fyb

// ------------------------------------------------------------------------------------------------------------------
// Allocation-free RMSNorm backward (declared and documented in noalloc.h; no counterpart in the reference).

namespace {
constexpr int kNoAllocMaxCtas = 64;
constexpr int kNoAllocMaxN = 8192;
}  // namespace

// the partial sums of the weight gradient: one row of N floats per block, at most 64 blocks (2 MiB per device)
static __device__ __align__(256) float g_fyb_rms_bwd_scratch[kNoAllocMaxCtas * kNoAllocMaxN];

namespace {
std::mutex g_noalloc_mu;
float* g_noalloc_scratch[64] = {nullptr};

// device address of the scratch array for the current device (looked up once per device, then cached)
int noalloc_scratch(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 5;
  if (dev < 0 || dev >= 64) return 5;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_scratch[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fyb_rms_bwd_scratch) != cudaSuccess || p == nullptr) return 4;
    g_noalloc_scratch[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_scratch[dev];
  return 0;
}
}  // namespace

extern "C" int fyb_rms_norm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* rstd, void* dx,
                                        void* dw, int64_t M, int64_t N, cudaStream_t stream) {
  using namespace fyb;
  if (N <= 0 || N > kNoAllocMaxN) return 1;
  if (N % 8 != 0) return 2;
  if (M < 0) return 2;
  if ((w == nullptr) != (dw == nullptr)) return 2;
  for (const void* p : {dy, x, static_cast<const void*>(dx)})
    if (p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 != 0) return 3;
  if (w != nullptr && reinterpret_cast<uintptr_t>(w) % 16 != 0) return 3;
  if (rstd == nullptr && M > 0) return 3;
  // an error left pending by the caller's earlier work is reported as such (code 7), not taken for our launch's
  if (cudaPeekAtLastError() != cudaSuccess) return 7;
  float* part = nullptr;
  if (w != nullptr) {
    const int rc = noalloc_scratch(&part);
    if (rc != 0) return rc;
  }
  if (M == 0) {
    if (dw != nullptr && cudaMemsetAsync(dw, 0, static_cast<size_t>(N) * 2, stream) != cudaSuccess) return 6;
    return 0;
  }
  const int P = static_cast<int>(std::min<int64_t>(M, kNoAllocMaxCtas));
  const int rows_per = static_cast<int>((M + P - 1) / P);
  const int grid = static_cast<int>((M + rows_per - 1) / rows_per);
  const size_t shm = w != nullptr ? static_cast<size_t>(N) * sizeof(float) : 0;
  rms_bwd_kernel<<<grid, kNormThreads, shm, stream>>>(
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x),
      static_cast<const __nv_bfloat16*>(w), rstd, static_cast<__nv_bfloat16*>(dx), part, static_cast<int>(M),
      static_cast<int>(N), rows_per);
  if (cudaGetLastError() != cudaSuccess) return 6;
  if (w != nullptr) {
    col_sum_kernel<<<static_cast<int>((N + 255) / 256), 256, 0, stream>>>(part, static_cast<__nv_bfloat16*>(dw), grid,
                                                                         static_cast<int>(N));
    if (cudaGetLastError() != cudaSuccess) return 6;
  }
  return 0;
}

extern "C" const char* fyb_noalloc_strerror(int code) {
  switch (code) {
    case 0: return "ok";
    case 1: return "N is beyond the static scratch limit: at most 8192 columns";
    case 2: return "invalid size: N must be a positive multiple of 8, M >= 0, and w / dw both given or both NULL";
    case 3: return "a pointer is NULL or not 16-byte aligned";
    case 4: return "cudaGetSymbolAddress of the static scratch array failed";
    case 5: return "no valid current CUDA device";
    case 6: return "kernel launch failed";
    case 7: return "a CUDA error from earlier work was already pending on entry (left pending, nothing launched)";
    default: return "unknown error code";
  }
}

