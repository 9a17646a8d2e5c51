// norm.cu -- the decoder block's elementwise steps as single launches:
//
//   residual add + RMSNorm  (model.py:34-38 rms_norm, and the residual adds of
//                            model.py:120-124, 298-301 that precede a norm)
//       x' = round(x + r)                     (skipped when r is null)
//       h  = round((x' * rsqrt(mean(x'^2) + eps)) * w)
//   SwiGLU activation       (model.py:70-74 swiglu_mlp, between its matmuls)
//       out = round(round(silu(g)) * u),  silu(g) = g / (1 + exp(-g))
//
// Each rounding is to the tensor dtype, at the same points as the unfused
// PyTorch expressions (a bf16 add rounds its fp32 sum; silu rounds before the
// product), with fp32 arithmetic in between.  In a decode step these replace
// ~8 launches per norm and 2 per activation: at batch 16 the step is a chain
// of small launches, so the count sets the token rate.
#include "common.cuh"
#include "kernels.h"

namespace pf {
namespace {

constexpr int kNormThreads = 128;

// One CTA per row (grid-strided).  Pass 1 forms x' (written to x_out when a
// residual is given) and the sum of squares; pass 2 re-reads x' -- the same
// thread wrote it, so x_out may alias x -- and writes h.
template <typename T>
__global__ void __launch_bounds__(kNormThreads)
add_rms_norm_kernel(const T* x, const T* __restrict__ res, const T* __restrict__ w, T* x_out,
                    T* __restrict__ h, long rows, int dim, float eps) {
  __shared__ float part[kNormThreads / 32];
  for (long row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + row * dim;
    T* xo = res != nullptr ? x_out + row * dim : nullptr;
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += kNormThreads) {
      float v = to_f(xr[i]);
      if (res != nullptr) {
        const T s = from_f<T>(v + to_f(res[row * dim + i]));
        xo[i] = s;
        v = to_f(s);
      }
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if (threadIdx.x % 32 == 0) part[threadIdx.x / 32] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < kNormThreads / 32; ++k) tot += part[k];
    __syncthreads();  // part[] is reused by the next row
    const float r = rsqrtf(tot / (float)dim + eps);
    const T* xs = res != nullptr ? xo : xr;
    for (int i = threadIdx.x; i < dim; i += kNormThreads)
      h[row * dim + i] = from_f<T>((to_f(xs[i]) * r) * to_f(w[i]));
  }
}

template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ out, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float a = to_f(g[i]);
    const T s = from_f<T>(a / (1.f + expf(-a)));
    out[i] = from_f<T>(to_f(s) * to_f(u[i]));
  }
}

template <typename T>
cudaError_t launch_norm_t(const void* x, const void* res, const void* w, void* x_out, void* h, long rows, int dim,
                          float eps, cudaStream_t st) {
  const long cap = (long)sm_count() * 16;
  const unsigned grid = (unsigned)(rows < cap ? rows : cap);
  add_rms_norm_kernel<T><<<grid, kNormThreads, 0, st>>>(static_cast<const T*>(x), static_cast<const T*>(res),
                                                        static_cast<const T*>(w), static_cast<T*>(x_out),
                                                        static_cast<T*>(h), rows, dim, eps);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_silu_t(const void* g, const void* u, void* out, long n, cudaStream_t st) {
  const int threads = 256;
  const long want = (n + threads - 1) / threads, cap = (long)sm_count() * 16;
  silu_mul_kernel<T><<<(unsigned)(want < cap ? want : cap), threads, 0, st>>>(
      static_cast<const T*>(g), static_cast<const T*>(u), static_cast<T*>(out), n);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_add_rms_norm(const void* x, const void* res, const void* w, void* x_out, void* h, int dtype,
                                long rows, int dim, float eps, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  switch (dtype) {
    case PF_F32: return launch_norm_t<float>(x, res, w, x_out, h, rows, dim, eps, st);
    case PF_BF16: return launch_norm_t<__nv_bfloat16>(x, res, w, x_out, h, rows, dim, eps, st);
    default: return launch_norm_t<__half>(x, res, w, x_out, h, rows, dim, eps, st);
  }
}

cudaError_t launch_silu_mul(const void* g, const void* u, void* out, int dtype, long n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  switch (dtype) {
    case PF_F32: return launch_silu_t<float>(g, u, out, n, st);
    case PF_BF16: return launch_silu_t<__nv_bfloat16>(g, u, out, n, st);
    default: return launch_silu_t<__half>(g, u, out, n, st);
  }
}

}  // namespace pf
