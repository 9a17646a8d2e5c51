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
// product), with fp32 arithmetic in between.  A third kernel advances a
// CUDA-graph decode step's position on the device, and a fourth ends the
// step: greedy token choice plus the next step's embedding row.  In a decode step these replace
// ~8 launches per norm and 2 per activation: at batch 16 the step is a chain
// of small launches, so the count sets the token rate.
#include <climits>
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

// Rows whose size is 32 * V 16-byte vectors: one warp per row, the row held in
// registers, every load issued before the first use (one memory round trip
// for x, the residual and the weight; a warp-shuffle reduction).  At decode
// sizes (16 rows of 512) the launch is latency-bound, which this shape minimises.
template <typename T, int V>
__global__ void __launch_bounds__(128)
add_rms_norm_warp_kernel(const uint4* x, const uint4* __restrict__ res, const uint4* __restrict__ w, uint4* x_out,
                         uint4* __restrict__ h, long rows, int dim, float eps) {
  constexpr int E = 16 / sizeof(T);
  const long row = (long)blockIdx.x * 4 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;  // uniform over the warp
  const long base = row * 32 * V;
  uint4 xv[V], rv[V], wv[V];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    xv[v] = x[base + v * 32 + lane];
    if (res != nullptr) rv[v] = res[base + v * 32 + lane];
    wv[v] = __ldg(w + v * 32 + lane);
  }
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    T* xe = reinterpret_cast<T*>(&xv[v]);
    if (res != nullptr) {
      const T* re = reinterpret_cast<const T*>(&rv[v]);
#pragma unroll
      for (int e = 0; e < E; ++e) xe[e] = from_f<T>(to_f(xe[e]) + to_f(re[e]));
    }
#pragma unroll
    for (int e = 0; e < E; ++e) ss = fmaf(to_f(xe[e]), to_f(xe[e]), ss);
  }
  if (res != nullptr) {
#pragma unroll
    for (int v = 0; v < V; ++v) x_out[base + v * 32 + lane] = xv[v];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)dim + eps);
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const T* xe = reinterpret_cast<const T*>(&xv[v]);
    const T* we = reinterpret_cast<const T*>(&wv[v]);
    uint4 o;
    T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int e = 0; e < E; ++e) oe[e] = from_f<T>((to_f(xe[e]) * r) * to_f(we[e]));
    h[base + v * 32 + lane] = o;
  }
}

// out[r, c] = round(round(silu(gate[r, c])) * up[r, c]) over rows x cols;
// gate and up rows are in_stride elements apart (both halves of one fused
// [rows, 2 * cols] projection, or two contiguous tensors with in_stride = cols).
template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ out, long rows,
                                int cols, long in_stride) {
  const long n = rows * cols;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long r = i / cols, src = r * in_stride + (i - r * cols);
    const float a = to_f(g[src]);
    const T s = from_f<T>(a / (1.f + expf(-a)));
    out[i] = from_f<T>(to_f(s) * to_f(u[src]));
  }
}

// Device-side bookkeeping of one decode step at position p = *pos (then
// *pos = p + 1): cache slot p % C, live length min(p + 1, C) and RoPE row p
// for each of the B sequences (ring slots: model.py:434-449, 475-476).
__global__ void decode_positions_kernel(int64_t* pos, int C, int32_t* slots, int32_t* lens, int32_t* rope_rows,
                                        int B) {
  const int64_t p = *pos;
  __syncthreads();  // every thread has read p before it is advanced
  if (threadIdx.x == 0) *pos = p + 1;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    slots[b] = (int32_t)(p % C);
    lens[b] = (int32_t)(p + 1 < C ? p + 1 : C);
    rope_rows[b] = (int32_t)p;
  }
}

template <typename T, int V>
void launch_norm_warp(const void* x, const void* res, const void* w, void* x_out, void* h, long rows, int dim,
                      float eps, cudaStream_t st) {
  add_rms_norm_warp_kernel<T, V><<<(unsigned)((rows + 3) / 4), 128, 0, st>>>(
      static_cast<const uint4*>(x), static_cast<const uint4*>(res), static_cast<const uint4*>(w),
      static_cast<uint4*>(x_out), static_cast<uint4*>(h), rows, dim, eps);
}

// Greedy-decode tail, one CTA per row b: token[b] = argmax_v logits[b, v] --
// the first index of the maximum, a NaN ranking above every number (the
// torch.argmax / jnp.argmax rule) -- and, when embed is given, x[b, :] =
// embed[token[b], :], the next decode step's input row.
struct ArgBest {
  float f;
  int i;
  bool nan;
};
__device__ __forceinline__ bool arg_beats(const ArgBest& a, const ArgBest& b) {
  if (a.nan != b.nan) return a.nan;
  if (!a.nan && a.f != b.f) return a.f > b.f;
  return a.i < b.i;
}
constexpr int kArgThreads = 512;
template <typename T>
__global__ void __launch_bounds__(kArgThreads)
argmax_embed_kernel(const T* __restrict__ logits, long row_stride, int vocab, int64_t* __restrict__ token,
                    const T* __restrict__ embed, T* __restrict__ x, int dim) {
  __shared__ ArgBest part[kArgThreads / 32];
  __shared__ int winner;
  const int b = blockIdx.x;
  const T* row = logits + (long)b * row_stride;
  ArgBest best{-INFINITY, INT_MAX, false};
  constexpr int E = 16 / sizeof(T);  // elements per 16-byte vector
  if (reinterpret_cast<uintptr_t>(row) % 16 == 0 && vocab % E == 0) {
    // 16-byte loads, four vectors per thread in flight before any compare
    // (arg_beats orders candidates by value, then index, so the scan order
    // does not change the winner).
    const int nvec = vocab / E;
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    for (int base = threadIdx.x; base < nvec; base += 4 * kArgThreads) {
      uint4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int iv = base + u * kArgThreads;
        q[u] = iv < nvec ? rv[iv] : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int iv = base + u * kArgThreads;
        if (iv >= nvec) continue;
        const T* e = reinterpret_cast<const T*>(&q[u]);
#pragma unroll
        for (int k = 0; k < E; ++k) {
          const float f = to_f(e[k]);
          const ArgBest c{f, iv * E + k, f != f};
          if (arg_beats(c, best)) best = c;
        }
      }
    }
  } else {
    for (int v = threadIdx.x; v < vocab; v += kArgThreads) {
      const float f = to_f(row[v]);
      const ArgBest c{f, v, f != f};
      if (arg_beats(c, best)) best = c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgBest c;
    c.f = __shfl_xor_sync(0xffffffffu, best.f, o);
    c.i = __shfl_xor_sync(0xffffffffu, best.i, o);
    c.nan = __shfl_xor_sync(0xffffffffu, (int)best.nan, o) != 0;
    if (arg_beats(c, best)) best = c;
  }
  if (threadIdx.x % 32 == 0) part[threadIdx.x / 32] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    ArgBest w = part[0];
    for (int k = 1; k < kArgThreads / 32; ++k)
      if (arg_beats(part[k], w)) w = part[k];
    const int t = w.i == INT_MAX ? 0 : w.i;  // vocab == 0 cannot reach here
    token[b] = t;
    winner = t;
  }
  __syncthreads();
  if (embed != nullptr) {
    const T* src = embed + (long)winner * dim;
    for (int d = threadIdx.x; d < dim; d += kArgThreads) x[(long)b * dim + d] = src[d];
  }
}

template <typename T>
cudaError_t launch_norm_t(const void* x, const void* res, const void* w, void* x_out, void* h, long rows, int dim,
                          float eps, cudaStream_t st) {
  const uintptr_t ptrs = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(res) |
                         reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x_out) |
                         reinterpret_cast<uintptr_t>(h);
  const long vecs = (long)dim * (long)sizeof(T) / 16;
  if (ptrs % 16 == 0 && (long)dim * (long)sizeof(T) % 512 == 0) {
    switch (vecs / 32) {
      case 1: launch_norm_warp<T, 1>(x, res, w, x_out, h, rows, dim, eps, st); return cudaGetLastError();
      case 2: launch_norm_warp<T, 2>(x, res, w, x_out, h, rows, dim, eps, st); return cudaGetLastError();
      case 4: launch_norm_warp<T, 4>(x, res, w, x_out, h, rows, dim, eps, st); return cudaGetLastError();
      case 8: launch_norm_warp<T, 8>(x, res, w, x_out, h, rows, dim, eps, st); return cudaGetLastError();
      default: break;
    }
  }
  const long cap = (long)sm_count() * 16;
  const unsigned grid = (unsigned)(rows < cap ? rows : cap);
  add_rms_norm_kernel<T><<<grid, kNormThreads, 0, st>>>(static_cast<const T*>(x), static_cast<const T*>(res),
                                                        static_cast<const T*>(w), static_cast<T*>(x_out),
                                                        static_cast<T*>(h), rows, dim, eps);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_silu_t(const void* g, const void* u, void* out, long rows, int cols, long in_stride,
                          cudaStream_t st) {
  const int threads = 256;
  const long n = rows * cols;
  const long want = (n + threads - 1) / threads, cap = (long)sm_count() * 16;
  silu_mul_kernel<T><<<(unsigned)(want < cap ? want : cap), threads, 0, st>>>(
      static_cast<const T*>(g), static_cast<const T*>(u), static_cast<T*>(out), rows, cols, in_stride);
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

cudaError_t launch_silu_mul(const void* g, const void* u, void* out, int dtype, long rows, int cols, long in_stride,
                            cudaStream_t st) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  switch (dtype) {
    case PF_F32: return launch_silu_t<float>(g, u, out, rows, cols, in_stride, st);
    case PF_BF16: return launch_silu_t<__nv_bfloat16>(g, u, out, rows, cols, in_stride, st);
    default: return launch_silu_t<__half>(g, u, out, rows, cols, in_stride, st);
  }
}

cudaError_t launch_argmax_embed(const void* logits, long row_stride, int vocab, int rows, int64_t* token,
                                const void* embed, void* x, int dim, int dtype, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
#define PF_AE(T)                                                                                              \
  argmax_embed_kernel<T><<<rows, kArgThreads, 0, st>>>(static_cast<const T*>(logits), row_stride, vocab, token, \
                                                       static_cast<const T*>(embed), static_cast<T*>(x), dim)
  if (dtype == PF_F32) PF_AE(float);
  else if (dtype == PF_BF16) PF_AE(__nv_bfloat16);
  else PF_AE(__half);
#undef PF_AE
  return cudaGetLastError();
}

cudaError_t launch_decode_positions(int64_t* pos, int C, int32_t* slots, int32_t* lens, int32_t* rope_rows, int B,
                                    cudaStream_t st) {
  decode_positions_kernel<<<1, 256, 0, st>>>(pos, C, slots, lens, rope_rows, B);
  return cudaGetLastError();
}

}  // namespace pf
