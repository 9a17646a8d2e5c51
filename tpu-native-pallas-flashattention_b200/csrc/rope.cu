// rope.cu -- standalone rotary embedding over [B, H, S, D] rows, and its
// inverse (the transpose of the rotation), for the differentiable RoPE
// attention path: forward rotates Q and K, backward maps the gradients of the
// rotated tensors back.
//
// y = x*cos + rotate_half(x)*sin with rotate_half([x1, x2]) = [-x2, x1]
// (fused_rope.py:43-50, model.py:41-67); row s of the [S, D] tables belongs to
// position s.  The inverse rotation is the same formula with sin negated.
// Arithmetic in fp32, one rounding to the output type.  out may alias x.
#include "common.cuh"
#include "kernels.h"

namespace pf {
namespace {

template <typename T>
__global__ void rope_apply_kernel(const T* __restrict__ x, const void* __restrict__ cos_t,
                                  const void* __restrict__ sin_t, int tdtype, T* out, long pairs, int S,
                                  int D, float sgn) {
  const int half = D / 2;
  for (long idx = blockIdx.x * (long)blockDim.x + threadIdx.x; idx < pairs; idx += (long)gridDim.x * blockDim.x) {
    const long row = idx / half;
    const int i = (int)(idx % half);
    const long s = row % S;
    const long base = row * D;
    const float x1 = to_f(x[base + i]), x2 = to_f(x[base + i + half]);
    const float c1 = load_any(cos_t, tdtype, s * D + i), s1 = sgn * load_any(sin_t, tdtype, s * D + i);
    const float c2 = load_any(cos_t, tdtype, s * D + i + half);
    const float s2 = sgn * load_any(sin_t, tdtype, s * D + i + half);
    out[base + i] = from_f<T>(rope_lo(x1, x2, c1, s1));
    out[base + i + half] = from_f<T>(rope_hi(x1, x2, c2, s2));
  }
}

template <typename T>
cudaError_t launch_t(const void* x, const void* c, const void* s, int tdtype, void* out, long rows, int S, int D,
                     bool inverse, cudaStream_t st) {
  const long pairs = rows * (D / 2);
  const int threads = 256;
  const long want = (pairs + threads - 1) / threads;
  const int blocks = (int)(want < 148L * 16 ? want : 148L * 16);
  rope_apply_kernel<T><<<blocks, threads, 0, st>>>(static_cast<const T*>(x), c, s, tdtype, static_cast<T*>(out),
                                                   pairs, S, D, inverse ? -1.f : 1.f);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_rope_apply(const void* x, const void* cos_t, const void* sin_t, int tdtype, void* out, int dtype,
                              long rows, int S, int D, bool inverse, cudaStream_t st) {
  switch (dtype) {
    case PF_F32: return launch_t<float>(x, cos_t, sin_t, tdtype, out, rows, S, D, inverse, st);
    case PF_BF16: return launch_t<__nv_bfloat16>(x, cos_t, sin_t, tdtype, out, rows, S, D, inverse, st);
    default: return launch_t<__half>(x, cos_t, sin_t, tdtype, out, rows, S, D, inverse, st);
  }
}

}  // namespace pf
