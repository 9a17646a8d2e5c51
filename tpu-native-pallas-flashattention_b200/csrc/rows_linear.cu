// rows_linear.cu -- the projections of a batched decode step (at most 16 rows)
// with their neighbouring elementwise steps folded in:
//
//   y = epilogue( prologue(x) @ W )        x: [M, K], W given as W^T: [N_w, K]
//
//   prologue  RMSNorm of each row (when a norm weight is given):
//               a = round((x * rsqrt(mean(x^2) + eps)) * w)      (model.py:34-38)
//   epilogue  0: y = round(acc)                                 (x @ W)
//             1: y = round(res + round(acc))                    (the residual add
//                after the attention output / MLP projections, model.py:120-124)
//             2: y = round(round(silu(round(acc_g))) * round(acc_u)), gate columns
//                in W^T rows [0, N), up columns in rows [N, 2N)   (swiglu_mlp,
//                model.py:70-74)
//
// Each rounding is where the unfused expression (a dtype matmul, then the norm /
// residual-add / activation kernels of norm.cu) rounds, with fp32 in between.
// At batch 16 the decode step is a chain of small launches; folding the norm
// and the activation into the projections takes a launch off every one of
// them.  The GEMM is tiny (M <= 16) and its weights sit in L2, so the kernel
// is latency-shaped: every CTA issues all of its weight loads first (one
// round trip), normalises the 16 rows while they are in flight, and runs
// m16n8k16 MMAs.
//
// Each launch is a programmatic dependent launch: its CTAs may start while the
// previous kernel on the stream finishes, issue their (constant) weight loads,
// and wait (griddepcontrol.wait) before reading activations or writing
// anything; the kernel lets its own dependents launch right after that wait.
//
// CTA = 32 output columns (16 in mode 2: 16 gate + 16 up weight rows), 8 warps
// that split K in 32-element units; the warps' fp32 partials are summed in a
// fixed order in shared memory (deterministic).  Inside a 32-element unit a
// lane holds k = 8c .. 8c + 7 (c = lane % 4) of both operands, one 16-byte
// load each; the MMA's k order is permuted the same way for A and B, so the
// dot products are unchanged.
#include <climits>
#include <type_traits>
#include "common.cuh"
#include "kernels.h"

namespace pf {
namespace {

// Mode 3: the fused q/k/v projection of one decode token per sequence, with
// RoPE and the K/V cache write as its epilogue (the arithmetic and addressing
// of rope_paged_write_kernel).  A CTA owns 16 rotation pairs (d, d + D/2) of
// one head: weight rows [head*D + 16s, +16) and [head*D + D/2 + 16s, +16).
struct RlRope {
  void* q_out;             // [M, H, 1, D]
  void* k_pages;           // [num_pages, Hkv, page_size, D]
  void* v_pages;
  const void* cos_t;       // [table_rows, D] (tdtype)
  const void* sin_t;
  const int32_t* tables;   // [M, pages_per_seq]
  const int32_t* positions;  // cache position written, per sequence
  const int32_t* rope_pos;   // RoPE table row, per sequence
  int tdtype, table_rows, H, Hkv, num_pages, page_size, pages_per_seq, D;
};

constexpr int kRlThreads = 256;
constexpr int kRlWarps = kRlThreads / 32;
constexpr int kRlCols = 32;     // weight rows (output features) per CTA
constexpr int kRlMaxUnits = 8;  // 32-element K units per warp: K <= 8 * 8 * 32 = 2048
static_assert(16 * kRlCols == 2 * kRlThreads, "the epilogue gives each thread two of the 16 x 32 outputs");
// Kernels are instantiated for at most 2, 4, 6 or 8 units per warp (K <= 512,
// 1024, 1536, 2048), so the weight registers of a short K are not reserved for a long one.

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

template <typename T, int MAXU>
__global__ void __launch_bounds__(kRlThreads)
rows_linear_kernel(const T* __restrict__ x, const T* __restrict__ norm_w, float eps, const T* __restrict__ wt,
                   const T* res, T* y, int M, int K, int N, int mode, RlRope rp) {
  extern __shared__ __align__(16) uint8_t rl_smem[];
  const int lda = K + 8;  // row stride of the A tile in elements (16 B of padding: no bank conflicts)
  T* A = reinterpret_cast<T*>(rl_smem);
  float* red = reinterpret_cast<float*>(rl_smem + (size_t)16 * lda * sizeof(T));  // [warps][16][32]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = lane / 4, c = lane % 4;

  // Weight rows of this CTA's four 8-row n-tiles.
  const int cb = blockIdx.x * (mode >= 2 ? kRlCols / 2 : kRlCols);
  int wrow[4];
  if (mode == 3) {
    const int per_head = rp.D / 32, head = blockIdx.x / per_head, s16 = 16 * (blockIdx.x % per_head);
#pragma unroll
    for (int t = 0; t < 4; ++t) wrow[t] = head * rp.D + (t >= 2 ? rp.D / 2 : 0) + s16 + 8 * (t & 1) + g;
  } else {
#pragma unroll
    for (int t = 0; t < 4; ++t) wrow[t] = (mode == 2 && t >= 2) ? N + cb + 8 * (t - 2) + g : cb + 8 * t + g;
  }

  // This warp's K units [u0, u1); every weight load is issued before the prologue.
  const int U = K / 32;
  const int u0 = U * warp / kRlWarps, u1 = U * (warp + 1) / kRlWarps;
  uint4 bq[MAXU][4];
#pragma unroll
  for (int i = 0; i < MAXU; ++i) {
    if (u0 + i < u1) {
#pragma unroll
      for (int t = 0; t < 4; ++t)
        bq[i][t] = __ldg(reinterpret_cast<const uint4*>(wt + (size_t)wrow[t] * K + (u0 + i) * 32 + 8 * c));
    }
  }

  // Launched as a programmatic dependent of the previous kernel on the stream:
  // the weights above are constants, everything below reads or writes data
  // that kernel may produce or consume, so wait for its completion here.  The
  // next kernel may launch now (it waits the same way before touching ours).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // The epilogue's residual values (mode 1) are fetched now as well.
  T resv[2];
  if (mode == 1) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int o = threadIdx.x + q * kRlThreads, r = o / kRlCols, j = o % kRlCols;
      resv[q] = r < M ? res[(size_t)r * N + cb + j] : from_f<T>(0.f);
    }
  }

  // Prologue: warp w stages rows w and w + 8 (zeros past M), normalised when a
  // norm weight is given -- the same lane/element order and reduction as
  // add_rms_norm_warp_kernel, so the staged rows equal its output.  A lane
  // holds vectors lane, lane + 32, ... of a row (at most MAXU: K <= 256 MAXU),
  // all loaded before the first use.
  {
    uint4 xv[2][MAXU], wv[MAXU];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = warp + h * kRlWarps;
      const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)r * K);
#pragma unroll
      for (int v = 0; v < MAXU; ++v) {
        const int i = lane + 32 * v;
        xv[h][v] = (r < M && i < K / 8) ? xr[i] : make_uint4(0, 0, 0, 0);
      }
    }
    if (norm_w != nullptr) {
#pragma unroll
      for (int v = 0; v < MAXU; ++v) {
        const int i = lane + 32 * v;
        wv[v] = i < K / 8 ? __ldg(reinterpret_cast<const uint4*>(norm_w) + i) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = warp + h * kRlWarps;
      T* ar = A + (size_t)r * lda;
      if (norm_w != nullptr && r < M) {
        float ss = 0.f;
#pragma unroll
        for (int v = 0; v < MAXU; ++v) {
          const T* e = reinterpret_cast<const T*>(&xv[h][v]);
#pragma unroll
          for (int q = 0; q < 8; ++q) ss = fmaf(to_f(e[q]), to_f(e[q]), ss);
        }
        ss = warp_sum(ss);
        const float rs = rsqrtf(ss / (float)K + eps);
#pragma unroll
        for (int v = 0; v < MAXU; ++v) {
          const T* e = reinterpret_cast<const T*>(&xv[h][v]);
          const T* we = reinterpret_cast<const T*>(&wv[v]);
          T* oe = reinterpret_cast<T*>(&xv[h][v]);
#pragma unroll
          for (int q = 0; q < 8; ++q) oe[q] = from_f<T>((to_f(e[q]) * rs) * to_f(we[q]));
        }
      }
#pragma unroll
      for (int v = 0; v < MAXU; ++v) {
        const int i = lane + 32 * v;
        if (i < K / 8) *reinterpret_cast<uint4*>(ar + 8 * i) = xv[h][v];
      }
    }
  }
  __syncthreads();

  float acc[4][4];
#pragma unroll
  for (int t = 0; t < 4; ++t)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[t][q] = 0.f;
#pragma unroll
  for (int i = 0; i < MAXU; ++i) {
    if (u0 + i < u1) {
      const int k = (u0 + i) * 32 + 8 * c;
      const uint4 lo = *reinterpret_cast<const uint4*>(A + (size_t)g * lda + k);
      const uint4 hi = *reinterpret_cast<const uint4*>(A + (size_t)(g + 8) * lda + k);
      // k-step 0: elements 0-3 of the lane's 8; k-step 1: elements 4-7.
      const uint32_t a0[4] = {lo.x, hi.x, lo.y, hi.y};
      const uint32_t a1[4] = {lo.z, hi.z, lo.w, hi.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        mma16816<T>(acc[t], a0, bq[i][t].x, bq[i][t].y);
        mma16816<T>(acc[t], a1, bq[i][t].z, bq[i][t].w);
      }
    }
  }
  // Partials: red[warp][row][col], col = 8t + 2c + {0, 1}.
  float* rw = red + warp * 16 * kRlCols;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    rw[g * kRlCols + 8 * t + 2 * c] = acc[t][0];
    rw[g * kRlCols + 8 * t + 2 * c + 1] = acc[t][1];
    rw[(g + 8) * kRlCols + 8 * t + 2 * c] = acc[t][2];
    rw[(g + 8) * kRlCols + 8 * t + 2 * c + 1] = acc[t][3];
  }
  __syncthreads();
  auto total = [&](int r, int j) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kRlWarps; ++w) s += red[(w * 16 + r) * kRlCols + j];
    return s;
  };
  if (mode == 3) {
    const int r = threadIdx.x / 16, j = threadIdx.x % 16;  // 16 rows x 16 rotation pairs
    if (r < M) {
      const int D = rp.D, half = D / 2, per_head = D / 32;
      const int head = blockIdx.x / per_head, i = 16 * (blockIdx.x % per_head) + j;
      const float x1 = to_f(from_f<T>(total(r, j))), x2 = to_f(from_f<T>(total(r, j + 16)));
      const long tr = min(max(rp.rope_pos[r], 0), rp.table_rows - 1);
      const float c1 = load_any(rp.cos_t, rp.tdtype, tr * D + i), s1 = load_any(rp.sin_t, rp.tdtype, tr * D + i);
      const float c2 = load_any(rp.cos_t, rp.tdtype, tr * D + i + half);
      const float s2 = load_any(rp.sin_t, rp.tdtype, tr * D + i + half);
      if (head < rp.H) {
        T* q = static_cast<T*>(rp.q_out) + ((long)r * rp.H + head) * D;
        q[i] = from_f<T>(rope_lo(x1, x2, c1, s1));
        q[i + half] = from_f<T>(rope_hi(x1, x2, c2, s2));
      } else {
        const int hk = head < rp.H + rp.Hkv ? head - rp.H : head - rp.H - rp.Hkv;
        const int pos = rp.positions[r], ps = rp.page_size;
        const int lp = min(max(pos / ps, 0), rp.pages_per_seq - 1);
        const int off = pos - (pos / ps) * ps;
        int page = rp.tables[(long)r * rp.pages_per_seq + lp];
        page = min(max(page, 0), rp.num_pages - 1);
        const long dst = (((long)page * rp.Hkv + hk) * ps + off) * D;
        if (head < rp.H + rp.Hkv) {
          T* kp = static_cast<T*>(rp.k_pages);
          kp[dst + i] = from_f<T>(rope_lo(x1, x2, c1, s1));
          kp[dst + i + half] = from_f<T>(rope_hi(x1, x2, c2, s2));
        } else {
          T* vp = static_cast<T*>(rp.v_pages);
          vp[dst + i] = from_f<T>(x1);
          vp[dst + i + half] = from_f<T>(x2);
        }
      }
    }
  } else if (mode == 2) {
    const int r = threadIdx.x / 16, j = threadIdx.x % 16;  // 256 threads = 16 rows x 16 columns
    if (r < M) {
      const float gv = to_f(from_f<T>(total(r, j))), uv = to_f(from_f<T>(total(r, j + 16)));
      const T s = from_f<T>(gv / (1.f + expf(-gv)));
      y[(size_t)r * N + cb + j] = from_f<T>(to_f(s) * uv);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int o = threadIdx.x + q * kRlThreads, r = o / kRlCols, j = o % kRlCols;
      if (r >= M) continue;
      const T v = from_f<T>(total(r, j));
      y[(size_t)r * N + cb + j] = mode == 1 ? from_f<T>(to_f(resv[q]) + to_f(v)) : v;
    }
  }
}

}  // namespace

size_t rows_linear_smem(int K) { return (size_t)16 * (K + 8) * 2 + (size_t)kRlWarps * 16 * kRlCols * 4; }

bool rows_linear_supported(int dtype, int M, int K, int N, int mode) {
  if (!(dtype == PF_BF16 || dtype == PF_F16)) return false;
  if (M < 1 || M > 16 || K < 32 || K % 32 != 0 || K > kRlWarps * kRlMaxUnits * 32) return false;
  if (mode < 0 || mode > 2) return false;
  return N > 0 && N % (mode == 2 ? kRlCols / 2 : kRlCols) == 0;
}

bool rows_linear_rope_supported(int dtype, int M, int K, int H, int Hkv, int D) {
  return rows_linear_supported(dtype, M, K, 32, 0) && H > 0 && Hkv > 0 && D >= 32 && D % 32 == 0;
}

static cudaError_t launch_rl(const void* x, const void* norm_w, float eps, const void* wt, const void* res, void* y,
                             int dtype, int M, int K, int N, int mode, const RlRope& rp, cudaStream_t st) {
  const size_t smem = rows_linear_smem(K);
  const unsigned grid = (unsigned)(N / (mode >= 2 ? kRlCols / 2 : kRlCols));
#define PF_RL(T, U)                                                                                              \
  do {                                                                                                           \
    cudaError_t e = ensure_smem(rows_linear_kernel<T, U>, (int)rows_linear_smem(kRlWarps * (U) * 32));         \
    if (e != cudaSuccess) return e;                                                                              \
    cudaLaunchConfig_t cfg = {};                                                                                 \
    cfg.gridDim = dim3(grid);                                                                                    \
    cfg.blockDim = dim3(kRlThreads);                                                                             \
    cfg.dynamicSmemBytes = smem;                                                                                 \
    cfg.stream = st;                                                                                             \
    cudaLaunchAttribute attr[1];                                                                                 \
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;                                             \
    attr[0].val.programmaticStreamSerializationAllowed = 1;                                                      \
    cfg.attrs = attr;                                                                                            \
    cfg.numAttrs = 1;                                                                                            \
    e = cudaLaunchKernelEx(&cfg, rows_linear_kernel<T, U>, static_cast<const T*>(x),                             \
                           static_cast<const T*>(norm_w), eps, static_cast<const T*>(wt),                        \
                           static_cast<const T*>(res), static_cast<T*>(y), M, K, N, mode, rp);                   \
    if (e != cudaSuccess) return e;                                                                              \
  } while (0)
#define PF_RL_U(T)                              \
  do {                                          \
    if (K <= kRlWarps * 2 * 32) PF_RL(T, 2);    \
    else if (K <= kRlWarps * 4 * 32) PF_RL(T, 4); \
    else if (K <= kRlWarps * 6 * 32) PF_RL(T, 6); \
    else PF_RL(T, 8);                           \
  } while (0)
  if (dtype == PF_BF16) PF_RL_U(__nv_bfloat16);
  else PF_RL_U(__half);
#undef PF_RL_U
#undef PF_RL
  return cudaGetLastError();
}

cudaError_t launch_rows_linear(const void* x, const void* norm_w, float eps, const void* wt, const void* res, void* y,
                               int dtype, int M, int K, int N, int mode, cudaStream_t st) {
  return launch_rl(x, norm_w, eps, wt, res, y, dtype, M, K, N, mode, RlRope{}, st);
}

cudaError_t launch_rows_linear_rope_write(const void* x, const void* norm_w, float eps, const void* wt, void* q_out,
                                          void* k_pages, void* v_pages, const void* cos_t, const void* sin_t,
                                          int tdtype, int table_rows, const int32_t* tables,
                                          const int32_t* positions, const int32_t* rope_pos, int dtype, int M, int K,
                                          int H, int Hkv, int num_pages, int page_size, int pages_per_seq, int D,
                                          cudaStream_t st) {
  RlRope rp{q_out, k_pages, v_pages, cos_t, sin_t, tables, positions, rope_pos,
            tdtype, table_rows, H, Hkv, num_pages, page_size, pages_per_seq, D};
  const int pairs = (H + 2 * Hkv) * D / 2;
  return launch_rl(x, norm_w, eps, wt, nullptr, nullptr, dtype, M, K, pairs, 3, rp, st);
}

}  // namespace pf
