// attn_simt.cu -- fp32 SIMT attention kernels (forward with LSE, fused RoPE,
// backward preprocess / dQ / dK,dV).  These carry the fp32-input path (which
// must match the reference's fp32 math to 1e-4 relative, beyond what bf16 or
// TF32 tensor cores give) and every head_dim the tensor-core kernels do not
// instantiate.  All arithmetic is fp32; inputs are up-cast on load, exactly as
// the reference kernels up-cast their VMEM blocks.
//
// Semantics follow src/pallas_flash/flash_attention.py of the reference:
//   mask = (k_pos < kv_len) [&& q_pos >= k_pos]            (:114-120, :266-268)
//   online softmax m/l/acc recurrence                      (:122-134)
//   block skipping on kv_len and the causal diagonal       (:136-147)
//   finalize: l == 0 -> o = 0, lse = 0                      (:150-159)
//   backward p = exp(s - lse), ds = p (dp - delta)          (:245-273)
//   dK/dV summed over the q heads of each kv head          (:433-436)
#include "common.cuh"
#include "kernels.h"

namespace pf {

__device__ int g_status = 0;
__device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;
#ifdef PF_TRACE
__device__ unsigned long long g_trace[kTraceCtas * kTraceEvents];
__device__ unsigned int g_trace_n[kTraceCtas];
#endif

namespace {

constexpr int kBQ = 16;       // query rows per CTA (4 warps x 4 rows)
constexpr int kBK = 32;       // keys per smem tile (one per lane)
constexpr int kThreads = 128;
constexpr int kRowsPerWarp = kBQ / (kThreads / 32);
// Key groups per forward CTA (shared memory: one K and one V tile per group).
template <int DMAX>
constexpr int fwd_groups() { return DMAX == 256 ? 2 : 4; }

// Loads rows [row0, row0 + nrows) of a [rows_total, D] matrix into smem
// (stride ld floats), zero-filling rows past `valid` and columns past D.
// When cos/sin tables are given, applies x*cos + rotate_half(x)*sin using
// table rows (row0 + r) -- the fused-RoPE prologue of fused_rope.py:75-78.
template <typename T>
__device__ void load_tile(float* dst, int ld, const T* src, int row0, int nrows, int valid,
                          int D, int DMAX, const void* cos_t, const void* sin_t, int tbl_dtype) {
  const int half = D / 2;
  for (int idx = threadIdx.x; idx < nrows * DMAX; idx += blockDim.x) {
    const int r = idx / DMAX, c = idx % DMAX;
    const int row = row0 + r;
    float x = 0.f;
    if (row < valid && c < D) {
      x = to_f(src[(long)row * D + c]);
      if (cos_t != nullptr) {
        const float partner = (c < half) ? -to_f(src[(long)row * D + c + half])
                                         : to_f(src[(long)row * D + c - half]);
        x = x * load_any(cos_t, tbl_dtype, (long)row * D + c) +
            partner * load_any(sin_t, tbl_dtype, (long)row * D + c);
      }
    }
    dst[r * ld + c] = x;
  }
}

// Like load_tile, by the 128 threads of one key group (`tid` in [0, 128)).
template <typename T>
__device__ void load_tile_group(float* dst, int ld, const T* src, int row0, int nrows, int valid, int D, int DMAX,
                                const void* cos_t, const void* sin_t, int tbl_dtype, int tid) {
  const int half = D / 2;
  for (int idx = tid; idx < nrows * DMAX; idx += 128) {
    const int r = idx / DMAX, c = idx % DMAX;
    const int row = row0 + r;
    float x = 0.f;
    if (row < valid && c < D) {
      x = to_f(src[(long)row * D + c]);
      if (cos_t != nullptr) {
        const float partner = (c < half) ? -to_f(src[(long)row * D + c + half])
                                         : to_f(src[(long)row * D + c - half]);
        x = x * load_any(cos_t, tbl_dtype, (long)row * D + c) +
            partner * load_any(sin_t, tbl_dtype, (long)row * D + c);
      }
    }
    dst[r * ld + c] = x;
  }
}

__device__ __forceinline__ void group_sync(int group) {  // the 128 threads of key group `group`
  asm volatile("bar.sync %0, 128;" ::"r"(group + 1) : "memory");
}

// Forward.  grid = (ceil(Sq / kBQ), H, B); kFwdGroups key groups of 4 warps
// per CTA split the key loop of the CTA's 16 query rows (every group takes
// every kFwdGroups-th key tile) and merge their (max, sum, accumulator) at
// the end, so the heaviest causal tile's serial chain is kFwdGroups times
// shorter.  Each group's warps run the same loop (its barrier is the
// group's own, the usual __syncthreads pattern within the group).
template <typename T, int DMAX, int kFwdGroups = fwd_groups<DMAX>()>
__global__ void __launch_bounds__(kThreads * kFwdGroups)
fwd_simt_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                T* __restrict__ o, float* __restrict__ lse, int H, int Hkv, int Sq, int Sk,
                int D, int causal, float sm_scale, int kv_len_max, const void* q_cos,
                const void* q_sin, const void* k_cos, const void* k_sin, int tbl_dtype,
                const int32_t* __restrict__ kv_lens, const int32_t* __restrict__ q_offs) {
  constexpr int LD = DMAX + 1;
  constexpr int NPL = DMAX / 32;  // output dims per lane
  extern __shared__ float smem[];
  const int kg = threadIdx.x / kThreads;     // key group
  const int gtid = threadIdx.x % kThreads;   // thread within the group
  float* sQ = smem;                                          // [kBQ][LD]
  float* sK = sQ + kBQ * LD + kg * 2 * kBK * LD;             // [kBK][LD] of this group
  float* sV = sK + kBK * LD;                                 // [kBK][LD]

  // Heaviest (last, under causal) query tiles first: they set the tail.
  const int qb = gridDim.x - 1 - blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (H / Hkv);
  const int warp = (threadIdx.x / 32) % (kThreads / 32), lane = threadIdx.x % 32;
  const int q0 = qb * kBQ;
  // Keys of this sequence and the position of query row 0 (causal offset).
  const int kv_len = kv_lens ? max(0, min(kv_lens[b], kv_len_max)) : kv_len_max;
  const int q_off = q_offs ? q_offs[b] : 0;
  const T* qp = q + ((long)b * H + h) * Sq * D;
  const T* kp = k + ((long)b * Hkv + hk) * Sk * D;
  const T* vp = v + ((long)b * Hkv + hk) * Sk * D;

  load_tile<T>(sQ, LD, qp, q0, kBQ, Sq, D, DMAX, q_cos, q_sin, tbl_dtype);
  __syncthreads();

  float m[kRowsPerWarp], l[kRowsPerWarp], acc[kRowsPerWarp][NPL];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i) acc[r][i] = 0.f;
  }

  // Last key any row of this tile may see (block skipping, :136-147).
  int k_end = kv_len;
  if (causal) k_end = min(k_end, q0 + q_off + kBQ);
  for (int k0 = kg * kBK; k0 < k_end; k0 += kFwdGroups * kBK) {
    group_sync(kg);
    load_tile_group<T>(sK, LD, kp, k0, kBK, kv_len, D, DMAX, k_cos, k_sin, tbl_dtype, gtid);
    load_tile_group<T>(sV, LD, vp, k0, kBK, kv_len, D, DMAX, nullptr, nullptr, 0, gtid);
    group_sync(kg);
    const int kpos = k0 + lane;
    // Scores of this lane's key for all of the warp's rows at once: the rows
    // are independent FMA chains (columns past D are zero in shared memory).
    float s[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) s[r] = 0.f;
    const float* qrow = sQ + warp * kRowsPerWarp * LD;
#pragma unroll 8
    for (int d = 0; d < DMAX; ++d) {
      const float kd = sK[lane * LD + d];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) s[r] = fmaf(qrow[r * LD + d], kd, s[r]);
    }
    float p[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const int qpos = q0 + warp * kRowsPerWarp + r;
      const bool ok = (kpos < kv_len) && (!causal || qpos + q_off >= kpos);
      const float sr = ok ? s[r] * sm_scale : -INFINITY;
      const float mn = fmaxf(m[r], warp_max(sr));
      if (mn == -INFINITY) {  // nothing visible yet for this row (warp-uniform)
        p[r] = 0.f;
        continue;
      }
      p[r] = ok ? expf(sr - mn) : 0.f;
      const float alpha = expf(m[r] - mn);  // exp(-inf) = 0 on the first live block
      l[r] = l[r] * alpha + warp_sum(p[r]);
      m[r] = mn;
#pragma unroll
      for (int i = 0; i < NPL; ++i) acc[r][i] *= alpha;
    }
    // O += P V: each V element is loaded once for all rows.
#pragma unroll 4
    for (int j = 0; j < kBK; ++j) {
      float vj[NPL];
#pragma unroll
      for (int i = 0; i < NPL; ++i) vj[i] = sV[j * LD + lane + 32 * i];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const float pj = __shfl_sync(0xffffffffu, p[r], j);
#pragma unroll
        for (int i = 0; i < NPL; ++i) acc[r][i] = fmaf(pj, vj[i], acc[r][i]);
      }
    }
  }

  // Merge the key groups: group g's (m, l, acc) of row i go to shared memory
  // (over the K/V tiles), then group 0 rescales to the common maximum.
  __syncthreads();
  float* mrg = smem + kBQ * LD;  // [kFwdGroups][kBQ][DMAX + 2]
  constexpr int MS = DMAX + 2;
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    float* slot = mrg + ((long)kg * kBQ + warp * kRowsPerWarp + r) * MS;
#pragma unroll
    for (int i = 0; i < NPL; ++i) slot[lane + 32 * i] = acc[r][i];
    if (lane == 0) {
      slot[DMAX] = m[r];
      slot[DMAX + 1] = l[r];
    }
  }
  __syncthreads();
  if (kg != 0) return;
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int row = warp * kRowsPerWarp + r;
    float mx = -INFINITY;
#pragma unroll
    for (int g = 0; g < kFwdGroups; ++g) mx = fmaxf(mx, mrg[((long)g * kBQ + row) * MS + DMAX]);
    float lsum = 0.f, a[NPL];
#pragma unroll
    for (int i = 0; i < NPL; ++i) a[i] = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int g = 0; g < kFwdGroups; ++g) {
        const float* slot = mrg + ((long)g * kBQ + row) * MS;
        const float gm = slot[DMAX];
        const float w = gm == -INFINITY ? 0.f : expf(gm - mx);
        lsum += slot[DMAX + 1] * w;
#pragma unroll
        for (int i = 0; i < NPL; ++i) a[i] = fmaf(slot[lane + 32 * i], w, a[i]);
      }
    }
    m[r] = mx;
    l[r] = lsum;
#pragma unroll
    for (int i = 0; i < NPL; ++i) acc[r][i] = a[i];
  }

#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int qpos = q0 + warp * kRowsPerWarp + r;
    if (qpos >= Sq) continue;
    const bool empty = (l[r] == 0.f);
    const float inv = empty ? 0.f : 1.f / l[r];
    T* op = o + (((long)b * H + h) * Sq + qpos) * D;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int d = lane + 32 * i;
      if (d < D) op[d] = from_f<T>(acc[r][i] * inv);
    }
    if (lse != nullptr && lane == 0)
      lse[((long)b * H + h) * Sq + qpos] = empty ? 0.f : m[r] + logf(l[r]);
  }
}

// delta[row] = sum_d o[row, d] * do[row, d]   (flash_attention.py:363-365)
template <typename T>
__global__ void bwd_preprocess_kernel(const T* __restrict__ o, const T* __restrict__ dout,
                                      float* __restrict__ delta, long rows, int D) {
  const long row = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  float s = 0.f;
  for (int d = lane; d < D; d += 32) s = fmaf(to_f(o[row * D + d]), to_f(dout[row * D + d]), s);
  s = warp_sum(s);
  if (lane == 0) delta[row] = s;
}

// Sum of the products of the 8 bf16/f16 (or 4 f32) elements packed in a and b.
template <typename T> __device__ __forceinline__ float dot16(uint4 a, uint4 b);
template <> __device__ __forceinline__ float dot16<float>(uint4 a, uint4 b) {
  return __uint_as_float(a.x) * __uint_as_float(b.x) + __uint_as_float(a.y) * __uint_as_float(b.y) +
         __uint_as_float(a.z) * __uint_as_float(b.z) + __uint_as_float(a.w) * __uint_as_float(b.w);
}
template <typename T2, typename F>
__device__ __forceinline__ float dot16_packed(uint4 a, uint4 b, F to2) {
  const unsigned av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = to2(*reinterpret_cast<const T2*>(&av[i])), y = to2(*reinterpret_cast<const T2*>(&bv[i]));
    s = fmaf(x.x, y.x, fmaf(x.y, y.y, s));
  }
  return s;
}
template <> __device__ __forceinline__ float dot16<__nv_bfloat16>(uint4 a, uint4 b) {
  return dot16_packed<__nv_bfloat162>(a, b, [](__nv_bfloat162 v) { return __bfloat1622float2(v); });
}
template <> __device__ __forceinline__ float dot16<__half>(uint4 a, uint4 b) {
  return dot16_packed<__half2>(a, b, [](__half2 v) { return __half22float2(v); });
}

// The same delta with 16-byte loads: L lanes share a row (L = row bytes / 16, a power
// of two <= 32), each lane keeps kRowsInFlight rows' loads in flight, and the grid
// strides over rows (HBM-bound: 2 * D * elt bytes read per row).
constexpr int kRowsInFlight = 4;
template <typename T, int L>
__global__ void __launch_bounds__(256)
bwd_preprocess_vec_kernel(const uint4* __restrict__ o, const uint4* __restrict__ dout,
                          float* __restrict__ delta, long rows) {
  constexpr int kRowsPerWarp = 32 / L;
  const int lane = threadIdx.x % 32, sub = lane % L;
  const long warp = ((long)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const long nwarps = (long)gridDim.x * blockDim.x / 32;
  // w0 is uniform across the warp, so every lane stays in the loop for the shuffles.
  for (long w0 = warp * kRowsPerWarp * kRowsInFlight; w0 < rows; w0 += nwarps * kRowsPerWarp * kRowsInFlight) {
    uint4 a[kRowsInFlight], b[kRowsInFlight];
#pragma unroll
    for (int u = 0; u < kRowsInFlight; ++u) {
      const long r = w0 + u * kRowsPerWarp + lane / L;
      if (r < rows) {
        a[u] = __ldg(o + r * L + sub);
        b[u] = __ldg(dout + r * L + sub);
      } else {
        a[u] = b[u] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < kRowsInFlight; ++u) {
      float s = dot16<T>(a[u], b[u]);
#pragma unroll
      for (int off = L / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      const long r = w0 + u * kRowsPerWarp + lane / L;
      if (sub == 0 && r < rows) delta[r] = s;
    }
  }
}

// dQ: grid = (ceil(Sq / kBQ), H, B).  Outer loop over query rows, inner over
// kv tiles, like _flash_attention_bwd_dq_kernel (:276-311).
template <typename T, int DMAX>
__global__ void __launch_bounds__(kThreads)
bwd_dq_simt_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                   const T* __restrict__ dout, const float* __restrict__ lse,
                   const float* __restrict__ delta, T* __restrict__ dq, int H, int Hkv, int Sq,
                   int Sk, int D, int causal, float sm_scale, int kv_len) {
  constexpr int LD = DMAX + 1;
  constexpr int NPL = DMAX / 32;
  extern __shared__ float smem[];
  float* sQ = smem;
  float* sDO = sQ + kBQ * LD;
  float* sK = sDO + kBQ * LD;
  float* sV = sK + kBK * LD;

  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (H / Hkv);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int q0 = qb * kBQ;
  const long qrow0 = ((long)b * H + h) * Sq;
  const T* kp = k + ((long)b * Hkv + hk) * Sk * D;
  const T* vp = v + ((long)b * Hkv + hk) * Sk * D;
  load_tile<T>(sQ, LD, q + qrow0 * D, q0, kBQ, Sq, D, DMAX, nullptr, nullptr, 0);
  load_tile<T>(sDO, LD, dout + qrow0 * D, q0, kBQ, Sq, D, DMAX, nullptr, nullptr, 0);

  float lse_r[kRowsPerWarp], dlt_r[kRowsPerWarp], acc[kRowsPerWarp][NPL];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int qpos = q0 + warp * kRowsPerWarp + r;
    lse_r[r] = qpos < Sq ? lse[qrow0 + qpos] : 0.f;
    dlt_r[r] = qpos < Sq ? delta[qrow0 + qpos] : 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i) acc[r][i] = 0.f;
  }
  int k_end = kv_len;
  if (causal) k_end = min(k_end, q0 + kBQ);
  for (int k0 = 0; k0 < k_end; k0 += kBK) {
    __syncthreads();
    load_tile<T>(sK, LD, kp, k0, kBK, kv_len, D, DMAX, nullptr, nullptr, 0);
    load_tile<T>(sV, LD, vp, k0, kBK, kv_len, D, DMAX, nullptr, nullptr, 0);
    __syncthreads();
    const int kpos = k0 + lane;
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const int qi = warp * kRowsPerWarp + r;
      const int qpos = q0 + qi;
      float s = 0.f, dp = 0.f;
      for (int d = 0; d < D; ++d) {
        s = fmaf(sQ[qi * LD + d], sK[lane * LD + d], s);
        dp = fmaf(sDO[qi * LD + d], sV[lane * LD + d], dp);
      }
      const bool ok = (kpos < kv_len) && (qpos < Sq) && (!causal || qpos >= kpos);
      const float p = ok ? expf(s * sm_scale - lse_r[r]) : 0.f;
      const float ds = p * (dp - dlt_r[r]);
      for (int j = 0; j < kBK; ++j) {
        const float dsj = __shfl_sync(0xffffffffu, ds, j);
        if (dsj != 0.f) {
#pragma unroll
          for (int i = 0; i < NPL; ++i) acc[r][i] = fmaf(dsj, sK[j * LD + lane + 32 * i], acc[r][i]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int qpos = q0 + warp * kRowsPerWarp + r;
    if (qpos >= Sq) continue;
    T* dp_out = dq + (qrow0 + qpos) * D;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int d = lane + 32 * i;
      if (d < D) dp_out[d] = from_f<T>(acc[r][i] * sm_scale);
    }
  }
}

// dK/dV: grid = (ceil(Sk / kBK), Hkv, B).  Outer loop over keys; the inner
// loop runs over every q head of the group and every query tile, so the GQA
// group-sum happens in registers (no per-q-head temporaries).
template <typename T, int DMAX>
__global__ void __launch_bounds__(kThreads)
bwd_dkv_simt_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                    const T* __restrict__ dout, const float* __restrict__ lse,
                    const float* __restrict__ delta, T* __restrict__ dk, T* __restrict__ dv,
                    int H, int Hkv, int Sq, int Sk, int D, int causal, float sm_scale,
                    int kv_len) {
  constexpr int LD = DMAX + 1;
  constexpr int NPT = DMAX / 4;  // accumulator dims per thread (key = lane)
  extern __shared__ float smem[];
  float* sK = smem;               // [kBK][LD]
  float* sV = sK + kBK * LD;
  float* sQ = sV + kBK * LD;      // [kBQ][LD]
  float* sDO = sQ + kBQ * LD;
  float* sP = sDO + kBQ * LD;     // [kBQ][kBK + 1]
  float* sDS = sP + kBQ * (kBK + 1);
  float* sL = sDS + kBQ * (kBK + 1);  // lse   [kBQ]
  float* sD = sL + kBQ;               // delta [kBQ]

  const int kb = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int group = H / Hkv;
  const int k0 = kb * kBK;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const T* kp = k + ((long)b * Hkv + hk) * Sk * D;
  const T* vp = v + ((long)b * Hkv + hk) * Sk * D;
  load_tile<T>(sK, LD, kp, k0, kBK, kv_len, D, DMAX, nullptr, nullptr, 0);
  load_tile<T>(sV, LD, vp, k0, kBK, kv_len, D, DMAX, nullptr, nullptr, 0);

  float adk[NPT], adv[NPT];
#pragma unroll
  for (int i = 0; i < NPT; ++i) adk[i] = adv[i] = 0.f;

  // First query row that can see key k0 under the causal mask.
  const int q_begin = causal ? (k0 / kBQ) * kBQ : 0;
  if (k0 < kv_len) {
    for (int hq = hk * group; hq < (hk + 1) * group; ++hq) {
      const long qrow0 = ((long)b * H + hq) * Sq;
      for (int q0 = q_begin; q0 < Sq; q0 += kBQ) {
        __syncthreads();
        load_tile<T>(sQ, LD, q + qrow0 * D, q0, kBQ, Sq, D, DMAX, nullptr, nullptr, 0);
        load_tile<T>(sDO, LD, dout + qrow0 * D, q0, kBQ, Sq, D, DMAX, nullptr, nullptr, 0);
        if (threadIdx.x < kBQ) {
          const int qpos = q0 + threadIdx.x;
          sL[threadIdx.x] = qpos < Sq ? lse[qrow0 + qpos] : 0.f;
          sD[threadIdx.x] = qpos < Sq ? delta[qrow0 + qpos] : 0.f;
        }
        __syncthreads();
        // P and dS for the kBQ x kBK tile: thread -> (query, key) pairs.
        for (int e = threadIdx.x; e < kBQ * kBK; e += blockDim.x) {
          const int qi = e / kBK, kj = e % kBK;
          const int qpos = q0 + qi, kpos = k0 + kj;
          float s = 0.f, dp = 0.f;
          for (int d = 0; d < D; ++d) {
            s = fmaf(sQ[qi * LD + d], sK[kj * LD + d], s);
            dp = fmaf(sDO[qi * LD + d], sV[kj * LD + d], dp);
          }
          const bool ok = (kpos < kv_len) && (qpos < Sq) && (!causal || qpos >= kpos);
          const float p = ok ? expf(s * sm_scale - sL[qi]) : 0.f;
          sP[qi * (kBK + 1) + kj] = p;
          sDS[qi * (kBK + 1) + kj] = p * (dp - sD[qi]);
        }
        __syncthreads();
        // dv[key][d] += sum_q p[q][key] do[q][d];  dk[key][d] += sum_q ds[q][key] q[q][d]
#pragma unroll 4
        for (int qi = 0; qi < kBQ; ++qi) {
          const float p = sP[qi * (kBK + 1) + lane];
          const float ds = sDS[qi * (kBK + 1) + lane];
#pragma unroll
          for (int i = 0; i < NPT; ++i) {
            const int d = warp + 4 * i;
            adv[i] = fmaf(p, sDO[qi * LD + d], adv[i]);
            adk[i] = fmaf(ds, sQ[qi * LD + d], adk[i]);
          }
        }
      }
    }
  }
  const int kpos = k0 + lane;
  if (kpos < Sk) {
    T* dkp = dk + (((long)b * Hkv + hk) * Sk + kpos) * D;
    T* dvp = dv + (((long)b * Hkv + hk) * Sk + kpos) * D;
#pragma unroll
    for (int i = 0; i < NPT; ++i) {
      const int d = warp + 4 * i;
      if (d < D) {
        dkp[d] = from_f<T>(adk[i] * sm_scale);
        dvp[d] = from_f<T>(adv[i]);
      }
    }
  }
}

template <typename T, int DMAX>
cudaError_t launch_fwd_t(const FwdArgs& a) {
  constexpr int LD = DMAX + 1;
  constexpr int kFwdGroups = fwd_groups<DMAX>();
  const size_t tiles = (size_t)(kBQ + kFwdGroups * 2 * kBK) * LD;
  const size_t merge = (size_t)kBQ * LD + (size_t)kFwdGroups * kBQ * (DMAX + 2);
  const size_t smem = (tiles > merge ? tiles : merge) * sizeof(float);
  auto kern = fwd_simt_kernel<T, DMAX>;
  cudaError_t e = ensure_smem(kern, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((a.Sq + kBQ - 1) / kBQ, a.H, a.B);
  kern<<<grid, kThreads * kFwdGroups, smem, a.stream>>>(
      (const T*)a.q, (const T*)a.k, (const T*)a.v, (T*)a.o, a.lse, a.H, a.Hkv, a.Sq, a.Sk, a.D,
      a.causal, a.sm_scale, a.kv_len, a.q_cos, a.q_sin, a.k_cos, a.k_sin, a.tbl_dtype, a.kv_lens, a.q_offs);
  return cudaGetLastError();
}

template <typename T, int DMAX>
cudaError_t launch_dq_t(const BwdArgs& a) {
  constexpr int LD = DMAX + 1;
  const size_t smem = (size_t)(2 * kBQ + 2 * kBK) * LD * sizeof(float);
  auto kern = bwd_dq_simt_kernel<T, DMAX>;
  cudaError_t e = ensure_smem(kern, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((a.Sq + kBQ - 1) / kBQ, a.H, a.B);
  kern<<<grid, kThreads, smem, a.stream>>>((const T*)a.q, (const T*)a.k, (const T*)a.v,
                                           (const T*)a.dout, a.lse, a.delta, (T*)a.dq, a.H,
                                           a.Hkv, a.Sq, a.Sk, a.D, a.causal, a.sm_scale, a.kv_len);
  return cudaGetLastError();
}

template <typename T, int DMAX>
cudaError_t launch_dkv_t(const BwdArgs& a) {
  constexpr int LD = DMAX + 1;
  const size_t smem = ((size_t)(2 * kBK + 2 * kBQ) * LD + 2 * kBQ * (kBK + 1) + 2 * kBQ) * sizeof(float);
  auto kern = bwd_dkv_simt_kernel<T, DMAX>;
  cudaError_t e = ensure_smem(kern, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((a.Sk + kBK - 1) / kBK, a.Hkv, a.B);
  kern<<<grid, kThreads, smem, a.stream>>>((const T*)a.q, (const T*)a.k, (const T*)a.v,
                                           (const T*)a.dout, a.lse, a.delta, (T*)a.dk, (T*)a.dv,
                                           a.H, a.Hkv, a.Sq, a.Sk, a.D, a.causal, a.sm_scale,
                                           a.kv_len);
  return cudaGetLastError();
}

}  // namespace

#define PF_DISPATCH_SIMT(LAUNCH, ARGS)                                                 \
  do {                                                                                 \
    const int dm = (ARGS).D <= 64 ? 64 : ((ARGS).D <= 128 ? 128 : 256);                \
    switch ((ARGS).dtype) {                                                            \
      case PF_F32:                                                                     \
        return dm == 64 ? LAUNCH<float, 64>(ARGS)                                      \
             : dm == 128 ? LAUNCH<float, 128>(ARGS) : LAUNCH<float, 256>(ARGS);        \
      case PF_BF16:                                                                    \
        return dm == 64 ? LAUNCH<__nv_bfloat16, 64>(ARGS)                              \
             : dm == 128 ? LAUNCH<__nv_bfloat16, 128>(ARGS)                            \
                         : LAUNCH<__nv_bfloat16, 256>(ARGS);                           \
      default:                                                                         \
        return dm == 64 ? LAUNCH<__half, 64>(ARGS)                                     \
             : dm == 128 ? LAUNCH<__half, 128>(ARGS) : LAUNCH<__half, 256>(ARGS);      \
    }                                                                                  \
  } while (0)

cudaError_t launch_fwd_simt(const FwdArgs& a) { PF_DISPATCH_SIMT(launch_fwd_t, a); }
cudaError_t launch_bwd_dq_simt(const BwdArgs& a) { PF_DISPATCH_SIMT(launch_dq_t, a); }
cudaError_t launch_bwd_dkv_simt(const BwdArgs& a) { PF_DISPATCH_SIMT(launch_dkv_t, a); }

cudaError_t launch_bwd_preprocess(const void* o, const void* dout, float* delta, int dtype,
                                  long rows, int D, cudaStream_t stream) {
  const int warps = 8;
  dim3 grid((unsigned)((rows + warps - 1) / warps));
  if (rows == 0) return cudaSuccess;
  const long row_bytes = (long)D * (dtype == PF_F32 ? 4 : 2);
  const int L = (int)(row_bytes / 16);
  const bool aligned = ((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(dout)) % 16) == 0;
  if (aligned && row_bytes % 16 == 0 && L >= 1 && L <= 32 && (L & (L - 1)) == 0) {
    const int sms = sm_count();
    const long per_block = 256 / 32 * (32 / L) * kRowsInFlight;
    const long want = (rows + per_block - 1) / per_block;
    const unsigned vgrid = (unsigned)(want < (long)sms * 8 ? want : (long)sms * 8);
    const uint4* o4 = static_cast<const uint4*>(o);
    const uint4* d4 = static_cast<const uint4*>(dout);
#define PF_PRE_VEC(T)                                                                                   \
  switch (L) {                                                                                          \
    case 1: bwd_preprocess_vec_kernel<T, 1><<<vgrid, 256, 0, stream>>>(o4, d4, delta, rows); break;     \
    case 2: bwd_preprocess_vec_kernel<T, 2><<<vgrid, 256, 0, stream>>>(o4, d4, delta, rows); break;     \
    case 4: bwd_preprocess_vec_kernel<T, 4><<<vgrid, 256, 0, stream>>>(o4, d4, delta, rows); break;     \
    case 8: bwd_preprocess_vec_kernel<T, 8><<<vgrid, 256, 0, stream>>>(o4, d4, delta, rows); break;     \
    case 16: bwd_preprocess_vec_kernel<T, 16><<<vgrid, 256, 0, stream>>>(o4, d4, delta, rows); break;   \
    default: bwd_preprocess_vec_kernel<T, 32><<<vgrid, 256, 0, stream>>>(o4, d4, delta, rows); break;   \
  }
    if (dtype == PF_F32) { PF_PRE_VEC(float) }
    else if (dtype == PF_BF16) { PF_PRE_VEC(__nv_bfloat16) }
    else { PF_PRE_VEC(__half) }
#undef PF_PRE_VEC
    return cudaGetLastError();
  }
  switch (dtype) {
    case PF_F32:
      bwd_preprocess_kernel<float><<<grid, warps * 32, 0, stream>>>((const float*)o, (const float*)dout, delta, rows, D);
      break;
    case PF_BF16:
      bwd_preprocess_kernel<__nv_bfloat16><<<grid, warps * 32, 0, stream>>>(
          (const __nv_bfloat16*)o, (const __nv_bfloat16*)dout, delta, rows, D);
      break;
    default:
      bwd_preprocess_kernel<__half><<<grid, warps * 32, 0, stream>>>((const __half*)o, (const __half*)dout, delta, rows, D);
  }
  return cudaGetLastError();
}

}  // namespace pf
