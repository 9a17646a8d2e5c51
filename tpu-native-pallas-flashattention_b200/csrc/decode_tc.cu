// decode_tc.cu -- decode attention (fixed or paged cache) for bf16/f16 with
// head_dim 64 or 128: TMA-swizzled K/V tiles + warp-level tensor-core MMA.
//
// Decode moves ~4 B of K/V per FLOP pair, so it is bound by HBM, not math;
// what limits a CUDA-core version is instruction issue (each key row is
// dotted with every query head of its group).  Here each warp turns a 32-key
// tile into two small GEMMs on the tensor cores --
//     S[16 x 32]  = Q[16 x D] K^T          (query heads of the kv group, padded to 16)
//     O[16 x D]  += P[16 x 32] V[32 x D]
// -- with m16n8k16 MMAs fed by ldmatrix from 128-byte-swizzled shared memory,
// so a tile costs ~100 instructions per warp and the SM keeps the TMA engine
// saturated.  (A decode step has 1..16 query rows per kv head: far below the
// 128-row tcgen05 tile, so the synchronous warp MMA is the right unit here.)
//
// K/V tiles arrive by TMA (cp.async.bulk.tensor, 128-byte swizzle): a fixed
// cache through a 3-D map [B*Hkv, cache_len, D] whose row extent is the valid
// length (rows past it are zero-filled), a paged pool through a 2-D map
// [num_pages*Hkv*page_size, D] with one box per page segment, addressed by
// block_tables[b, pos / page_size] (paged.py:158-159).  Page segments wholly
// past the context are never requested; rows past the context inside a
// loaded box are zeroed in shared memory before use, so NaN there cannot
// reach P.V.  Split-KV partials and the combine are shared with decode.cu.
#include <type_traits>
#include "common.cuh"
#include "kernels.h"
#include "sm100_util.cuh"

namespace pf {
namespace {

constexpr int kWarps = 4;
constexpr int kStages = 3;
constexpr int kTileKeys = 32;
// Page ids of one split staged in shared memory: a split spans at most 4096
// positions (the split planner's cap) and pages hold >= 8 rows, so 513 ids
// (+1 for a split that starts inside a page); larger spans read the table
// from global memory instead.
constexpr int kTblCap = 4096 / 8 + 8;

template <int D>
struct TcCfg {
  static constexpr int kBoxes = D / 64;
  static constexpr int kBoxBytes = kTileKeys * 128;          // 32 rows x 128 B
  static constexpr int kOperand = kBoxes * kBoxBytes;        // K (or V) of one tile
  static constexpr int kStageBytes = 2 * kOperand;
  static constexpr int kRing = kWarps * kStages * kStageBytes;
  static constexpr int kRed = kWarps * 16 * (D + 2) * 4;     // per-warp (acc, m, l), reuses the ring
  static constexpr int kBarOff = kRing > kRed ? kRing : kRed;
  static constexpr int kTblOff = kBarOff + 128;                // after the kWarps * kStages barriers
  static constexpr int kSmem = kTblOff + kTblCap * 4 + 1024;
  static_assert(kWarps * kStages * 8 <= 128, "barriers overlap the page-id table");
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

template <int FMT>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (FMT == 1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Byte offset of row `row`, 64-column box `box` in a tile whose rows arrive in
// segments of SEG rows, each segment laid out [box][row][128 B].  SEG = 32 (a
// whole tile) is the plain [box][32 rows] layout; a paged tile whose pages
// are 16 (or 8) rows long and whose two D = 128 halves come in one copy per
// page segment has SEG = 16 (8).  SEG is a multiple of 8, so every segment
// starts on a 1024-byte swizzle atom and (row & 7) is the swizzle phase.
template <int D, int SEG>
__device__ __forceinline__ uint32_t row_off(int row, int box) {
  return (row / SEG) * (D / 64 * SEG * 128) + box * (SEG * 128) + (row % SEG) * 128;
}
// Byte address of (row, column d) in such a tile (128-byte swizzle).
template <int D, int SEG>
__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int d) {
  const int box = d >> 6, chunk = (d & 63) >> 3;
  return base + row_off<D, SEG>(row, box) + ((chunk ^ (row & 7)) << 4);
}

// grid = (num_splits, Hkv * head_chunks, B); block = kWarps * 32.
// SEG: the tile's shared-memory segment length (see row_off); paired = the
// paged maps bring both D = 128 halves of a page segment in one copy (SEG is
// then the segment length), else one copy per 64-column half.
template <typename T, int D, int SEG>
__global__ void __launch_bounds__(kWarps * 32)
decode_tc_kernel(DecodeArgs a, const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                 int head_chunks, int seg_rows, bool paired) {
  using Cfg = TcCfg<D>;
  constexpr int FMT = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr int NB = D / 8;  // output n-blocks
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  int* tbl = reinterpret_cast<int*>(smem + Cfg::kTblOff);

  const int split = blockIdx.x;
  const int hk = blockIdx.y / head_chunks;
  const int hchunk = blockIdx.y % head_chunks;
  const int b = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int G = a.H / a.Hkv;
  const int h0 = hk * G + hchunk * 16;
  const int gcount = min(16, hk * G + G - h0);
  const bool paged = a.block_tables != nullptr;

  // Launched as a programmatic dependent of the previous kernel on the stream
  // (a decode step's RoPE + cache write): wait for it before reading lengths,
  // tables, q or the cache, then let the next kernel launch (the output
  // projection prefetches its weights while this one runs).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  int len = a.context_lens ? a.context_lens[b] : a.fixed_len;
  if (paged && len > a.pages_per_seq * a.page_size) {
    if (threadIdx.x == 0) flag_status(PF_DEV_BAD_PAGE);
    len = a.pages_per_seq * a.page_size;
  }
  // A length beyond the call's promised maximum would lose the keys past the
  // planned splits: record it (once per sequence and head group) instead of
  // silently attending a prefix.
  if (len > a.max_len && split == 0 && threadIdx.x == 0) flag_status(PF_DEV_LEN_OVER_MAX);
  const int k_begin = split * a.split_len;
  const int k_end = min(len, k_begin + a.split_len);
  if (k_begin >= k_end) {  // uniform over the CTA
    if (a.num_splits == 1)  // no combine follows: an empty sequence's output is 0
      for (int e = threadIdx.x; e < gcount * D; e += blockDim.x)
        static_cast<T*>(a.o)[((long)b * a.H + h0 + e / D) * D + e % D] = from_f<T>(0.f);
    return;
  }

  // Paged: every page id of the split is read (and validated) once, by all
  // threads in parallel, so the TMA issue below never waits on a global load.
  const int p_first = paged ? k_begin / a.page_size : 0;
  const bool tbl_smem = paged && (k_end - 1) / a.page_size - p_first + 1 <= kTblCap;
  if (tbl_smem) {
    const int n_ids = (k_end - 1) / a.page_size - p_first + 1;
    const int* row_ids = a.block_tables + (long)b * a.pages_per_seq + p_first;
    for (int i = threadIdx.x; i < n_ids; i += blockDim.x) {
      int page = row_ids[i];
      if (page < 0 || page >= a.num_pages) {
        flag_status(PF_DEV_BAD_PAGE);
        page = 0;
      }
      tbl[i] = page;
    }
    __syncthreads();
  }

  uint64_t* wbar = bars + warp * kStages;
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
  }
  __syncwarp();

  // Q fragments (A operand, rows = query heads of this chunk, zero-padded).
  const T* qb = static_cast<const T*>(a.q) + ((long)b * a.H + h0) * D;
  uint32_t qa[D / 16][4];
  {
    const int r0 = lane / 4, r1 = r0 + 8, c = (lane % 4) * 2;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int d0 = ks * 16 + c;
      auto ld2 = [&](int r, int d) -> uint32_t {
        return r < gcount ? *reinterpret_cast<const uint32_t*>(qb + (long)r * D + d) : 0u;
      };
      qa[ks][0] = ld2(r0, d0);
      qa[ks][1] = ld2(r1, d0);
      qa[ks][2] = ld2(r0, d0 + 8);
      qa[ks][3] = ld2(r1, d0 + 8);
    }
  }

  uint8_t* wring = smem + (size_t)warp * kStages * Cfg::kStageBytes;
  const int n_tiles = (k_end - k_begin + kWarps * kTileKeys - 1) / (kWarps * kTileKeys);
  auto tile_key = [&](int t) { return k_begin + (t * kWarps + warp) * kTileKeys; };
  auto tile_valid = [&](int t) { return max(0, min(kTileKeys, k_end - tile_key(t))); };
  const long plane = (long)b * a.Hkv + hk;

  auto issue = [&](int t) {  // lane 0 only
    const int kt = tile_key(t), nv = tile_valid(t);
    if (nv <= 0) return;
    uint64_t* bar = &wbar[t % kStages];
    uint8_t* kdst = wring + (size_t)(t % kStages) * Cfg::kStageBytes;
    uint8_t* vdst = kdst + Cfg::kOperand;
    if (!paged) {
      mbar_expect_tx(bar, 2 * Cfg::kOperand);
#pragma unroll
      for (int c = 0; c < Cfg::kBoxes; ++c) {
        tma_load_3d(kdst + c * Cfg::kBoxBytes, &tm_k, bar, c * 64, kt, (int)plane);
        tma_load_3d(vdst + c * Cfg::kBoxBytes, &tm_v, bar, c * 64, kt, (int)plane);
      }
      return;
    }
    const int nseg = (nv + seg_rows - 1) / seg_rows;
    mbar_expect_tx(bar, (uint32_t)(2 * nseg * seg_rows * 128 * Cfg::kBoxes));
    for (int sg = 0; sg < nseg; ++sg) {
      const int pos = kt + sg * seg_rows;
      int page;
      if (tbl_smem) {
        page = tbl[pos / a.page_size - p_first];
      } else {
        page = a.block_tables[(long)b * a.pages_per_seq + pos / a.page_size];
        if (page < 0 || page >= a.num_pages) {
          flag_status(PF_DEV_BAD_PAGE);
          page = 0;
        }
      }
      const int row = (int)(((long)page * a.Hkv + hk) * a.page_size + pos % a.page_size);
      if (paired) {  // both halves of the segment in one copy each for K and V
        const uint32_t off = row_off<D, SEG>(sg * seg_rows, 0);
        tma_load_3d(kdst + off, &tm_k, bar, 0, row, 0);
        tma_load_3d(vdst + off, &tm_v, bar, 0, row, 0);
        continue;
      }
#pragma unroll
      for (int c = 0; c < Cfg::kBoxes; ++c) {
        const uint32_t off = row_off<D, SEG>(sg * seg_rows, c);
        tma_load_3d(kdst + off, &tm_k, bar, c * 64, row, 0);
        tma_load_3d(vdst + off, &tm_v, bar, c * 64, row, 0);
      }
    }
  };

  if (lane == 0)
    for (int t = 0; t < kStages && t < n_tiles; ++t) issue(t);
  __syncwarp();

  float o[NB][4];
#pragma unroll
  for (int i = 0; i < NB; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = a.sm_scale * kLog2e;

  int t_stop = 0;  // first tile not consumed
  for (int t = 0; t < n_tiles; ++t, t_stop = t) {
    const int nv = tile_valid(t);
    if (nv <= 0) break;
    if (!mbar_wait(&wbar[t % kStages], (t / kStages) & 1)) break;
    uint8_t* kbuf = wring + (size_t)(t % kStages) * Cfg::kStageBytes;
    uint8_t* vbuf = kbuf + Cfg::kOperand;
    if (nv < kTileKeys) {
      // Rows past the valid length: zero K and V (never-loaded or past-context bytes).
      const int rows = kTileKeys - nv;
      for (int i = lane; i < rows * 8 * Cfg::kBoxes; i += 32) {
        const int r = nv + i / (8 * Cfg::kBoxes), rest = i % (8 * Cfg::kBoxes);
        const int box = rest / 8, ch = rest % 8;
        uint4* pk = reinterpret_cast<uint4*>(kbuf + row_off<D, SEG>(r, box) + ch * 16);
        uint4* pv = reinterpret_cast<uint4*>(vbuf + row_off<D, SEG>(r, box) + ch * 16);
        *pk = make_uint4(0, 0, 0, 0);
        *pv = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();  // these generic writes precede the next TMA into the stage
      __syncwarp();
    }
    const uint32_t kb = smem_u32(kbuf), vb = smem_u32(vbuf);

    // S = Q K^T : 4 key blocks of 8.
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    const int mi = lane / 8, mr = lane % 8;
#pragma unroll
    for (int nb2 = 0; nb2 < 2; ++nb2) {
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t b0, b1, b2, b3;
        const int key = nb2 * 16 + (mi >> 1) * 8 + mr;
        const int d = ks * 16 + (mi & 1) * 8;
        ldsm_x4(swz<D, SEG>(kb, key, d), b0, b1, b2, b3);
        mma16816<FMT>(s[2 * nb2], qa[ks], b0, b1);
        mma16816<FMT>(s[2 * nb2 + 1], qa[ks], b2, b3);
      }
    }
    // Online softmax over the tile (rows r0 = lane/4 -> regs 0,1; r1 = r0+8 -> regs 2,3).
    float mt0 = -INFINITY, mt1 = -INFINITY;
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int key = nb * 8 + (lane % 4) * 2 + u;
        const bool ok = key < nv;
        s[nb][u] = ok ? s[nb][u] * sl2 : -INFINITY;
        s[nb][2 + u] = ok ? s[nb][2 + u] * sl2 : -INFINITY;
        mt0 = fmaxf(mt0, s[nb][u]);
        mt1 = fmaxf(mt1, s[nb][2 + u]);
      }
    }
    mt0 = fmaxf(mt0, __shfl_xor_sync(0xffffffffu, mt0, 1));
    mt0 = fmaxf(mt0, __shfl_xor_sync(0xffffffffu, mt0, 2));
    mt1 = fmaxf(mt1, __shfl_xor_sync(0xffffffffu, mt1, 1));
    mt1 = fmaxf(mt1, __shfl_xor_sync(0xffffffffu, mt1, 2));
    const float mn0 = fmaxf(m0, mt0), mn1 = fmaxf(m1, mt1);  // finite: nv >= 1
    const float al0 = fast_exp2(m0 - mn0), al1 = fast_exp2(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    l0 *= al0;
    l1 *= al1;
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      o[i][0] *= al0;
      o[i][1] *= al0;
      o[i][2] *= al1;
      o[i][3] *= al1;
    }
    uint32_t pa[2][4];
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
      const float p0 = fast_exp2(s[nb][0] - mn0), p1 = fast_exp2(s[nb][1] - mn0);
      const float p2 = fast_exp2(s[nb][2] - mn1), p3 = fast_exp2(s[nb][3] - mn1);
      l0 += p0 + p1;
      l1 += p2 + p3;
      const uint32_t lo = FMT == 1 ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
      const uint32_t hi = FMT == 1 ? pack_bf16x2(p2, p3) : pack_f16x2(p2, p3);
      // A fragment of k-step nb/2: regs {row r0 k..k+1, row r1, row r0 k+8, row r1 k+8}
      pa[nb >> 1][(nb & 1) * 2 + 0] = lo;
      pa[nb >> 1][(nb & 1) * 2 + 1] = hi;
    }
    // O += P V : 2 k-steps of 16 keys, D/16 pairs of output blocks.
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
      for (int nd2 = 0; nd2 < D / 16; ++nd2) {
        uint32_t b0, b1, b2, b3;
        const int key = ks * 16 + (mi & 1) * 8 + mr;
        const int d = nd2 * 16 + (mi >> 1) * 8;
        ldsm_x4_t(swz<D, SEG>(vb, key, d), b0, b1, b2, b3);
        mma16816<FMT>(o[2 * nd2], pa[ks], b0, b1);
        mma16816<FMT>(o[2 * nd2 + 1], pa[ks], b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0 && t + kStages < n_tiles) issue(t + kStages);
    __syncwarp();
  }
  // Exit drain (only a timed-out wait leaves copies in flight): tiles
  // [0, t_stop + kStages) were issued, those before t_stop consumed.
  if (lane == 0)
    for (int u = t_stop; u < t_stop + kStages && u < n_tiles; ++u)
      if (tile_valid(u) > 0) mbar_wait(&wbar[u % kStages], (u / kStages) & 1);
  __syncwarp();
  // Row sums across the quad.
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  __syncthreads();  // every warp is done with its ring: reuse it for the merge
  float* red = reinterpret_cast<float*>(smem);  // [kWarps][16][D + 2]
  {
    float* my = red + warp * 16 * (D + 2);
    const int r0 = lane / 4, r1 = r0 + 8, c = (lane % 4) * 2;
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      my[r0 * (D + 2) + nb * 8 + c] = o[nb][0];
      my[r0 * (D + 2) + nb * 8 + c + 1] = o[nb][1];
      my[r1 * (D + 2) + nb * 8 + c] = o[nb][2];
      my[r1 * (D + 2) + nb * 8 + c + 1] = o[nb][3];
    }
    if ((lane % 4) == 0) {
      my[r0 * (D + 2) + D] = m0;
      my[r0 * (D + 2) + D + 1] = l0;
      my[r1 * (D + 2) + D] = m1;
      my[r1 * (D + 2) + D + 1] = l1;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < gcount * D; e += blockDim.x) {
    const int g = e / D, d = e % D;
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, red[(w * 16 + g) * (D + 2) + D]);
    float L = 0.f, A = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float* r = red + (w * 16 + g) * (D + 2);
      if (r[D] == -INFINITY) continue;
      const float sc = fast_exp2(r[D] - M);
      L += r[D + 1] * sc;
      A += r[d] * sc;
    }
    if (a.num_splits == 1) {  // the whole sequence: normalise and write the output
      static_cast<T*>(a.o)[((long)b * a.H + h0 + g) * D + d] = from_f<T>(L == 0.f ? 0.f : A / L);
      continue;
    }
    float* out = a.partial + (((long)b * a.H + h0 + g) * a.num_splits + split) * (D + 2);
    out[d] = A;
    if (d == 0) {
      out[D] = M;
      out[D + 1] = L;
    }
  }
}

template <typename T, int D, int SEG>
cudaError_t launch_tc_kernel(const DecodeArgs& a, const CUtensorMap& tk, const CUtensorMap& tv, int seg_rows,
                             bool paired) {
  using Cfg = TcCfg<D>;
  const int G = a.H / a.Hkv;
  const int head_chunks = (G + 15) / 16;
  auto kern = decode_tc_kernel<T, D, SEG>;
  cudaError_t e = ensure_smem(kern, Cfg::kSmem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.num_splits, a.Hkv * head_chunks, a.B);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a, tk, tv, head_chunks, seg_rows, paired);
}

template <typename T, int D>
cudaError_t launch_tc_t(const DecodeArgs& a) {
  CUtensorMap tk, tv;
  int seg_rows = kTileKeys;
  bool paired = false;
  if (a.block_tables == nullptr) {
    if (!make_tile_map(&tk, a.k_src, a.dtype, D, a.fixed_len, a.cache_rows, a.B * a.Hkv, kTileKeys) ||
        !make_tile_map(&tv, a.v_src, a.dtype, D, a.fixed_len, a.cache_rows, a.B * a.Hkv, kTileKeys))
      return cudaErrorInvalidValue;
  } else {
    seg_rows = a.page_size < kTileKeys ? a.page_size : kTileKeys;
    const long rows = (long)a.num_pages * a.Hkv * a.page_size;
    // D = 128: one copy per page segment for both column halves (half the
    // copies of two 64-column boxes; the copy count bounds small-page decode).
    paired = D == 128 && make_paged_pair_map(&tk, a.k_src, a.dtype, rows, seg_rows) &&
             make_paged_pair_map(&tv, a.v_src, a.dtype, rows, seg_rows);
    if (!paired && (!make_tile_map(&tk, a.k_src, a.dtype, D, (int)rows, rows, 1, seg_rows) ||
                    !make_tile_map(&tv, a.v_src, a.dtype, D, (int)rows, rows, 1, seg_rows)))
      return cudaErrorInvalidValue;
  }
  cudaError_t e;
  if (paired && seg_rows == 8) e = launch_tc_kernel<T, D, 8>(a, tk, tv, seg_rows, true);
  else if (paired && seg_rows == 16) e = launch_tc_kernel<T, D, 16>(a, tk, tv, seg_rows, true);
  else e = launch_tc_kernel<T, D, kTileKeys>(a, tk, tv, seg_rows, paired);
  if (e != cudaSuccess) return e;
  return a.num_splits == 1 ? cudaSuccess : launch_decode_combine(a);
}

}  // namespace

bool decode_tc_supported(int dtype, int D, int page_size, bool paged, long rows) {
  if (!(dtype == PF_BF16 || dtype == PF_F16) || !(D == 64 || D == 128)) return false;
  if (!paged) return true;
  // Page segments must start on 1024-byte swizzle atoms: 8-row multiples
  // (or whole 32-row tiles), and the pool row count must fit a 32-bit TMA extent.
  const bool seg_ok = page_size % 32 == 0 || page_size == 8 || page_size == 16;
  return seg_ok && rows < (1l << 31);
}

cudaError_t launch_decode_tc(const DecodeArgs& a) {
  if (a.dtype == PF_BF16) return a.D == 128 ? launch_tc_t<__nv_bfloat16, 128>(a) : launch_tc_t<__nv_bfloat16, 64>(a);
  return a.D == 128 ? launch_tc_t<__half, 128>(a) : launch_tc_t<__half, 64>(a);
}

}  // namespace pf
