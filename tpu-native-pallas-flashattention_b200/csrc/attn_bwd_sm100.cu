// attn_bwd_sm100.cu -- tensor-core (tcgen05 / TMEM / TMA) backward for bf16
// and f16 inputs, head_dim 64 or 128.
//
// The reference's backward (flash_attention.py:276-351) runs two kernels with
// transposed loops, each recomputing P from the saved log-sum-exp:
//   p = exp(s*scale - lse),  ds = p (dp - delta).
// Here:
//   dK/dV kernel: CTA = (batch, kv head, 128-key tile).  Loops over every q
//     head of the GQA group and every 128-row query tile that can see the
//     keys, so the group-sum of flash_attention.py:433-436 happens in TMEM:
//        S^T  = K Q^T         dP^T = V dO^T            (M = 128 keys, N = 128)
//        dV  += P^T dO        dK  += dS^T Q             (A = P^T, dS^T from TMEM)
//     With the dS spill (pf_bwd with room in its workspace) it also writes
//     every 16-bit dS tile to global memory, straight from registers, in the
//     core-matrix layout the dQ GEMM's tensor core reads (one bulk copy per
//     tile, no shared-memory staging on either side).
//   dQ GEMM:      persistent; dQ of a 128-row query tile = scale * sum over its
//     key tiles of dS K, streaming the spilled tiles (HBM-bound), so each
//     (key tile, query tile) pair costs 5 tile GEMMs instead of 7.
//   dQ kernel (without the spill): CTA = (batch, head, 128-row query tile),
//     loops over 128-key tiles recomputing S and dP:
//        S    = Q K^T         dP   = dO V^T             (M = 128 rows, N = 128)
//        dQ  += dS K                                     (A = dS from TMEM)
//
// All MMAs are 128 x 128 tiles: at N = 128 a shared-memory operand pair
// streams at the rate the tensor core needs for full throughput, where N = 64
// tiles reach only ~2/3 of it.  TMEM (512 columns) holds S and dP (128 each)
// and the accumulators (dV, dK: 2 x D; dQ: D, with S double-buffered).  The
// elementwise warps work in two phases per tile -- P (exp, needs S) then dS
// (needs dP) -- and the MMA issue order interleaves the GEMMs so that each
// phase overlaps tensor work of a neighbouring tile.
#include <algorithm>
#include <climits>
#include <type_traits>
#include "common.cuh"
#include "kernels.h"
#include "sm100_util.cuh"

namespace pf {
namespace {


// Warp 0: TMA producer; warp 1: MMA issuer; warps 2 .. 2 + 4*EWG - 1: EWG
// elementwise warpgroups, each owning 128/EWG columns of a tile (a warp
// reads TMEM lane quadrant warp % 4, so every four consecutive warps cover
// the 128 lanes); warp kCertWarp: the data certifier, which adds one arrival
// to each phase of two elementwise barriers once the tiles the MMA issuer
// reads after that phase have landed, so the issuer polls only the
// elementwise barriers (each poll it waits on costs tensor-core time).
// More elementwise warps hide more of the dependent-latency chains of the P
// and dS steps; fewer leave more registers per thread and less issue
// pressure beside the MMA warp.  Measured best (interleaved A/B, min over
// rounds): 2 warpgroups for both kernels.
template <int EWG>
struct Ew {
  static constexpr int kEWG = EWG;
  static constexpr int kNCH = 4 / EWG;  // 32-column chunks per elementwise thread
  static constexpr int kEWThreads = 128 * EWG;
  static constexpr int kCertWarp = 2 + 4 * EWG;
  static constexpr int kThreads = 64 + kEWThreads + 32;
};
#ifndef PF_DKV_EWG
#define PF_DKV_EWG 2
#endif
#ifndef PF_DQ_EWG
#define PF_DQ_EWG 2
#endif
using EwDkv = Ew<PF_DKV_EWG>;
using EwDq = Ew<PF_DQ_EWG>;

struct BwdBars {
  uint64_t fixed;                  // the CTA's resident tiles
  uint64_t full[4], empty[4];      // streamed stages (dK/dV: Q + statistics; dQ: K)
  uint64_t vfull[4], vempty[4];    // streamed stages (dK/dV: dO; dQ: V)
  uint64_t s_full[2], dp_full;     // S / dP in TMEM
  uint64_t p_ready, ds_ready;      // P / dS written for the accumulating MMAs
  uint64_t pv_done;                // dK/dV: dV(it) has read the P^T tile
  uint64_t p_half, ds_half;        // dK/dV: the first 32-column chunk of P^T / dS written
  uint64_t s_free, dp_free;        // S (dK/dV) / dP (dQ) loaded into registers
  uint64_t stats_free[2];          // dK/dV: a column-statistics slot has been read
  uint64_t done;                   // accumulators final
  uint32_t tmem_base;
};
static_assert(sizeof(BwdBars) <= 256, "barrier block exceeds its shared-memory slot");

// dK/dV: K, V resident; NQ stages of Q and NO of dO (128-row tiles), and two
// slots of their column statistics.  Q is live from S(it) to dK(it), so a
// third stage lets Q(it+1) load while Q(it-1) and Q(it) are still read; dO
// (dP(it) to dV(it)) needs two.  A statistics slot is refilled once the
// elementwise warps have read it (stats_free), not when its Q stage frees.
template <int D>
struct DkvCfg {
  static constexpr int kNQ = D == 128 ? 3 : 4;
  static constexpr int kNO = D == 128 ? 2 : 4;
  static constexpr int kBoxes = D / 64;
  static constexpr int kTile = 128 * D * 2;
  static constexpr int kFixedOff = 0;
  static constexpr int kQOff = 2 * kTile;
  static constexpr int kOOff = kQOff + kNQ * kTile;
  static constexpr int kStatOff = kOOff + kNO * kTile;  // [2][2][128] f32: -lse*log2e, -delta
  static constexpr int kBarOff = kStatOff + 2 * 256 * 4;
  // No alignment slack: at D = 128 the tiles fill the 227 KB limit, so the
  // kernel requires (and checks) a 1024-byte aligned dynamic shared window.
  static constexpr int kSmem = kBarOff + 256;
  static_assert(kSmem <= 232448, "dK/dV shared memory exceeds the per-block limit");
  static constexpr uint32_t kS = 0, kDP = 128, kDV = 256, kDK = 256 + D;
};

// dQ: Q, dO resident; a ring of 3 K tiles (each lives from S(j) to dQ(j)) and 2 V tiles.
template <int D>
struct DqCfg {
  static constexpr int kNK = 3, kNV = 2;
  static constexpr int kBoxes = D / 64;
  static constexpr int kTile = 128 * D * 2;
  static constexpr int kFixedOff = 0;
  static constexpr int kKOff = 2 * kTile;
  static constexpr int kVOff = kKOff + kNK * kTile;
  static constexpr int kBarOff = kVOff + kNV * kTile;
  static constexpr int kSmem = kBarOff + 256 + 1024;
  static constexpr uint32_t kS = 0, kDP = 256, kDQ = 384;  // S double-buffered at 0 / 128
};

// Elementwise steps on one 32-column chunk of a TMEM lane:
//   P:  p = exp2(s * scale*log2e + nl2) (0 where not visible)
//   dS: ds = p * (dp + nd)
// nl2 is -lse*log2(e) and nd is -delta (per column in the dK/dV kernel, per
// row in the dQ kernel).  `FULL` (chosen per chunk by a warp-uniform test)
// drops the per-element visibility selects.  p stays in f32 registers; the
// 16-bit packed P (FMT 1: bf16, 0: f16, -1: not needed) feeds an MMA.
template <int FMT, bool FULL, typename NL2, typename Vis>
__device__ __forceinline__ void p_chunk(const uint32_t (&rs)[32], float (&p)[32], uint32_t (&pk)[16], float2 sc2,
                                        NL2 nl2, Vis visible);

// Variant for the dK/dV kernel: p is kept as packed f16 pairs (relative
// error 2^-12, below the 16-bit rounding of dS itself) to save registers.
template <int FMT, bool FULL, typename NL2, typename Vis>
__device__ __forceinline__ void p_chunk_keep16(const uint32_t (&rs)[32], uint32_t (&keep)[16], uint32_t (&pk)[16],
                                               float2 sc2, NL2 nl2, Vis visible) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = 2 * i;
    const float2 x = fma2(make_float2(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1])), sc2, nl2(c));
    float2 e = make_float2(fast_exp2(x.x), fast_exp2(x.y));
    if (!FULL) {
      e.x = visible(c) ? e.x : 0.f;
      e.y = visible(c + 1) ? e.y : 0.f;
    }
    keep[i] = pack_f16x2(e.x, e.y);
    pk[i] = FMT == 1 ? pack_bf16x2(e.x, e.y) : keep[i];
  }
}

template <int FMT, typename ND>
__device__ __forceinline__ void ds_chunk_keep16(const uint32_t (&rd)[32], const uint32_t (&keep)[16], ND nd,
                                                uint32_t out, uint32_t (&pk)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = 2 * i;
    const float2 pf = __half22float2(*reinterpret_cast<const __half2*>(&keep[i]));
    const float2 t = add2(make_float2(__uint_as_float(rd[c]), __uint_as_float(rd[c + 1])), nd(c));
    const float2 ds = mul2(pf, t);
    pk[i] = FMT == 1 ? pack_bf16x2(ds.x, ds.y) : pack_f16x2(ds.x, ds.y);
  }
  tmem_st16(out, pk);
}

// dS spill layout: one 128 x 128 16-bit tile (32 KiB) per live (key tile kt,
// query tile qi) pair of a (batch, head) plane, stored as 8 x 8 core matrices
// (8 keys x 8 queries, one key's 8 queries in 16 contiguous bytes): key k,
// query q sits at byte (q / 8) * 2048 + k * 16 + (q % 8) * 2.  The tensor core
// reads that as the MN-major, unswizzled A operand (M = queries, K = keys) of
// dQ = dS K, and the 32 keys of a warp's TMEM lanes store 512 contiguous bytes
// per 8-query group.  A plane's tiles are ordered by key tile, then query tile;
// key tile kt has the query tiles [i0(kt), nq) with i0 = kt under the causal
// mask (0 otherwise) and none when its first key is at or past kv_len.
__host__ __device__ __forceinline__ long ds_tile_offset(int kt, int nq, int causal) {
  // sum over k < kt of (nq - (causal ? min(k, nq) : 0))
  long off = (long)kt * nq;
  if (causal) off -= kt <= nq ? (long)kt * (kt - 1) / 2 : (long)nq * (nq - 1) / 2 + (long)(kt - nq) * nq;
  return off;
}
__host__ __device__ __forceinline__ long ds_tiles_per_plane(int nq, int kv_len, int causal) {
  return ds_tile_offset((kv_len + 127) / 128, nq, causal);
}

template <int FMT, bool FULL, typename NL2, typename Vis>
__device__ __forceinline__ void p_chunk(const uint32_t (&rs)[32], float (&p)[32], uint32_t (&pk)[16], float2 sc2,
                                        NL2 nl2, Vis visible) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = 2 * i;
    const float2 x = fma2(make_float2(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1])), sc2, nl2(c));
    float2 e = make_float2(fast_exp2(x.x), fast_exp2(x.y));
    if (!FULL) {
      e.x = visible(c) ? e.x : 0.f;
      e.y = visible(c + 1) ? e.y : 0.f;
    }
    p[c] = e.x;
    p[c + 1] = e.y;
    if (FMT >= 0) pk[i] = FMT == 1 ? pack_bf16x2(e.x, e.y) : pack_f16x2(e.x, e.y);
  }
}

// dS of one chunk from dP in registers, packed over the first 16 columns of
// the chunk at TMEM address `out` (the A operand of the dK / dQ MMA).
template <int FMT, typename ND>
__device__ __forceinline__ void ds_chunk(const uint32_t (&rd)[32], const float (&p)[32], ND nd, uint32_t out) {
  uint32_t pk[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = 2 * i;
    const float2 t = add2(make_float2(__uint_as_float(rd[c]), __uint_as_float(rd[c + 1])), nd(c));
    const float2 ds = mul2(make_float2(p[c], p[c + 1]), t);
    pk[i] = FMT == 1 ? pack_bf16x2(ds.x, ds.y) : pack_f16x2(ds.x, ds.y);
  }
  tmem_st16(out, pk);
}

// The thread's 32 or 64 consecutive TMEM columns (one instruction either way).
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[1][32]) { tmem_ld32(taddr, r[0]); }
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[2][32]) { tmem_ld64x1(taddr, r); }

// N consecutive floats of a shared-memory array into registers.
template <int N>
__device__ __forceinline__ void load_cols(const float* src, float (&dst)[N]) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
  for (int i = 0; i < N / 4; ++i) {
    const float4 v = s4[i];
    dst[4 * i] = v.x;
    dst[4 * i + 1] = v.y;
    dst[4 * i + 2] = v.z;
    dst[4 * i + 3] = v.w;
  }
}



// Writes an f32 accumulator row (TMEM columns [col0, col0 + n)) times `scale`
// to a row of T, or zeros when `zero`.
template <typename T, int FMT>
__device__ __forceinline__ void store_acc_row(uint32_t taddr, T* dst, int n, float scale, bool zero,
                                              bool write) {
  for (int c = 0; c < n; c += 32) {
    uint32_t r[32];
    if (!zero) {
      tmem_ld32(taddr + c, r);
      tmem_wait_ld();
    }
    if (write) {
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float a0 = zero ? 0.f : __uint_as_float(r[2 * i]) * scale;
        const float a1 = zero ? 0.f : __uint_as_float(r[2 * i + 1]) * scale;
        pk[i] = FMT == 1 ? pack_bf16x2(a0, a1) : pack_f16x2(a0, a1);
      }
      uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
      for (int i = 0; i < 4; ++i) d4[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
    }
  }
}

// The thread's TMEM lane row of n f32 accumulator columns, times `scale`, to
// an f32 row (the head-split partial sums), or zeros when `zero`.
__device__ __forceinline__ void store_acc_row_f32(uint32_t taddr, float* dst, int n, float scale, bool zero,
                                                  bool write) {
  for (int c = 0; c < n; c += 32) {
    uint32_t r[32];
    if (!zero) {
      tmem_ld32(taddr + c, r);
      tmem_wait_ld();
    }
    if (write) {
      float4* d4 = reinterpret_cast<float4*>(dst + c);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        d4[i] = zero ? make_float4(0.f, 0.f, 0.f, 0.f)
                     : make_float4(__uint_as_float(r[4 * i]) * scale, __uint_as_float(r[4 * i + 1]) * scale,
                                   __uint_as_float(r[4 * i + 2]) * scale, __uint_as_float(r[4 * i + 3]) * scale);
    }
  }
}

// ============================================================================
// dK / dV
// ============================================================================
// P stays in TMEM (packed over the consumed S tile) and dV is a TS MMA.  With
// the spill (ds_buf != nullptr) every dS tile also goes to global memory
// straight from the elementwise warps' registers.
// Head split (parts > 1, for problems with fewer key tiles than SMs): the q
// heads of a kv group are divided over `parts` CTAs per key tile, each of
// which writes its f32 partial dV and scaled dK to `part` ([2][parts][B*Hkv,
// Sk, D]); dkv_part_reduce_kernel sums them in a fixed order.
template <typename T, int D>
__global__ void __launch_bounds__(EwDkv::kThreads, 1)
bwd_dkv_sm100_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                     uint8_t* __restrict__ ds_buf, float* __restrict__ part, int parts,
                     const float* __restrict__ lse, const float* __restrict__ delta,
                     T* __restrict__ dk, T* __restrict__ dv, int H, int Hkv,
                     int Sq, int Sk, int kv_len, int causal, float sm_scale, float scale_log2, int n_kt) {
  using Cfg = DkvCfg<D>;
  constexpr int NQ = Cfg::kNQ, NO = Cfg::kNO;
  constexpr int kEWG = EwDkv::kEWG, kNCH = EwDkv::kNCH, kEWThreads = EwDkv::kEWThreads;
  constexpr int kCertWarp = EwDkv::kCertWarp;
  constexpr int FMT = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t idesc_s = make_idesc_f16(FMT, 128, 128, 0, 0);
  constexpr uint32_t idesc_acc = make_idesc_f16(FMT, 128, D, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {  // uniform over the CTA: nothing initialised yet
    if (threadIdx.x == 0) flag_status(PF_DEV_SMEM_LAYOUT);
    return;
  }
  uint8_t* smem = smem_raw;
  BwdBars* bars = reinterpret_cast<BwdBars*>(smem + Cfg::kBarOff);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  // Causal: heaviest (first) key tiles of every head first.
  const int units = gridDim.x / n_kt;  // (batch, kv head, head part) per key tile
  const int BHk = units / parts;
  const int kt = blockIdx.x / units;
  const int bhk = (blockIdx.x % units) / parts, hp = (blockIdx.x % units) % parts;
  const int b = bhk / Hkv, hk = bhk % Hkv;
  const int G = H / Hkv, Gp = G / parts;
  const int g0 = hk * G + hp * Gp;  // first q head of this CTA, within the batch
  const int k0 = kt * 128;
  const int nq = (Sq + 127) / 128;
  int i0 = causal ? k0 / 128 : 0;
  if (k0 >= kv_len) i0 = nq;  // no live key in this tile
  const int nqi = max(0, nq - i0);
  const int n_it = Gp * nqi;

  if (threadIdx.x == 0) {
    mbar_init(&bars->fixed, 1);
    for (int s = 0; s < NQ; ++s) {
      mbar_init(&bars->full[s], 1 + 32);  // TMA tx arrive + the producer warp's 32 stat writers
      mbar_init(&bars->empty[s], 1);
    }
    for (int s = 0; s < NO; ++s) {
      mbar_init(&bars->vfull[s], 1);
      mbar_init(&bars->vempty[s], 1);
    }
    mbar_init(&bars->s_full[0], 1);
    mbar_init(&bars->dp_full, 1);
    mbar_init(&bars->p_ready, kEWThreads);
    mbar_init(&bars->ds_ready, kEWThreads + 1);  // + certifier: dO(it+1) landed
    mbar_init(&bars->p_half, kEWThreads);
    mbar_init(&bars->ds_half, kEWThreads);
    mbar_init(&bars->s_free, kEWThreads + 1);  // + certifier: Q(it+1) and its statistics landed
    mbar_init(&bars->stats_free[0], kEWThreads);
    mbar_init(&bars->stats_free[1], kEWThreads);
    mbar_init(&bars->done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  float* stats = reinterpret_cast<float*>(smem + Cfg::kStatOff);

  if (warp == 0) {
    if (n_it > 0) {
      // All 32 lanes: lane 0 issues the TMA copies, every lane stages four of
      // the 128 (-lse*log2e, -delta) column statistics of the query tile.
      const int kv_plane = b * Hkv + hk;
      if (lane == 0) {
        mbar_expect_tx(&bars->fixed, 2 * Cfg::kTile);
        for (int c = 0; c < Cfg::kBoxes; ++c) {
          tma_load_3d(smem + Cfg::kFixedOff + c * 128 * 128, &tm_k, &bars->fixed, c * 64, k0, kv_plane);
          tma_load_3d(smem + Cfg::kFixedOff + Cfg::kTile + c * 128 * 128, &tm_v, &bars->fixed, c * 64, k0,
                      kv_plane);
        }
      }
      // Column statistics are fetched one tile ahead, so their global-load
      // latency stays off the Q barrier.
      float pl[4], pd[4];
      auto fetch_stats = [&](int it) {
        const int plane = b * H + g0 + it / nqi;
        const int qi = i0 + it % nqi;
        const long srow = (long)plane * Sq;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int qp = qi * 128 + lane + 32 * u;
          pl[u] = qp < Sq ? -lse[srow + qp] * kLog2e : 0.f;
          pd[u] = qp < Sq ? -delta[srow + qp] : 0.f;
        }
      };
      fetch_stats(0);
      int last_q = -1, last_do = -1;
      for (int it = 0; it < n_it; ++it) {
        const int s = it % NQ, so = it % NO, ss = it & 1;
        if (it >= NQ && !mbar_wait(&bars->empty[s], ((it / NQ) - 1) & 1)) break;
        if (lane == 0) trace(15, it - 1);
        const int qi = i0 + it % nqi;
        const int plane = b * H + g0 + it / nqi;
        if (lane == 0) {
          mbar_expect_tx(&bars->full[s], Cfg::kTile);
          for (int c = 0; c < Cfg::kBoxes; ++c)
            tma_load_3d(smem + Cfg::kQOff + s * Cfg::kTile + c * 128 * 128, &tm_q, &bars->full[s], c * 64,
                        qi * 128, plane);
        }
        last_q = it;
        // The statistics slot of tile it - 2 has been read by its dS step.
        if (it >= 2 && !mbar_wait(&bars->stats_free[ss], ((it >> 1) - 1) & 1)) break;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          stats[ss * 256 + lane + 32 * u] = pl[u];
          stats[ss * 256 + 128 + lane + 32 * u] = pd[u];
        }
        mbar_arrive(&bars->full[s]);
        if (it + 1 < n_it) fetch_stats(it + 1);
        // dO is needed later (by dP) and released earlier (after dV) than Q.
        if (it >= NO && !mbar_wait(&bars->vempty[so], ((it / NO) - 1) & 1)) break;
        if (lane == 0) {
          mbar_expect_tx(&bars->vfull[so], Cfg::kTile);
          for (int c = 0; c < Cfg::kBoxes; ++c)
            tma_load_3d(smem + Cfg::kOOff + so * Cfg::kTile + c * 128 * 128, &tm_do, &bars->vfull[so], c * 64,
                        qi * 128, plane);
        }
        last_do = it;
      }
      if (lane == 0) {  // exit drain: no copy may land after the CTA is gone
        mbar_wait(&bars->fixed, 0);
        drain_ring(bars->full, NQ, last_q);
        drain_ring(bars->vfull, NO, last_do);
      }
    }
  } else if (warp == 1) {
    // Tensor-core order per iteration:
    //   dV(it) [P(it) in TMEM, in two halves]   S(it+1)   dK(it) [dS(it) in TMEM, two halves]   dP(it+1)
    // The elementwise warps release the S tile as soon as they have loaded
    // it, so S(it+1) queues behind dV(it) (which reads P over the S columns;
    // the tensor core runs its queue in order) and runs under the dS
    // arithmetic of tile it.  dS stays in TMEM; dP(it+1) overwrites it only
    // after dK(it) read it.
    if (lane == 0 && n_it > 0) {
      bool ok = mbar_wait(&bars->fixed, 0);
      tc_fence_after();
      const uint32_t k_addr = sbase + Cfg::kFixedOff, v_addr = k_addr + Cfg::kTile;
      const uint64_t kd = desc_k_base<128>(k_addr), vd = desc_k_base<128>(v_addr);
      auto q_stage = [&](int it) { return sbase + Cfg::kQOff + (it % NQ) * Cfg::kTile; };
      auto o_stage = [&](int it) { return sbase + Cfg::kOOff + (it % NO) * Cfg::kTile; };
      auto issue_s = [&](int it) {
        const uint64_t qd = desc_k_base<128>(q_stage(it));
        umma_ss(tmem + Cfg::kS, kd, qd, idesc_s, 0);
#pragma unroll
        for (int kk = 1; kk < D / 16; ++kk)
          umma_ss_acc(tmem + Cfg::kS, kd + koff<128>(kk), qd + koff<128>(kk), idesc_s);
        umma_commit(&bars->s_full[0]);
      };
      auto issue_dp = [&](int it) -> bool {
        if (it == 0 && !mbar_wait_spin(&bars->vfull[0], 0)) return false;  // later tiles: certified
        tc_fence_after();
        const uint64_t od = desc_k_base<128>(o_stage(it));
        umma_ss(tmem + Cfg::kDP, vd, od, idesc_s, 0);
#pragma unroll
        for (int kk = 1; kk < D / 16; ++kk)
          umma_ss_acc(tmem + Cfg::kDP, vd + koff<128>(kk), od + koff<128>(kk), idesc_s);
        umma_commit(&bars->dp_full);
        return true;
      };
      if (ok) ok = mbar_wait_spin(&bars->full[0], 0);
      if (ok) {
        tc_fence_after();
        issue_s(0);
        ok = issue_dp(0);
      }
      for (int it = 0; ok && it < n_it; ++it) {
        // dV(it) in two halves: k-steps {0,1,4,5} read the first 32-column
        // chunk each elementwise warpgroup wrote (p_half), {2,3,6,7} the
        // second (p_ready).
        const uint64_t om = desc_mn_base<128>(o_stage(it));
        ok = mbar_wait_spin(&bars->p_half, it & 1);
        if (!ok) break;
        trace(1, it);
        tc_fence_after();
        umma_ts(tmem + Cfg::kDV, tmem + Cfg::kS, om, idesc_acc, it > 0);
        umma_ts_acc(tmem + Cfg::kDV, tmem + Cfg::kS + split_packed_col(1), om + mnoff(1), idesc_acc);
        umma_ts_acc(tmem + Cfg::kDV, tmem + Cfg::kS + split_packed_col(4), om + mnoff(4), idesc_acc);
        umma_ts_acc(tmem + Cfg::kDV, tmem + Cfg::kS + split_packed_col(5), om + mnoff(5), idesc_acc);
        ok = mbar_wait_spin(&bars->p_ready, it & 1);
        if (!ok) break;
        tc_fence_after();
        umma_ts_acc(tmem + Cfg::kDV, tmem + Cfg::kS + split_packed_col(2), om + mnoff(2), idesc_acc);
        umma_ts_acc(tmem + Cfg::kDV, tmem + Cfg::kS + split_packed_col(3), om + mnoff(3), idesc_acc);
        umma_ts_acc(tmem + Cfg::kDV, tmem + Cfg::kS + split_packed_col(6), om + mnoff(6), idesc_acc);
        umma_ts_acc(tmem + Cfg::kDV, tmem + Cfg::kS + split_packed_col(7), om + mnoff(7), idesc_acc);
        umma_commit(&bars->vempty[it % NO]);
        if (it + 1 < n_it) {
          ok = mbar_wait_spin(&bars->s_free, it & 1);  // Q(it+1) certified
          if (!ok) break;
          tc_fence_after();
          issue_s(it + 1);
          trace(14, it);
        }
        trace(2, it);
        // dK(it) in the same two halves (ds_half, then ds_ready).
        const uint64_t qm = desc_mn_base<128>(q_stage(it));
        ok = mbar_wait_spin(&bars->ds_half, it & 1);
        if (!ok) break;
        tc_fence_after();
        umma_ts(tmem + Cfg::kDK, tmem + Cfg::kDP, qm, idesc_acc, it > 0);
        umma_ts_acc(tmem + Cfg::kDK, tmem + Cfg::kDP + split_packed_col(1), qm + mnoff(1), idesc_acc);
        umma_ts_acc(tmem + Cfg::kDK, tmem + Cfg::kDP + split_packed_col(4), qm + mnoff(4), idesc_acc);
        umma_ts_acc(tmem + Cfg::kDK, tmem + Cfg::kDP + split_packed_col(5), qm + mnoff(5), idesc_acc);
        ok = mbar_wait_spin(&bars->ds_ready, it & 1);
        if (!ok) break;
        trace(3, it);
        tc_fence_after();
        umma_ts_acc(tmem + Cfg::kDK, tmem + Cfg::kDP + split_packed_col(2), qm + mnoff(2), idesc_acc);
        umma_ts_acc(tmem + Cfg::kDK, tmem + Cfg::kDP + split_packed_col(3), qm + mnoff(3), idesc_acc);
        umma_ts_acc(tmem + Cfg::kDK, tmem + Cfg::kDP + split_packed_col(6), qm + mnoff(6), idesc_acc);
        umma_ts_acc(tmem + Cfg::kDK, tmem + Cfg::kDP + split_packed_col(7), qm + mnoff(7), idesc_acc);
        umma_commit(&bars->empty[it % NQ]);
        if (it + 1 < n_it && !(ok = issue_dp(it + 1))) break;
        trace(4, it);
      }
      umma_commit(&bars->done);
    }
  } else if (warp == kCertWarp) {
    if (lane == 0) {
      bool ok = true;
      for (int it = 0; ok && it < n_it; ++it) {
        const bool next = it + 1 < n_it;
        if (next) ok = mbar_wait(&bars->full[(it + 1) % NQ], ((it + 1) / NQ) & 1);
        if (!ok) break;
        mbar_arrive(&bars->s_free);
        if (next) ok = mbar_wait(&bars->vfull[(it + 1) % NO], ((it + 1) / NO) & 1);
        if (!ok) break;
        mbar_arrive(&bars->ds_ready);
        // Never arrive twice in one phase.
        ok = mbar_wait(&bars->s_free, it & 1) && mbar_wait(&bars->ds_ready, it & 1);
      }
    }
  } else if (warp >= 2) {
    const int cw = (warp - 2) / 4;      // elementwise warpgroup
    const int col0 = 32 * kNCH * cw;    // its first query column of the tile
    const int quad = warp % 4;
    const int row = quad * 32 + lane;   // key row within the tile
    const int kpos = k0 + row;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const bool key_ok = kpos < kv_len;
    const bool tr = lane == 0 && quad == 2 && cw == 0;  // trace writer
    const float2 sc2 = make_float2(scale_log2, scale_log2);
    const long plane_tiles = ds_tiles_per_plane(nq, kv_len, causal);
    const long kt_tiles = ds_tile_offset(kt, nq, causal);
    const uint64_t ds_pol = l2_evict_first_policy();
    bool ok = true;
    for (int it = 0; ok && it < n_it; ++it) {
      const int st = it % NQ, ss = it & 1;
      const int qc = (i0 + it % nqi) * 128 + col0;  // first query column of this thread
      // The slot's statistics were written by the producer warp before its
      // arrive on full[st]; the slot is not refilled before stats_free.
      // Loading them before the S wait keeps their latency off the critical path.
      if (!mbar_wait(&bars->full[st], (it / NQ) & 1)) { ok = false; break; }
      float nl2[kNCH * 32];
      load_cols<kNCH * 32>(stats + ss * 256 + col0, nl2);
      if (!mbar_wait_spin(&bars->s_full[0], it & 1)) { ok = false; break; }
      if (tr) trace(8, it);
      tc_fence_after();
      uint32_t keep[kNCH][16], pk[kNCH][16];
      {
        uint32_t rs[kNCH][32];
        tmem_ld_cols(lane_base + Cfg::kS + col0, rs);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&bars->s_free);  // S(it+1) may now overwrite the tile
        // Chunk by chunk: P of a thread's first chunk is published (p_half)
        // before the second is computed, so dV can start on half the queries.
        static_assert(kNCH == 2, "the two-phase P / dS publication assumes two chunks per thread");
#pragma unroll
        for (int h = 0; h < kNCH; ++h) {
          const int q0 = qc + 32 * h;
          auto nl2_h = [&](int c) { return make_float2(nl2[32 * h + c], nl2[32 * h + c + 1]); };
          if ((k0 + 127 < kv_len) && (q0 + 32 <= Sq) && (!causal || q0 >= k0 + 127)) {
            p_chunk_keep16<FMT, true>(rs[h], keep[h], pk[h], sc2, nl2_h, [](int) { return true; });
          } else {
            p_chunk_keep16<FMT, false>(rs[h], keep[h], pk[h], sc2, nl2_h, [&](int c) {
              const int qp = q0 + c;
              return key_ok && qp < Sq && (!causal || qp >= kpos);
            });
          }
          // P packed over the chunk's own (consumed) S columns: the A operand of dV.
          tmem_st16(lane_base + Cfg::kS + col0 + 32 * h, pk[h]);
          if (h == 0) {
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bars->p_half);
          }
        }
      }
      if (tr) trace(7, it);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_ready);
      float nd[kNCH * 32];
      load_cols<kNCH * 32>(stats + ss * 256 + 128 + col0, nd);
      mbar_arrive(&bars->stats_free[ss]);  // release: the slot's loads are done
      if (tr) trace(9, it);
      if (!mbar_wait_spin(&bars->dp_full, it & 1)) { ok = false; break; }
      if (tr) trace(0, it);
      tc_fence_after();
      // This thread's key row of the spilled tile: 8-query group q8 at q8 * 2048 + row * 16.
      uint8_t* ds_row = ds_buf != nullptr
                            ? ds_buf + ((long)(b * H + g0 + it / nqi) * plane_tiles + kt_tiles + it % nqi) *
                                           (128 * 128 * 2) + row * 16
                            : nullptr;
      // Each chunk's spill stores follow the barrier that lets dK read it.
      auto spill = [&](int h, const uint32_t (&pkd)[16]) {
        if (ds_row == nullptr) return;
#pragma unroll
        for (int g = 0; g < 4; ++g)
          st_global_hint(ds_row + ((col0 + 32 * h) / 8 + g) * 2048,
                         make_uint4(pkd[4 * g], pkd[4 * g + 1], pkd[4 * g + 2], pkd[4 * g + 3]), ds_pol);
      };
      uint32_t pkd[kNCH][16];
#pragma unroll
      for (int h = 0; h < kNCH; ++h) {
        uint32_t rd[32];
        tmem_ld32(lane_base + Cfg::kDP + col0 + 32 * h, rd);
        tmem_wait_ld();
        ds_chunk_keep16<FMT>(rd, keep[h], [&](int c) { return make_float2(nd[32 * h + c], nd[32 * h + c + 1]); },
                             lane_base + Cfg::kDP + col0 + 32 * h, pkd[h]);
        if (h == 0) {  // first chunk of dS in place: dK may start on it
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&bars->ds_half);
          spill(0, pkd[0]);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->ds_ready);
      spill(1, pkd[1]);
      if (tr) trace(10, it);
    }
    // Epilogue: the first half of the warpgroups writes dV, the second half
    // dK (scaled), each a contiguous slice of the D columns.
    const bool have = n_it > 0 && ok && mbar_wait(&bars->done, 0);
    if (n_it > 0) tc_fence_after();
    const bool write = kpos < Sk;
    const long orow = ((long)(b * Hkv + hk) * Sk + kpos) * D;
    constexpr int kHalf = kEWG / 2, kCols = D / kHalf;
    const int cpart = cw % kHalf;
    if (parts > 1) {
      // f32 partial rows: [dV | dK][hp][b * Hkv + hk][kpos][D]
      const size_t plane_elems = (size_t)parts * BHk * Sk * D;
      float* prow = part + ((size_t)hp * BHk + bhk) * Sk * D + (size_t)kpos * D + cpart * kCols;
      if (cw < kHalf)
        store_acc_row_f32(lane_base + Cfg::kDV + cpart * kCols, prow, kCols, 1.f, !have, write);
      else
        store_acc_row_f32(lane_base + Cfg::kDK + cpart * kCols, prow + plane_elems, kCols, sm_scale, !have, write);
    } else if (cw < kHalf) {
      store_acc_row<T, FMT>(lane_base + Cfg::kDV + cpart * kCols, dv + orow + cpart * kCols, kCols, 1.f, !have,
                            write);
    } else {
      store_acc_row<T, FMT>(lane_base + Cfg::kDK + cpart * kCols, dk + orow + cpart * kCols, kCols, sm_scale,
                            !have, write);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // `done` follows every MMA this CTA issued (committed after the issue
    // loop on every path), so TMEM is never freed under a running MMA.
    if (lane == 0 && n_it > 0) mbar_wait(&bars->done, 0);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================
// dQ
// ============================================================================
template <typename T, int D>
__global__ void __launch_bounds__(EwDq::kThreads, 1)
bwd_dq_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                    const float* __restrict__ lse, const float* __restrict__ delta, T* __restrict__ dq,
                    int H, int Hkv, int Sq, int kv_len, int causal, float sm_scale, float scale_log2,
                    int n_qt) {
  using Cfg = DqCfg<D>;
  constexpr int NK = Cfg::kNK, NV = Cfg::kNV;
  constexpr int kNCH = EwDq::kNCH, kEWThreads = EwDq::kEWThreads;
  constexpr int kCertWarp = EwDq::kCertWarp;
  constexpr int FMT = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t idesc_s = make_idesc_f16(FMT, 128, 128, 0, 0);
  constexpr uint32_t idesc_acc = make_idesc_f16(FMT, 128, D, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  BwdBars* bars = reinterpret_cast<BwdBars*>(smem + Cfg::kBarOff);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  // Heaviest (last, under causal) query tiles first.
  const int BH = gridDim.x / n_qt;
  const int bh = blockIdx.x % BH;
  const int qt = n_qt - 1 - blockIdx.x / BH;
  const int b = bh / H, h = bh % H;
  const int hk = h / (H / Hkv);
  const int q0 = qt * 128;
  const int kvb = (kv_len + 127) / 128;
  const int q_last = min(q0 + 127, Sq - 1);
  const int n_it = causal ? min(kvb, q_last / 128 + 1) : kvb;

  if (threadIdx.x == 0) {
    mbar_init(&bars->fixed, 1);
    for (int s = 0; s < NK; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int s = 0; s < NV; ++s) {
      mbar_init(&bars->vfull[s], 1);
      mbar_init(&bars->vempty[s], 1);
    }
    mbar_init(&bars->s_full[0], 1);
    mbar_init(&bars->s_full[1], 1);
    mbar_init(&bars->dp_full, 1);
    mbar_init(&bars->ds_ready, kEWThreads + 1);  // + certifier: V(it+1) and K(it+2) landed
    mbar_init(&bars->done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0 && n_it > 0) {
      mbar_expect_tx(&bars->fixed, 2 * Cfg::kTile);
      for (int c = 0; c < Cfg::kBoxes; ++c) {
        tma_load_3d(smem + Cfg::kFixedOff + c * 128 * 128, &tm_q, &bars->fixed, c * 64, q0, bh);
        tma_load_3d(smem + Cfg::kFixedOff + Cfg::kTile + c * 128 * 128, &tm_do, &bars->fixed, c * 64, q0, bh);
      }
      const int kv_plane = b * Hkv + hk;
      int last_k = -1, last_v = -1;
      for (int it = 0; it < n_it; ++it) {
        const int sk = it % NK, sv = it % NV;
        if (it >= NK && !mbar_wait(&bars->empty[sk], ((it / NK) - 1) & 1)) break;
        mbar_expect_tx(&bars->full[sk], Cfg::kTile);
        for (int c = 0; c < Cfg::kBoxes; ++c)
          tma_load_3d(smem + Cfg::kKOff + sk * Cfg::kTile + c * 128 * 128, &tm_k, &bars->full[sk], c * 64,
                      it * 128, kv_plane);
        last_k = it;
        if (it >= NV && !mbar_wait(&bars->vempty[sv], ((it / NV) - 1) & 1)) break;
        mbar_expect_tx(&bars->vfull[sv], Cfg::kTile);
        for (int c = 0; c < Cfg::kBoxes; ++c)
          tma_load_3d(smem + Cfg::kVOff + sv * Cfg::kTile + c * 128 * 128, &tm_v, &bars->vfull[sv], c * 64,
                      it * 128, kv_plane);
        last_v = it;
      }
      // Exit drain: no copy may land after the CTA is gone.
      mbar_wait(&bars->fixed, 0);
      drain_ring(bars->full, NK, last_k);
      drain_ring(bars->vfull, NV, last_v);
    }
  } else if (warp == 1) {
    // Tensor-core order per iteration:  [dS(it) in TMEM] dQ(it) dP(it+1) S(it+2)
    // One poll per tile: each barrier poll the issuing thread waits on costs
    // tensor-core time, more than overlapping dP(it+1) with the dS arithmetic
    // of tile it gains.  S is double-buffered and dS(it) is written over the
    // consumed S(it) tile; S(it+2) (same buffer) queues behind dQ(it).
    if (lane == 0 && n_it > 0) {
      bool ok = mbar_wait(&bars->fixed, 0);
      tc_fence_after();
      const uint32_t q_addr = sbase + Cfg::kFixedOff, do_addr = q_addr + Cfg::kTile;
      const uint64_t qd = desc_k_base<128>(q_addr), od = desc_k_base<128>(do_addr);
      auto k_tile = [&](int it) { return sbase + Cfg::kKOff + (it % NK) * Cfg::kTile; };
      auto issue_s = [&](int it) -> bool {  // K(0), K(1) polled here; later tiles certified
        if (it < 2 && !mbar_wait_spin(&bars->full[it % NK], (it / NK) & 1)) return false;
        tc_fence_after();
        const uint32_t k_addr = k_tile(it);
        const uint64_t kdesc = desc_k_base<128>(k_addr);
        const uint32_t dst = tmem + Cfg::kS + 128 * (it & 1);
        umma_ss(dst, qd, kdesc, idesc_s, 0);
#pragma unroll
        for (int kk = 1; kk < D / 16; ++kk) umma_ss_acc(dst, qd + koff<128>(kk), kdesc + koff<128>(kk), idesc_s);
        umma_commit(&bars->s_full[it & 1]);
        return true;
      };
      auto issue_dp = [&](int it) -> bool {  // V(0) polled here; later tiles certified
        if (it == 0 && !mbar_wait_spin(&bars->vfull[0], 0)) return false;
        tc_fence_after();
        const uint32_t v_addr = sbase + Cfg::kVOff + (it % NV) * Cfg::kTile;
        const uint64_t vdesc = desc_k_base<128>(v_addr);
        umma_ss(tmem + Cfg::kDP, od, vdesc, idesc_s, 0);
#pragma unroll
        for (int kk = 1; kk < D / 16; ++kk)
          umma_ss_acc(tmem + Cfg::kDP, od + koff<128>(kk), vdesc + koff<128>(kk), idesc_s);
        umma_commit(&bars->vempty[it % NV]);
        umma_commit(&bars->dp_full);
        return true;
      };
      if (ok) ok = issue_s(0) && (n_it < 2 || issue_s(1)) && issue_dp(0);
      for (int it = 0; ok && it < n_it; ++it) {
        trace(2, it);
        ok = mbar_wait_spin(&bars->ds_ready, it & 1);
        if (!ok) break;
        trace(3, it);
        tc_fence_after();
        const uint32_t k_addr = k_tile(it);
        const uint32_t ds_addr = tmem + Cfg::kS + 128 * (it & 1);
        const uint64_t km = desc_mn_base<128>(k_addr);
        umma_ts(tmem + Cfg::kDQ, ds_addr, km, idesc_acc, it > 0);
#pragma unroll
        for (int kk = 1; kk < 8; ++kk)
          umma_ts_acc(tmem + Cfg::kDQ, ds_addr + split_packed_col(kk), km + mnoff(kk), idesc_acc);
        umma_commit(&bars->empty[it % NK]);
        if (it + 1 < n_it && !(ok = issue_dp(it + 1))) break;
        if (it + 2 < n_it && !(ok = issue_s(it + 2))) break;
        trace(4, it);
      }
      umma_commit(&bars->done);
    }
  } else if (warp == kCertWarp) {
    if (lane == 0) {
      bool ok = true;
      for (int it = 0; ok && it < n_it; ++it) {
        if (it + 1 < n_it) ok = mbar_wait(&bars->vfull[(it + 1) % NV], ((it + 1) / NV) & 1);
        if (ok && it + 2 < n_it) ok = mbar_wait(&bars->full[(it + 2) % NK], ((it + 2) / NK) & 1);
        if (!ok) break;
        mbar_arrive(&bars->ds_ready);
        ok = mbar_wait(&bars->ds_ready, it & 1);  // never arrive twice in one phase
      }
    }
  } else if (warp >= 2) {
    const int cw = (warp - 2) / 4;      // elementwise warpgroup
    const int col0 = 32 * kNCH * cw;    // its first key column of the tile
    const int quad = warp % 4;
    const int row = quad * 32 + lane;   // query row within the tile
    const int qpos = q0 + row;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const long srow = (long)bh * Sq + qpos;
    const float nl2 = qpos < Sq ? -lse[srow] * kLog2e : 0.f;
    const float nd = qpos < Sq ? -delta[srow] : 0.f;
    const bool tr = lane == 0 && quad == 2 && cw < 2;
    bool ok = true;
    const float2 sc2 = make_float2(scale_log2, scale_log2);
    const float2 nl2v = make_float2(nl2, nl2), ndv = make_float2(nd, nd);
    for (int it = 0; it < n_it; ++it) {
      if (!mbar_wait_spin(&bars->s_full[it & 1], (it >> 1) & 1)) { ok = false; break; }
      if (tr) trace(8 + 3 * cw, it);
      tc_fence_after();
      const uint32_t s_addr = lane_base + Cfg::kS + 128 * (it & 1) + col0;
      const int kc = it * 128 + col0;  // first key column of this thread
      float p[kNCH][32];
      {
        uint32_t rs[kNCH][32];
        uint32_t unused[16];
        tmem_ld_cols(s_addr, rs);
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < kNCH; ++h) {
          const int kb = kc + 32 * h;
          if ((kb + 32 <= kv_len) && (!causal || kb + 31 <= q0)) {
            p_chunk<-1, true>(rs[h], p[h], unused, sc2, [&](int) { return nl2v; }, [](int) { return true; });
          } else {
            p_chunk<-1, false>(rs[h], p[h], unused, sc2, [&](int) { return nl2v; }, [&](int c) {
              const int kp = kb + c;
              return kp < kv_len && (!causal || kp <= qpos);
            });
          }
        }
      }
      if (tr) trace(9 + 3 * cw, it);
      if (!mbar_wait_spin(&bars->dp_full, it & 1)) { ok = false; break; }
      tc_fence_after();
      {
        uint32_t rd[kNCH][32];
        tmem_ld_cols(lane_base + Cfg::kDP + col0, rd);
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < kNCH; ++h)
          ds_chunk<FMT>(rd[h], p[h], [&](int) { return ndv; }, s_addr + 32 * h);
      }
      tmem_wait_st();
      tc_fence_before();
      // Arrivals for phase it cannot run ahead: dP(it) was issued only after
      // phase it-1 of ds_ready completed.
      mbar_arrive(&bars->ds_ready);
      if (tr) trace(10 + 3 * cw, it);
    }
    const bool have = n_it > 0 && ok && mbar_wait(&bars->done, 0);
    if (n_it > 0) tc_fence_after();
    // The first two warpgroups write half of the D columns of their rows each.
    if (cw < 2)
      store_acc_row<T, FMT>(lane_base + Cfg::kDQ + cw * (D / 2), dq + srow * D + cw * (D / 2), D / 2, sm_scale,
                            !have, qpos < Sq);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // `done` follows every MMA this CTA issued (committed after the issue
    // loop on every path), so TMEM is never freed under a running MMA.
    if (lane == 0 && n_it > 0) mbar_wait(&bars->done, 0);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================
// dQ from the spilled dS tiles: dQ = scale * sum over key tiles of dS K
// ============================================================================
// The dK/dV kernel wrote every dS tile it computed (16-bit, rows = keys,
// columns = queries); dQ of a 128-row query tile is then one GEMM over its key
// tiles, A = dS (M = queries, K = keys, MN-major as stored) and B = K
// (K = keys, N = D, MN-major), without recomputing S and dP.  It streams each
// dS tile once from HBM, so it is bandwidth-bound (32 KB per tile pair
// against 128 x 128 x D MACs).
// Persistent: one CTA per SM walks query-tile items (heaviest first, in
// serpentine rounds), the producer streams (dS, K) stages across item
// boundaries and the dQ accumulator is double-buffered in TMEM, so an item's
// epilogue overlaps the next item's loads and MMAs.
// Warp 0: TMA producer; warp 1: MMA issuer; warps 2-5: epilogue (a warp reads
// TMEM lane quadrant warp % 4).
template <int D>
struct DqGemmCfg {
  static constexpr int kNS = D == 128 ? 3 : 4;
  static constexpr int kBoxes = D / 64;
  static constexpr int kDsTile = 128 * 128 * 2;
  static constexpr int kKTile = 128 * D * 2;
  static constexpr int kStage = kDsTile + kKTile;
  static constexpr int kBarOff = kNS * kStage;
  static constexpr int kSmem = kBarOff + 256 + 1024;
  static constexpr int kThreads = 6 * 32;
  static constexpr uint32_t kCols = 2 * D;  // TMEM: two dQ accumulators
};

struct DqGemmBars {
  uint64_t full[4], empty[4];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t done;
  uint32_t tmem_base;
};

// The item a CTA processes in its round r (serpentine over the CTAs).
__device__ __forceinline__ int dq_gemm_item(int r, int cta, int ctas) {
  return r * ctas + ((r & 1) ? ctas - 1 - cta : cta);
}

template <typename T, int D>
__global__ void __launch_bounds__(DqGemmCfg<D>::kThreads, 1)
bwd_dq_gemm_sm100_kernel(const uint8_t* __restrict__ ds_buf, const __grid_constant__ CUtensorMap tm_k,
                         T* __restrict__ dq, int H, int Hkv, int Sq, int kv_len, int causal, float sm_scale,
                         int n_qt, int n_items) {
  using Cfg = DqGemmCfg<D>;
  constexpr int NS = Cfg::kNS;
  constexpr int FMT = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t idesc = make_idesc_f16(FMT, 128, D, 1, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  DqGemmBars* bars = reinterpret_cast<DqGemmBars*>(smem + Cfg::kBarOff);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  const int BH = n_items / n_qt;
  const int nkt = (kv_len + 127) / 128;
  const long plane_tiles = ds_tiles_per_plane(n_qt, kv_len, causal);
  const int ctas = gridDim.x, cta = blockIdx.x;
  const int n_rounds = (n_items + ctas - 1) / ctas;
  // Item w: query tile qt = n_qt - 1 - w / BH (heaviest first under causal), plane bh = w % BH.
  auto item_qt = [&](int w) { return n_qt - 1 - w / BH; };
  auto item_iters = [&](int w) { return causal ? min(nkt, item_qt(w) + 1) : nkt; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->acc_full[a], 1);
      mbar_init(&bars->acc_empty[a], 128);
    }
    mbar_init(&bars->done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, Cfg::kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      int g = 0, last = -1;  // stage counter across items
      bool ok = true;
      for (int r = 0; ok && r < n_rounds; ++r) {
        const int w = dq_gemm_item(r, cta, ctas);
        if (w >= n_items) continue;
        const int qt = item_qt(w), bh = w % BH, n_it = item_iters(w);
        const int kvp = (bh / H) * Hkv + (bh % H) / (H / Hkv);
        for (int it = 0; it < n_it; ++it, ++g) {
          const int s = g % NS;
          if (g >= NS && !mbar_wait(&bars->empty[s], ((g / NS) - 1) & 1)) { ok = false; break; }
          uint8_t* dst = smem + s * Cfg::kStage;
          const long tile = (long)bh * plane_tiles + ds_tile_offset(it, n_qt, causal) + (qt - (causal ? it : 0));
          mbar_expect_tx(&bars->full[s], Cfg::kStage);
          // The spilled tile is already in the tensor core's operand layout: one bulk copy (read once: evict first).
          bulk_load_hint(dst, ds_buf + tile * Cfg::kDsTile, Cfg::kDsTile, &bars->full[s], pol);
          for (int c = 0; c < Cfg::kBoxes; ++c)
            tma_load_3d(dst + Cfg::kDsTile + c * 128 * 128, &tm_k, &bars->full[s], c * 64, it * 128, kvp);
          last = g;
        }
      }
      drain_ring(bars->full, NS, last);  // no copy may land after the CTA is gone
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = true;
      int g = 0, j = 0;  // stage counter, item counter of this CTA
      for (int r = 0; ok && r < n_rounds; ++r) {
        const int w = dq_gemm_item(r, cta, ctas);
        if (w >= n_items) continue;
        const int n_it = item_iters(w);
        const int ab = j & 1;
        if (j >= 2 && !mbar_wait_spin(&bars->acc_empty[ab], ((j >> 1) - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t acc = tmem + ab * D;
        for (int it = 0; it < n_it; ++it, ++g) {
          const int s = g % NS;
          if (!mbar_wait_spin(&bars->full[s], (g / NS) & 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t ds_addr = sbase + s * Cfg::kStage;
          // A = dS: MN-major, unswizzled; 8-key groups 128 B apart (LBO), 8-query groups 2048 B apart (SBO);
          // k-step kk (16 keys) starts 256 B further.
          const uint64_t ad = smem_desc_noswz(ds_addr, 128, 2048), bd = desc_mn_base<128>(ds_addr + Cfg::kDsTile);
          umma_ss(acc, ad, bd, idesc, it > 0);
#pragma unroll
          for (int kk = 1; kk < 8; ++kk) umma_ss_acc(acc, ad + (uint64_t)(kk * 256 >> 4), bd + mnoff(kk), idesc);
          umma_commit(&bars->empty[s]);
        }
        if (!ok) break;
        umma_commit(&bars->acc_full[ab]);
        ++j;
      }
      umma_commit(&bars->done);
    }
  } else {
    const int quad = warp % 4;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    bool ok = true;
    int j = 0;
    for (int r = 0; r < n_rounds; ++r) {
      const int w = dq_gemm_item(r, cta, ctas);
      if (w >= n_items) continue;
      const int qpos = item_qt(w) * 128 + row, bh = w % BH;
      const int ab = j & 1;
      if (ok) ok = mbar_wait(&bars->acc_full[ab], (j >> 1) & 1);
      tc_fence_after();
      store_acc_row<T, FMT>(lane_base + ab * D, dq + ((long)bh * Sq + qpos) * D, D, sm_scale, !ok, qpos < Sq);
      tc_fence_before();
      mbar_arrive(&bars->acc_empty[ab]);
      ++j;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // `done` follows every MMA this CTA issued, so TMEM is never freed under a running MMA.
    if (lane == 0) mbar_wait(&bars->done, 0);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kCols);
  }
}

// dK, dV = the sum over head parts of the f32 partials (fixed order), cast to T.
template <typename T>
__global__ void dkv_part_reduce_kernel(const float* __restrict__ part, T* __restrict__ dk, T* __restrict__ dv,
                                       long n4, int parts) {
  const long n = n4 * 4;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < 2 * n4; i += (long)gridDim.x * blockDim.x) {
    const bool is_k = i >= n4;
    const long j = (is_k ? i - n4 : i) * 4;
    const float* src = part + (is_k ? (long)parts * n : 0) + j;
    float4 acc = *reinterpret_cast<const float4*>(src);
    for (int p = 1; p < parts; ++p) {
      const float4 v = *reinterpret_cast<const float4*>(src + (long)p * n);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    T* dst = (is_k ? dk : dv) + j;
    dst[0] = from_f<T>(acc.x);
    dst[1] = from_f<T>(acc.y);
    dst[2] = from_f<T>(acc.z);
    dst[3] = from_f<T>(acc.w);
  }
}

template <typename T, int D>
cudaError_t launch_dkv_t(const BwdArgs& a) {
  using Cfg = DkvCfg<D>;
  CUtensorMap tk, tv, tq, tdo;
  const int BH = a.B * a.H, BHk = a.B * a.Hkv;
  if (!make_tile_map(&tk, a.k, a.dtype, D, a.kv_len, a.Sk, BHk, 128) ||
      !make_tile_map(&tv, a.v, a.dtype, D, a.kv_len, a.Sk, BHk, 128) ||
      !make_tile_map(&tq, a.q, a.dtype, D, a.Sq, a.Sq, BH, 128) ||
      !make_tile_map(&tdo, a.dout, a.dtype, D, a.Sq, a.Sq, BH, 128))
    return cudaErrorInvalidValue;
  if (a.ds_buf != nullptr && (reinterpret_cast<uintptr_t>(a.ds_buf) & 15)) return cudaErrorInvalidValue;
  const int parts = a.dkv_part != nullptr ? a.head_parts : 1;
  if (parts < 1 || (a.H / a.Hkv) % parts != 0 || (reinterpret_cast<uintptr_t>(a.dkv_part) & 15))
    return cudaErrorInvalidValue;
  auto kern = bwd_dkv_sm100_kernel<T, D>;
  cudaError_t e = ensure_smem(kern, Cfg::kSmem);
  if (e != cudaSuccess) return e;
  const int n_kt = (a.Sk + 127) / 128;
  kern<<<n_kt * BHk * parts, EwDkv::kThreads, Cfg::kSmem, a.stream>>>(
      tk, tv, tq, tdo, reinterpret_cast<uint8_t*>(a.ds_buf), a.dkv_part, parts, a.lse, a.delta, (T*)a.dk, (T*)a.dv,
      a.H, a.Hkv, a.Sq, a.Sk, a.kv_len, a.causal, a.sm_scale, a.sm_scale * kLog2e, n_kt);
  e = cudaGetLastError();
  if (e != cudaSuccess || parts == 1) return e;
  const long n4 = (long)BHk * a.Sk * D / 4;
  const long blocks = std::min((2 * n4 + 255) / 256, (long)sm_count() * 8);
  dkv_part_reduce_kernel<T><<<(unsigned)blocks, 256, 0, a.stream>>>(a.dkv_part, (T*)a.dk, (T*)a.dv, n4, parts);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_dq_t(const BwdArgs& a) {
  using Cfg = DqCfg<D>;
  CUtensorMap tq, tdo, tk, tv;
  const int BH = a.B * a.H, BHk = a.B * a.Hkv;
  if (!make_tile_map(&tq, a.q, a.dtype, D, a.Sq, a.Sq, BH, 128) ||
      !make_tile_map(&tdo, a.dout, a.dtype, D, a.Sq, a.Sq, BH, 128) ||
      !make_tile_map(&tk, a.k, a.dtype, D, a.kv_len, a.Sk, BHk, 128) ||
      !make_tile_map(&tv, a.v, a.dtype, D, a.kv_len, a.Sk, BHk, 128))
    return cudaErrorInvalidValue;
  auto kern = bwd_dq_sm100_kernel<T, D>;
  cudaError_t e = ensure_smem(kern, Cfg::kSmem);
  if (e != cudaSuccess) return e;
  const int n_qt = (a.Sq + 127) / 128;
  kern<<<n_qt * BH, EwDq::kThreads, Cfg::kSmem, a.stream>>>(tq, tdo, tk, tv, a.lse, a.delta, (T*)a.dq, a.H, a.Hkv,
                                                      a.Sq, a.kv_len, a.causal, a.sm_scale, a.sm_scale * kLog2e,
                                                      n_qt);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_dq_gemm_t(const BwdArgs& a) {
  using Cfg = DqGemmCfg<D>;
  const int BH = a.B * a.H, BHk = a.B * a.Hkv;
  const int n_qt = (a.Sq + 127) / 128;
  const long tiles = (long)BH * ds_tiles_per_plane(n_qt, a.kv_len, a.causal);
  if (tiles <= 0 || tiles > INT_MAX) return cudaErrorInvalidValue;
  CUtensorMap tk;
  if ((reinterpret_cast<uintptr_t>(a.ds_buf) & 15) || !make_tile_map(&tk, a.k, a.dtype, D, a.kv_len, a.Sk, BHk, 128))
    return cudaErrorInvalidValue;
  auto kern = bwd_dq_gemm_sm100_kernel<T, D>;
  cudaError_t e = ensure_smem(kern, Cfg::kSmem);
  if (e != cudaSuccess) return e;
  const int n_items = n_qt * BH;
  const int grid = std::min(n_items, a.dq_ctas > 0 ? a.dq_ctas : sm_count());
  kern<<<grid, Cfg::kThreads, Cfg::kSmem, a.stream>>>(reinterpret_cast<const uint8_t*>(a.ds_buf), tk, (T*)a.dq, a.H, a.Hkv, a.Sq, a.kv_len, a.causal,
                                                    a.sm_scale, n_qt, n_items);
  return cudaGetLastError();
}

}  // namespace

int bwd_dkv_head_parts(int B, int H, int Hkv, int Sk) {
  if (B <= 0 || H <= 0 || Hkv <= 0 || H % Hkv != 0 || Sk <= 0) return 1;
  const int G = H / Hkv;
  const long ctas = (long)((Sk + 127) / 128) * B * Hkv;
  int parts = 1;
  while (G % (parts * 2) == 0 && ctas * parts < sm_count()) parts *= 2;
  return parts;
}

size_t bwd_dkv_part_bytes(int B, int Hkv, int Sk, int D, int parts) {
  return parts > 1 ? (size_t)2 * parts * B * Hkv * Sk * D * sizeof(float) : 0;
}

size_t bwd_ds_spill_bytes(int B, int H, int Sq, int kv_len, int causal) {
  return (size_t)B * H * ds_tiles_per_plane((Sq + 127) / 128, kv_len, causal) * (128 * 128 * 2);
}

cudaError_t launch_bwd_dq_gemm_sm100(const BwdArgs& a) {
  if (a.dtype == PF_BF16)
    return a.D == 128 ? launch_dq_gemm_t<__nv_bfloat16, 128>(a) : launch_dq_gemm_t<__nv_bfloat16, 64>(a);
  return a.D == 128 ? launch_dq_gemm_t<__half, 128>(a) : launch_dq_gemm_t<__half, 64>(a);
}

bool bwd_sm100_supported(int dtype, int D) { return fwd_sm100_supported(dtype, D); }

cudaError_t launch_bwd_dkv_sm100(const BwdArgs& a) {
  if (a.dtype == PF_BF16) return a.D == 128 ? launch_dkv_t<__nv_bfloat16, 128>(a) : launch_dkv_t<__nv_bfloat16, 64>(a);
  return a.D == 128 ? launch_dkv_t<__half, 128>(a) : launch_dkv_t<__half, 64>(a);
}

cudaError_t launch_bwd_dq_sm100(const BwdArgs& a) {
  if (a.dtype == PF_BF16) return a.D == 128 ? launch_dq_t<__nv_bfloat16, 128>(a) : launch_dq_t<__nv_bfloat16, 64>(a);
  return a.D == 128 ? launch_dq_t<__half, 128>(a) : launch_dq_t<__half, 64>(a);
}

}  // namespace pf
