// attn_bwd_sm100.cu -- tensor-core (tcgen05 / TMEM / TMA) backward for bf16
// and f16 inputs, head_dim 64 or 128.
//
// Two kernels with transposed loops, as the reference's backward
// (flash_attention.py:276-351), each recomputing P from the saved
// log-sum-exp:  p = exp(s*scale - lse),  ds = p (dp - delta):
//
//   dK/dV kernel: CTA = (batch, kv head, 128-key tile).  Loops over every q
//     head of the GQA group and every 128-row query tile that can see the
//     keys, so the group-sum of flash_attention.py:433-436 happens in TMEM:
//        S^T  = K Q^T         dP^T = V dO^T            (M = 128 keys, N = 128)
//        dV  += P^T dO        dK  += dS^T Q             (A = P^T, dS^T from TMEM)
//   dQ kernel:    CTA = (batch, head, 128-row query tile), loops over 128-key tiles:
//        S    = Q K^T         dP   = dO V^T             (M = 128 rows, N = 128)
//        dQ  += dS K                                     (A = dS from TMEM)
//
// All MMAs are 128 x 128 tiles: at N = 128 a shared-memory operand pair
// streams at the rate the tensor core needs for full throughput, where N = 64
// tiles reach only ~2/3 of it.  TMEM (512 columns) holds S and dP (128 each)
// and the accumulators (dV, dK: 2 x D; dQ: D, with S double-buffered).  The
// elementwise warps work in two phases per tile -- P (exp, needs S) then dS
// (needs dP) -- with P kept in f32 registers between them, and the MMA issue
// order interleaves the two kernels' GEMMs so that each phase overlaps tensor
// work of a neighbouring tile.
#include <type_traits>
#include "common.cuh"
#include "kernels.h"
#include "sm100_util.cuh"

namespace pf {
namespace {

constexpr int kThreads = 384;  // warp 0 TMA, warp 1 MMA, warps 4-11 elementwise

struct BwdBars {
  uint64_t fixed;                  // the CTA's resident tiles
  uint64_t full[4], empty[4];      // streamed stages (dK/dV: Q+dO pairs; dQ: K ring)
  uint64_t vfull[2], vempty[2];    // dQ: V ring
  uint64_t s_full[2], dp_full;     // S / dP in TMEM
  uint64_t p_ready, ds_ready;      // P / dS written back to TMEM
  uint64_t done;                   // accumulators final
  uint32_t tmem_base;
};

// dK/dV: K, V resident; NS stages of (Q, dO) 128-row tiles plus their column statistics.
template <int D>
struct DkvCfg {
  static constexpr int kNS = D == 128 ? 2 : 4;
  static constexpr int kBoxes = D / 64;
  static constexpr int kTile = 128 * D * 2;
  static constexpr int kFixedOff = 0;
  static constexpr int kStreamOff = 2 * kTile;
  static constexpr int kStatOff = kStreamOff + kNS * 2 * kTile;  // [kNS][128] float2 (-lse*log2e, -delta)
  static constexpr int kBarOff = kStatOff + kNS * 128 * 8;
  static constexpr int kSmem = kBarOff + 256 + 1024;
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

// Elementwise steps shared by both kernels.  A thread owns one TMEM lane and
// 64 columns of S / dP (two 32-column chunks at c0 and c0 + 32).
//
// P phase:  p = exp2(s * scale*log2e + nl2(c)) (0 where not visible), kept in
//   f32 registers and written back packed to 16-bit pairs over the first 16
//   columns of each chunk of the S buffer (the A operand of dV += P^T dO).
// dS phase: ds = p * (dp + nd(c)), packed the same way over the dP buffer.
//
// nl2(h, c) is -lse*log2(e) and nd(h, c) is -delta for column c of chunk h (or
// for the thread's row).  `FULL` (chosen per chunk by a warp-uniform test)
// drops the per-element visibility selects.
template <int FMT, bool FULL, typename Vis, typename NL2>
__device__ __forceinline__ void p_chunk(const uint32_t (&rs)[32], float (&p)[32], uint32_t (&pk)[16], float2 sc2,
                                        Vis visible, NL2 nl2) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = 2 * i;
    const float2 x = fma2(make_float2(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1])), sc2,
                          nl2(c));
    float2 e = make_float2(fast_exp2(x.x), fast_exp2(x.y));
    if (!FULL) {
      e.x = visible(c) ? e.x : 0.f;
      e.y = visible(c + 1) ? e.y : 0.f;
    }
    p[c] = e.x;
    p[c + 1] = e.y;
    pk[i] = FMT == 1 ? pack_bf16x2(e.x, e.y) : pack_f16x2(e.x, e.y);
  }
}

template <int FMT, typename Vis, typename Full, typename NL2>
__device__ __forceinline__ void p_phase(uint32_t s_addr, float scale_log2, Full full, Vis visible, NL2 nl2,
                                        float (&p)[2][32]) {
  uint32_t rs[2][32];
  tmem_ld32(s_addr, rs[0]);
  tmem_ld32(s_addr + 32, rs[1]);
  tmem_wait_ld();
  const float2 sc2 = make_float2(scale_log2, scale_log2);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t pk[16];
    auto vis_h = [&](int c) { return visible(h, c); };
    auto nl2_h = [&](int c) { return nl2(h, c); };
    if (full(h)) p_chunk<FMT, true>(rs[h], p[h], pk, sc2, vis_h, nl2_h);
    else p_chunk<FMT, false>(rs[h], p[h], pk, sc2, vis_h, nl2_h);
    tmem_st16(s_addr + 32 * h, pk);
  }
}

template <int FMT, typename ND>
__device__ __forceinline__ void ds_phase(uint32_t dp_addr, ND nd, const float (&p)[2][32]) {
  uint32_t rd[2][32];
  tmem_ld32(dp_addr, rd[0]);
  tmem_ld32(dp_addr + 32, rd[1]);
  tmem_wait_ld();
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int c = 2 * i;
      const float2 t = add2(make_float2(__uint_as_float(rd[h][c]), __uint_as_float(rd[h][c + 1])), nd(h, c));
      const float2 ds = mul2(make_float2(p[h][c], p[h][c + 1]), t);
      pk[i] = FMT == 1 ? pack_bf16x2(ds.x, ds.y) : pack_f16x2(ds.x, ds.y);
    }
    tmem_st16(dp_addr + 32 * h, pk);
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

// ============================================================================
// dK / dV
// ============================================================================
template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
bwd_dkv_sm100_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                     const float* __restrict__ lse, const float* __restrict__ delta,
                     T* __restrict__ dk, T* __restrict__ dv, int H, int Hkv, int Sq, int Sk,
                     int kv_len, int causal, float sm_scale, float scale_log2, int n_kt) {
  using Cfg = DkvCfg<D>;
  constexpr int NS = Cfg::kNS;
  constexpr int FMT = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t idesc_s = make_idesc_f16(FMT, 128, 128, 0, 0);
  constexpr uint32_t idesc_acc = make_idesc_f16(FMT, 128, D, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  BwdBars* bars = reinterpret_cast<BwdBars*>(smem + Cfg::kBarOff);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  // Causal: heaviest (first) key tiles of every head first.
  const int BHk = gridDim.x / n_kt;
  const int kt = blockIdx.x / BHk;
  const int bhk = blockIdx.x % BHk;
  const int b = bhk / Hkv, hk = bhk % Hkv;
  const int G = H / Hkv;
  const int k0 = kt * 128;
  const int nq = (Sq + 127) / 128;
  int i0 = causal ? k0 / 128 : 0;
  if (k0 >= kv_len) i0 = nq;  // no live key in this tile
  const int nqi = max(0, nq - i0);
  const int n_it = G * nqi;

  if (threadIdx.x == 0) {
    mbar_init(&bars->fixed, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bars->full[s], 1 + 32);  // TMA tx arrive + the producer warp's 32 stat writers
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->s_full[0], 1);
    mbar_init(&bars->dp_full, 1);
    mbar_init(&bars->p_ready, 256);
    mbar_init(&bars->ds_ready, 256);
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
  float2* stats = reinterpret_cast<float2*>(smem + Cfg::kStatOff);

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
      for (int it = 0; it < n_it; ++it) {
        const int s = it % NS;
        if (it >= NS && !mbar_wait(&bars->empty[s], ((it / NS) - 1) & 1)) break;
        const int g = it / nqi, qi = i0 + it % nqi;
        const int plane = b * H + hk * G + g;
        if (lane == 0) {
          uint8_t* qdst = smem + Cfg::kStreamOff + s * 2 * Cfg::kTile;
          mbar_expect_tx(&bars->full[s], 2 * Cfg::kTile);
          for (int c = 0; c < Cfg::kBoxes; ++c) {
            tma_load_3d(qdst + c * 128 * 128, &tm_q, &bars->full[s], c * 64, qi * 128, plane);
            tma_load_3d(qdst + Cfg::kTile + c * 128 * 128, &tm_do, &bars->full[s], c * 64, qi * 128, plane);
          }
        }
        const long srow = (long)plane * Sq;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = lane + 32 * u, qp = qi * 128 + c;
          stats[s * 128 + c] = qp < Sq ? make_float2(-lse[srow + qp] * kLog2e, -delta[srow + qp])
                                       : make_float2(0.f, 0.f);
        }
        mbar_arrive(&bars->full[s]);
      }
    }
  } else if (warp == 1) {
    // Tensor-core order per iteration:  dV(it) [P ready]  S(it+1)  dK(it) [dS ready]  dP(it+1).
    // The P phase of it+1 overlaps dK(it) and dP(it+1); the dS phase of it
    // overlaps dV(it) and S(it+1).  In-order execution makes S(it+1) overwrite
    // P(it) only after dV(it) read it, and dP(it+1) overwrite dS(it) after dK(it).
    if (lane == 0 && n_it > 0) {
      bool ok = mbar_wait(&bars->fixed, 0);
      tc_fence_after();
      const uint32_t k_addr = sbase + Cfg::kFixedOff, v_addr = k_addr + Cfg::kTile;
      auto stage = [&](int it) { return sbase + Cfg::kStreamOff + (it % NS) * 2 * Cfg::kTile; };
      auto issue_s = [&](int it) {
        const uint32_t q_addr = stage(it);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(tmem + Cfg::kS, desc_k<128>(k_addr, kk), desc_k<128>(q_addr, kk), idesc_s, kk > 0);
        umma_commit(&bars->s_full[0]);
      };
      auto issue_dp = [&](int it) {
        const uint32_t do_addr = stage(it) + Cfg::kTile;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(tmem + Cfg::kDP, desc_k<128>(v_addr, kk), desc_k<128>(do_addr, kk), idesc_s, kk > 0);
        umma_commit(&bars->dp_full);
      };
      if (ok) ok = mbar_wait_spin(&bars->full[0], 0);
      if (ok) {
        tc_fence_after();
        issue_s(0);
        issue_dp(0);
      }
      for (int it = 0; ok && it < n_it; ++it) {
        const uint32_t q_addr = stage(it), do_addr = q_addr + Cfg::kTile;
        ok = mbar_wait_spin(&bars->p_ready, it & 1);
        if (!ok) break;
        trace(1, it);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts(tmem + Cfg::kDV, tmem + Cfg::kS + split_packed_col(kk), desc_mn<128>(do_addr, kk), idesc_acc,
                  (it > 0 || kk > 0));
        if (it + 1 < n_it) {
          ok = mbar_wait_spin(&bars->full[(it + 1) % NS], ((it + 1) / NS) & 1);
          if (!ok) break;
          tc_fence_after();
          issue_s(it + 1);
        }
        trace(2, it);
        ok = mbar_wait_spin(&bars->ds_ready, it & 1);
        if (!ok) break;
        trace(3, it);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts(tmem + Cfg::kDK, tmem + Cfg::kDP + split_packed_col(kk), desc_mn<128>(q_addr, kk), idesc_acc,
                  (it > 0 || kk > 0));
        umma_commit(&bars->empty[it % NS]);
        if (it + 1 < n_it) issue_dp(it + 1);
        trace(4, it);
      }
      umma_commit(&bars->done);
    }
  } else if (warp >= 4) {
    const int w = (warp - 4) / 4;  // query columns [64w, 64w + 64) of each tile
    const int quad = warp % 4;
    const int row = quad * 32 + lane;  // key row within the tile
    const int kpos = k0 + row;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const bool key_ok = kpos < kv_len;
    bool ok = true;
    float p[2][32];
    for (int it = 0; ok && it < n_it; ++it) {
      const int st = it % NS;
      const int qc = (i0 + it % nqi) * 128 + 64 * w;  // first query column of this thread's half
      // The stage's statistics were written by the producer warp before its
      // arrive on full[st]; the stage is not refilled before dK(it) retires.
      if (!mbar_wait_spin(&bars->s_full[0], it & 1) || !mbar_wait(&bars->full[st], (it / NS) & 1)) {
        ok = false;
        break;
      }
      if (threadIdx.x == 128 || threadIdx.x == 256) trace(8 + 2 * w, it);
      tc_fence_after();
      const float4* st4 = reinterpret_cast<const float4*>(stats + st * 128 + 64 * w);
      p_phase<FMT>(
          lane_base + Cfg::kS + 64 * w, scale_log2,
          [&](int h) {
            const int q0 = qc + 32 * h;
            return (k0 + 127 < kv_len) && (q0 + 32 <= Sq) && (!causal || q0 >= k0 + 127);
          },
          [&](int h, int c) {
            const int qp = qc + 32 * h + c;
            return key_ok && qp < Sq && (!causal || qp >= kpos);
          },
          [&](int h, int c) {
            const float4 v4 = st4[16 * h + c / 2];
            return make_float2(v4.x, v4.z);
          },
          p);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_ready);
      if (threadIdx.x == 128 || threadIdx.x == 256) trace(9 + 2 * w, it);
      if (!mbar_wait_spin(&bars->dp_full, it & 1)) { ok = false; break; }
      tc_fence_after();
      ds_phase<FMT>(lane_base + Cfg::kDP + 64 * w,
                    [&](int h, int c) {
                      const float4 v4 = st4[16 * h + c / 2];
                      return make_float2(v4.y, v4.w);
                    },
                    p);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->ds_ready);
      if (threadIdx.x == 128 || threadIdx.x == 256) trace(10 + 2 * w, it);
    }
    // Epilogue: warpgroup 0 writes dV, warpgroup 1 writes dK (scaled).
    const bool have = n_it > 0 && ok && mbar_wait(&bars->done, 0);
    if (n_it > 0) tc_fence_after();
    const bool write = kpos < Sk;
    const long orow = ((long)(b * Hkv + hk) * Sk + kpos) * D;
    if (w == 0)
      store_acc_row<T, FMT>(lane_base + Cfg::kDV, dv + orow, D, 1.f, !have, write);
    else
      store_acc_row<T, FMT>(lane_base + Cfg::kDK, dk + orow, D, sm_scale, !have, write);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================
// dQ
// ============================================================================
template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
bwd_dq_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                    const float* __restrict__ lse, const float* __restrict__ delta, T* __restrict__ dq,
                    int H, int Hkv, int Sq, int kv_len, int causal, float sm_scale, float scale_log2,
                    int n_qt) {
  using Cfg = DqCfg<D>;
  constexpr int NK = Cfg::kNK, NV = Cfg::kNV;
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
    mbar_init(&bars->ds_ready, 256);
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
      for (int it = 0; it < n_it; ++it) {
        const int sk = it % NK, sv = it % NV;
        if (it >= NK && !mbar_wait(&bars->empty[sk], ((it / NK) - 1) & 1)) break;
        mbar_expect_tx(&bars->full[sk], Cfg::kTile);
        for (int c = 0; c < Cfg::kBoxes; ++c)
          tma_load_3d(smem + Cfg::kKOff + sk * Cfg::kTile + c * 128 * 128, &tm_k, &bars->full[sk], c * 64,
                      it * 128, kv_plane);
        if (it >= NV && !mbar_wait(&bars->vempty[sv], ((it / NV) - 1) & 1)) break;
        mbar_expect_tx(&bars->vfull[sv], Cfg::kTile);
        for (int c = 0; c < Cfg::kBoxes; ++c)
          tma_load_3d(smem + Cfg::kVOff + sv * Cfg::kTile + c * 128 * 128, &tm_v, &bars->vfull[sv], c * 64,
                      it * 128, kv_plane);
      }
    }
  } else if (warp == 1) {
    // Tensor-core order per iteration:  S(it+1)  dQ(it) [dS ready]  dP(it+1).
    // S is double-buffered, so S(it+1) runs while the elementwise warps still
    // work on tile it; dP(it+1) overwrites dS(it) only after dQ(it) read it.
    if (lane == 0 && n_it > 0) {
      bool ok = mbar_wait(&bars->fixed, 0);
      tc_fence_after();
      const uint32_t q_addr = sbase + Cfg::kFixedOff, do_addr = q_addr + Cfg::kTile;
      auto k_tile = [&](int it) { return sbase + Cfg::kKOff + (it % NK) * Cfg::kTile; };
      auto issue_s = [&](int it) -> bool {
        if (!mbar_wait_spin(&bars->full[it % NK], (it / NK) & 1)) return false;
        tc_fence_after();
        const uint32_t k_addr = k_tile(it);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(tmem + Cfg::kS + 128 * (it & 1), desc_k<128>(q_addr, kk), desc_k<128>(k_addr, kk), idesc_s,
                  kk > 0);
        umma_commit(&bars->s_full[it & 1]);
        return true;
      };
      auto issue_dp = [&](int it) -> bool {
        if (!mbar_wait_spin(&bars->vfull[it % NV], (it / NV) & 1)) return false;
        tc_fence_after();
        const uint32_t v_addr = sbase + Cfg::kVOff + (it % NV) * Cfg::kTile;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(tmem + Cfg::kDP, desc_k<128>(do_addr, kk), desc_k<128>(v_addr, kk), idesc_s, kk > 0);
        umma_commit(&bars->vempty[it % NV]);
        umma_commit(&bars->dp_full);
        return true;
      };
      if (ok) ok = issue_s(0) && issue_dp(0);
      for (int it = 0; ok && it < n_it; ++it) {
        if (it + 1 < n_it && !(ok = issue_s(it + 1))) break;
        trace(2, it);
        ok = mbar_wait_spin(&bars->ds_ready, it & 1);
        if (!ok) break;
        trace(3, it);
        tc_fence_after();
        const uint32_t k_addr = k_tile(it);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts(tmem + Cfg::kDQ, tmem + Cfg::kDP + split_packed_col(kk), desc_mn<128>(k_addr, kk), idesc_acc,
                  (it > 0 || kk > 0));
        umma_commit(&bars->empty[it % NK]);
        if (it + 1 < n_it && !(ok = issue_dp(it + 1))) break;
        trace(4, it);
      }
      umma_commit(&bars->done);
    }
  } else if (warp >= 4) {
    const int w = (warp - 4) / 4;  // key columns [64w, 64w + 64) of each tile
    const int quad = warp % 4;
    const int row = quad * 32 + lane;  // query row within the tile
    const int qpos = q0 + row;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const long srow = (long)bh * Sq + qpos;
    const float nl2 = qpos < Sq ? -lse[srow] * kLog2e : 0.f;
    const float nd = qpos < Sq ? -delta[srow] : 0.f;
    bool ok = true;
    float p[2][32];
    for (int it = 0; it < n_it; ++it) {
      if (!mbar_wait_spin(&bars->s_full[it & 1], (it >> 1) & 1)) { ok = false; break; }
      if (threadIdx.x == 128 || threadIdx.x == 256) trace(8 + 2 * w, it);
      tc_fence_after();
      const int kc = it * 128 + 64 * w;  // first key column of this thread's half
      p_phase<FMT>(
          lane_base + Cfg::kS + 128 * (it & 1) + 64 * w, scale_log2,
          [&](int hh) { const int kb = kc + 32 * hh; return (kb + 32 <= kv_len) && (!causal || kb + 31 <= q0); },
          [&](int hh, int c) {
            const int kp = kc + 32 * hh + c;
            return kp < kv_len && (!causal || kp <= qpos);
          },
          [&](int, int) { return make_float2(nl2, nl2); }, p);
      if (threadIdx.x == 128 || threadIdx.x == 256) trace(9 + 2 * w, it);
      if (!mbar_wait_spin(&bars->dp_full, it & 1)) { ok = false; break; }
      tc_fence_after();
      ds_phase<FMT>(lane_base + Cfg::kDP + 64 * w, [&](int, int) { return make_float2(nd, nd); }, p);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->ds_ready);
      if (threadIdx.x == 128 || threadIdx.x == 256) trace(10 + 2 * w, it);
    }
    const bool have = n_it > 0 && ok && mbar_wait(&bars->done, 0);
    if (n_it > 0) tc_fence_after();
    // Each warpgroup writes half of the D columns of its rows.
    store_acc_row<T, FMT>(lane_base + Cfg::kDQ + w * (D / 2), dq + srow * D + w * (D / 2), D / 2, sm_scale,
                          !have, qpos < Sq);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
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
  auto kern = bwd_dkv_sm100_kernel<T, D>;
  cudaError_t e = ensure_smem(kern, Cfg::kSmem);
  if (e != cudaSuccess) return e;
  const int n_kt = (a.Sk + 127) / 128;
  kern<<<n_kt * BHk, kThreads, Cfg::kSmem, a.stream>>>(tk, tv, tq, tdo, a.lse, a.delta, (T*)a.dk, (T*)a.dv, a.H,
                                                       a.Hkv, a.Sq, a.Sk, a.kv_len, a.causal, a.sm_scale,
                                                       a.sm_scale * kLog2e, n_kt);
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
  kern<<<n_qt * BH, kThreads, Cfg::kSmem, a.stream>>>(tq, tdo, tk, tv, a.lse, a.delta, (T*)a.dq, a.H, a.Hkv,
                                                      a.Sq, a.kv_len, a.causal, a.sm_scale, a.sm_scale * kLog2e,
                                                      n_qt);
  return cudaGetLastError();
}

}  // namespace

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
