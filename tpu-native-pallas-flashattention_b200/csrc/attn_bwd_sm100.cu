// attn_bwd_sm100.cu -- tensor-core (tcgen05 / TMEM / TMA) backward for bf16
// and f16 inputs, head_dim 64 or 128.
//
// Two kernels with transposed loops, as the reference's backward
// (flash_attention.py:276-351), each recomputing P from the saved
// log-sum-exp:  p = exp(s*scale - lse),  ds = p (dp - delta):
//
//   dK/dV kernel: CTA = (batch, kv head, 128-key tile).  Loops over every q
//     head of the GQA group and every 64-row query tile that can see the keys,
//     so the group-sum of flash_attention.py:433-436 happens in TMEM:
//        S^T  = K Q^T         dP^T = V dO^T            (M = 128 keys, N = 64)
//        dV  += P^T dO        dK  += dS^T Q             (A = P^T, dS^T from TMEM)
//   dQ kernel:    CTA = (batch, head, 128-row query tile), loops over 64-key tiles:
//        S    = Q K^T         dP   = dO V^T             (M = 128 rows, N = 64)
//        dQ  += dS K                                     (A = dS from TMEM)
//
// S and dP are double-buffered in TMEM (2 x 64 columns each) so the MMA warp
// issues the next tile's S/dP while two elementwise warpgroups (each owning
// 32 of the 64 columns) turn the current tile into P and dS, packed as 16-bit
// pairs over their own input columns.  TMEM: S0 S1 dP0 dP1 (256 columns) +
// accumulators (2 x D for dK/dV, D for dQ).
#include <type_traits>
#include "common.cuh"
#include "kernels.h"
#include "sm100_util.cuh"

namespace pf {
namespace {

constexpr int kThreads = 384;  // warp 0 TMA, warp 1 MMA, warps 4-11 elementwise
constexpr int kNS = 4;         // stages of the streamed operand pair

struct BwdBars {
  uint64_t fixed;                    // the CTA's resident tiles
  uint64_t full[kNS], empty[kNS];    // streamed stages
  uint64_t s_full[2], p_ready[2];    // TMEM S/dP buffers
  uint64_t done;                     // accumulators final
  uint32_t tmem_base;
};

template <int D>
struct BwdCfg {
  static constexpr int kBoxes = D / 64;
  static constexpr int kFixedTile = 128 * D * 2;  // 128-row resident tile
  static constexpr int kStreamTile = 64 * D * 2;  // 64-row streamed tile
  static constexpr int kFixedOff = 0;             // two resident tiles
  static constexpr int kStreamOff = 2 * kFixedTile;
  static constexpr int kStatOff = kStreamOff + kNS * 2 * kStreamTile;  // [kNS][64] float2 (-lse2, -delta)
  static constexpr int kBarOff = kStatOff + kNS * 64 * 8;
  static constexpr int kSmem = kBarOff + 256 + 1024;
  static constexpr uint32_t kS = 0, kDP = 128, kAcc = 256;
  static constexpr uint32_t kTmemCols = 512;
};

// Elementwise step shared by both kernels.  Thread owns TMEM lane `row`; its
// 32 columns [32w, 32w + 32) of S/dP buffer b become P and dS, packed to
// 16-bit pairs over the first 16 of those columns.  `full` (warp-uniform)
// means every column is visible; otherwise visible(c) decides.  nl2(c) is
// -lse*log2(e) and nd(c) is -delta for column c (or the thread's row).
template <int FMT, typename Vis, typename NL2, typename ND>
__device__ __forceinline__ void p_ds_step(uint32_t s_addr, uint32_t dp_addr, float scale_log2, bool full,
                                          Vis visible, NL2 nl2, ND nd) {
  uint32_t rs[32], rd[32];
  tmem_ld32(s_addr, rs);
  tmem_ld32(dp_addr, rd);
  tmem_wait_ld();
  uint32_t pp[16], pd[16];
  const float2 sc2 = make_float2(scale_log2, scale_log2);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = 2 * i;
    const float2 x = fma2(make_float2(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1])), sc2,
                          make_float2(nl2(c), nl2(c + 1)));
    float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
    if (!full) {
      p.x = visible(c) ? p.x : 0.f;
      p.y = visible(c + 1) ? p.y : 0.f;
    }
    const float2 t = add2(make_float2(__uint_as_float(rd[c]), __uint_as_float(rd[c + 1])),
                          make_float2(nd(c), nd(c + 1)));
    const float2 ds = mul2(p, t);
    pp[i] = FMT == 1 ? pack_bf16x2(p.x, p.y) : pack_f16x2(p.x, p.y);
    pd[i] = FMT == 1 ? pack_bf16x2(ds.x, ds.y) : pack_f16x2(ds.x, ds.y);
  }
  tmem_st16(s_addr, pp);
  tmem_st16(dp_addr, pd);
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
  using Cfg = BwdCfg<D>;
  constexpr int FMT = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t idesc_s = make_idesc_f16(FMT, 128, 64, 0, 0);
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
  const int nq = (Sq + 63) / 64;
  int i0 = causal ? k0 / 64 : 0;
  if (k0 >= kv_len) i0 = nq;  // no live key in this tile
  const int nqi = max(0, nq - i0);
  const int n_it = G * nqi;

  if (threadIdx.x == 0) {
    mbar_init(&bars->fixed, 1);
    for (int s = 0; s < kNS; ++s) {
      mbar_init(&bars->full[s], 1 + 32);  // TMA tx arrive + the producer warp's 32 stat writes
      mbar_init(&bars->empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_ready[i], 256);
    }
    mbar_init(&bars->done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  float2* stats = reinterpret_cast<float2*>(smem + Cfg::kStatOff);

  if (warp == 0) {
    if (n_it > 0) {
      // All 32 lanes: lane 0 issues the TMA copies, every lane stages two of
      // the 64 (-lse*log2e, -delta) column statistics of the query tile.
      const int kv_plane = b * Hkv + hk;
      if (lane == 0) {
        mbar_expect_tx(&bars->fixed, 2 * Cfg::kFixedTile);
        for (int c = 0; c < Cfg::kBoxes; ++c) {
          tma_load_3d(smem + Cfg::kFixedOff + c * 128 * 128, &tm_k, &bars->fixed, c * 64, k0, kv_plane);
          tma_load_3d(smem + Cfg::kFixedOff + Cfg::kFixedTile + c * 128 * 128, &tm_v, &bars->fixed, c * 64, k0,
                      kv_plane);
        }
      }
      for (int it = 0; it < n_it; ++it) {
        const int s = it % kNS;
        if (it >= kNS && !mbar_wait(&bars->empty[s], ((it / kNS) - 1) & 1)) break;
        const int g = it / nqi, qi = i0 + it % nqi;
        const int plane = b * H + hk * G + g;
        if (lane == 0) {
          uint8_t* qdst = smem + Cfg::kStreamOff + s * 2 * Cfg::kStreamTile;
          mbar_expect_tx(&bars->full[s], 2 * Cfg::kStreamTile);
          for (int c = 0; c < Cfg::kBoxes; ++c) {
            tma_load_3d(qdst + c * 64 * 128, &tm_q, &bars->full[s], c * 64, qi * 64, plane);
            tma_load_3d(qdst + Cfg::kStreamTile + c * 64 * 128, &tm_do, &bars->full[s], c * 64, qi * 64, plane);
          }
        }
        const long srow = (long)plane * Sq;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int c = lane + 32 * u, qp = qi * 64 + c;
          stats[s * 64 + c] = qp < Sq ? make_float2(-lse[srow + qp] * kLog2e, -delta[srow + qp])
                                      : make_float2(0.f, 0.f);
        }
        mbar_arrive(&bars->full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_it > 0) {
      bool ok = mbar_wait(&bars->fixed, 0);
      tc_fence_after();
      const uint32_t k_addr = sbase + Cfg::kFixedOff, v_addr = k_addr + Cfg::kFixedTile;
      for (int it = 0; ok && it <= n_it; ++it) {
        if (it < n_it) {
          const int s = it % kNS, bf = it & 1;
          ok = mbar_wait(&bars->full[s], (it / kNS) & 1);
          if (!ok) break;
          trace(1, it);
          tc_fence_after();
          const uint32_t q_addr = sbase + Cfg::kStreamOff + s * 2 * Cfg::kStreamTile;
          const uint32_t do_addr = q_addr + Cfg::kStreamTile;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(tmem + Cfg::kS + bf * 64, desc_k<128>(k_addr, kk), desc_k<64>(q_addr, kk), idesc_s, kk > 0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(tmem + Cfg::kDP + bf * 64, desc_k<128>(v_addr, kk), desc_k<64>(do_addr, kk), idesc_s, kk > 0);
          umma_commit(&bars->s_full[bf]);
          trace(2, it);
        }
        if (it >= 1) {
          const int j = it - 1, s = j % kNS, bf = j & 1;
          ok = mbar_wait(&bars->p_ready[bf], (j >> 1) & 1);
          if (!ok) break;
          trace(3, j);
          tc_fence_after();
          const uint32_t q_addr = sbase + Cfg::kStreamOff + s * 2 * Cfg::kStreamTile;
          const uint32_t do_addr = q_addr + Cfg::kStreamTile;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ts(tmem + Cfg::kAcc, tmem + Cfg::kS + bf * 64 + split_packed_col(kk), desc_mn<64>(do_addr, kk),
                    idesc_acc, (j > 0 || kk > 0));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ts(tmem + Cfg::kAcc + D, tmem + Cfg::kDP + bf * 64 + split_packed_col(kk), desc_mn<64>(q_addr, kk),
                    idesc_acc, (j > 0 || kk > 0));
          umma_commit(&bars->empty[s]);
          trace(4, j);
        }
      }
      umma_commit(&bars->done);
    }
  } else if (warp >= 4) {
    const int w = (warp - 4) / 4;  // column half
    const int quad = warp % 4;
    const int row = quad * 32 + lane;  // key row within the tile
    const int kpos = k0 + row;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int bf = it & 1, st = it % kNS;
      const int qi = i0 + it % nqi;
      const int q0 = qi * 64 + 32 * w;  // first query column of this thread's half
      if (!mbar_wait(&bars->s_full[bf], (it >> 1) & 1)) { ok = false; break; }
      if (threadIdx.x == 128 || threadIdx.x == 256) trace(8 + 2 * w, it);
      tc_fence_after();
      // The producer warp wrote this stage's statistics before arriving on its
      // full barrier; acquire that barrier (already complete, and it cannot
      // advance before this warpgroup arrives on p_ready) and read them as
      // broadcast float4 loads.
      if (!mbar_wait(&bars->full[st], (it / kNS) & 1)) { ok = false; break; }
      float2 cs[32];
      const float4* src = reinterpret_cast<const float4*>(stats + st * 64 + 32 * w);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float4 v4 = src[c];
        cs[2 * c] = make_float2(v4.x, v4.y);
        cs[2 * c + 1] = make_float2(v4.z, v4.w);
      }
      const bool key_ok = kpos < kv_len;
      const bool full = (k0 + 127 < kv_len) && (q0 + 32 <= Sq) && (!causal || q0 >= k0 + 127);
      p_ds_step<FMT>(
          lane_base + Cfg::kS + bf * 64 + 32 * w, lane_base + Cfg::kDP + bf * 64 + 32 * w, scale_log2, full,
          [&](int c) { const int qp = q0 + c; return key_ok && qp < Sq && (!causal || qp >= kpos); },
          [&](int c) { return cs[c].x; }, [&](int c) { return cs[c].y; });
      tmem_wait_st();
      tc_fence_before();
      if (threadIdx.x == 128 || threadIdx.x == 256) trace(9 + 2 * w, it);
      mbar_arrive(&bars->p_ready[bf]);
    }
    // Epilogue: warpgroup 0 writes dV, warpgroup 1 writes dK (scaled).
    const bool have = n_it > 0 && ok && mbar_wait(&bars->done, 0);
    if (n_it > 0) tc_fence_after();
    const bool write = kpos < Sk;
    const long orow = ((long)(b * Hkv + hk) * Sk + kpos) * D;
    if (w == 0)
      store_acc_row<T, FMT>(lane_base + Cfg::kAcc, dv + orow, D, 1.f, !have, write);
    else
      store_acc_row<T, FMT>(lane_base + Cfg::kAcc + D, dk + orow, D, sm_scale, !have, write);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
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
  using Cfg = BwdCfg<D>;
  constexpr int FMT = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t idesc_s = make_idesc_f16(FMT, 128, 64, 0, 0);
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
  const int kvb = (kv_len + 63) / 64;
  const int q_last = min(q0 + 127, Sq - 1);
  const int n_it = causal ? min(kvb, q_last / 64 + 1) : kvb;

  if (threadIdx.x == 0) {
    mbar_init(&bars->fixed, 1);
    for (int s = 0; s < kNS; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_ready[i], 256);
    }
    mbar_init(&bars->done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0 && n_it > 0) {
      mbar_expect_tx(&bars->fixed, 2 * Cfg::kFixedTile);
      for (int c = 0; c < Cfg::kBoxes; ++c) {
        tma_load_3d(smem + Cfg::kFixedOff + c * 128 * 128, &tm_q, &bars->fixed, c * 64, q0, bh);
        tma_load_3d(smem + Cfg::kFixedOff + Cfg::kFixedTile + c * 128 * 128, &tm_do, &bars->fixed, c * 64, q0, bh);
      }
      const int kv_plane = b * Hkv + hk;
      for (int it = 0; it < n_it; ++it) {
        const int s = it % kNS;
        if (it >= kNS && !mbar_wait(&bars->empty[s], ((it / kNS) - 1) & 1)) break;
        uint8_t* kdst = smem + Cfg::kStreamOff + s * 2 * Cfg::kStreamTile;
        mbar_expect_tx(&bars->full[s], 2 * Cfg::kStreamTile);
        for (int c = 0; c < Cfg::kBoxes; ++c) {
          tma_load_3d(kdst + c * 64 * 128, &tm_k, &bars->full[s], c * 64, it * 64, kv_plane);
          tma_load_3d(kdst + Cfg::kStreamTile + c * 64 * 128, &tm_v, &bars->full[s], c * 64, it * 64, kv_plane);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_it > 0) {
      bool ok = mbar_wait(&bars->fixed, 0);
      tc_fence_after();
      const uint32_t q_addr = sbase + Cfg::kFixedOff, do_addr = q_addr + Cfg::kFixedTile;
      for (int it = 0; ok && it <= n_it; ++it) {
        if (it < n_it) {
          const int s = it % kNS, bf = it & 1;
          ok = mbar_wait(&bars->full[s], (it / kNS) & 1);
          if (!ok) break;
          tc_fence_after();
          const uint32_t k_addr = sbase + Cfg::kStreamOff + s * 2 * Cfg::kStreamTile;
          const uint32_t v_addr = k_addr + Cfg::kStreamTile;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(tmem + Cfg::kS + bf * 64, desc_k<128>(q_addr, kk), desc_k<64>(k_addr, kk), idesc_s, kk > 0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(tmem + Cfg::kDP + bf * 64, desc_k<128>(do_addr, kk), desc_k<64>(v_addr, kk), idesc_s, kk > 0);
          umma_commit(&bars->s_full[bf]);
        }
        if (it >= 1) {
          const int j = it - 1, s = j % kNS, bf = j & 1;
          ok = mbar_wait(&bars->p_ready[bf], (j >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
          const uint32_t k_addr = sbase + Cfg::kStreamOff + s * 2 * Cfg::kStreamTile;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ts(tmem + Cfg::kAcc, tmem + Cfg::kDP + bf * 64 + split_packed_col(kk), desc_mn<64>(k_addr, kk),
                    idesc_acc, (j > 0 || kk > 0));
          umma_commit(&bars->empty[s]);
        }
      }
      umma_commit(&bars->done);
    }
  } else if (warp >= 4) {
    const int w = (warp - 4) / 4;
    const int quad = warp % 4;
    const int row = quad * 32 + lane;  // query row within the tile
    const int qpos = q0 + row;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const long srow = (long)bh * Sq + qpos;
    const float nl2 = qpos < Sq ? -lse[srow] * kLog2e : 0.f;
    const float nd = qpos < Sq ? -delta[srow] : 0.f;
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int bf = it & 1;
      const int kb = it * 64 + 32 * w;  // first key column of this thread's half
      if (!mbar_wait(&bars->s_full[bf], (it >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      int vis = min(32, kv_len - kb);
      if (causal) vis = min(vis, qpos - kb + 1);
      const bool full = (kb + 32 <= kv_len) && (!causal || kb + 31 <= q0);
      p_ds_step<FMT>(lane_base + Cfg::kS + bf * 64 + 32 * w, lane_base + Cfg::kDP + bf * 64 + 32 * w, scale_log2,
                     full, [&](int c) { return c < vis; }, [&](int) { return nl2; }, [&](int) { return nd; });
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_ready[bf]);
    }
    const bool have = n_it > 0 && ok && mbar_wait(&bars->done, 0);
    if (n_it > 0) tc_fence_after();
    // Each warpgroup writes half of the D columns of its rows.
    store_acc_row<T, FMT>(lane_base + Cfg::kAcc + w * (D / 2), dq + srow * D + w * (D / 2), D / 2, sm_scale,
                          !have, qpos < Sq);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

template <typename T, int D>
cudaError_t launch_dkv_t(const BwdArgs& a) {
  using Cfg = BwdCfg<D>;
  CUtensorMap tk, tv, tq, tdo;
  const int BH = a.B * a.H, BHk = a.B * a.Hkv;
  if (!make_tile_map(&tk, a.k, a.dtype, D, a.kv_len, a.Sk, BHk, 128) ||
      !make_tile_map(&tv, a.v, a.dtype, D, a.kv_len, a.Sk, BHk, 128) ||
      !make_tile_map(&tq, a.q, a.dtype, D, a.Sq, a.Sq, BH, 64) ||
      !make_tile_map(&tdo, a.dout, a.dtype, D, a.Sq, a.Sq, BH, 64))
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
  using Cfg = BwdCfg<D>;
  CUtensorMap tq, tdo, tk, tv;
  const int BH = a.B * a.H, BHk = a.B * a.Hkv;
  if (!make_tile_map(&tq, a.q, a.dtype, D, a.Sq, a.Sq, BH, 128) ||
      !make_tile_map(&tdo, a.dout, a.dtype, D, a.Sq, a.Sq, BH, 128) ||
      !make_tile_map(&tk, a.k, a.dtype, D, a.kv_len, a.Sk, BHk, 64) ||
      !make_tile_map(&tv, a.v, a.dtype, D, a.kv_len, a.Sk, BHk, 64))
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
