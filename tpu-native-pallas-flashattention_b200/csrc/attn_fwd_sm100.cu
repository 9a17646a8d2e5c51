// attn_fwd_sm100.cu -- tensor-core (tcgen05 / TMEM / TMA) prefill forward for
// bf16 and f16 inputs, head_dim 64 or 128, with the saved log-sum-exp.
//
// A work item is two 128-row query tiles of one (batch, head); a persistent
// CTA per SM walks the items and, for each, streams the 128-key K/V tiles of the matching kv head (h / (H/Hkv), the GQA map of
// flash_attention.py:187-190) through a TMA-fed shared-memory ring:
//
//   warps 0-3   softmax for query tile 0 (TMEM lanes 0-127 = its rows)
//   warps 4-7   softmax for query tile 1
//   warp 8      TMA producer: Q0, Q1 once per item, then K_j / V_j per stage
//   warp 9      MMA issuer (one elected thread) and TMEM owner:
//                 S_w = Q_w K_j^T        (SS: both operands K-major in smem)
//                 O_w += P_w V_j          (TS: P from TMEM, V MN-major in smem)
//   warp 10     data certifier (folds the K/V "full" waits into the softmax
//               barrier phases the MMA issuer polls anyway)
//
// The two tiles ping-pong on the tensor core: while one warpgroup turns S
// into P, the MMA warp runs the other tile's GEMMs.  S, O live in TMEM
// (S0 | S1 | O0 | O1 = 512 columns at D = 128); P overwrites the first half of
// its S buffer as packed 16-bit pairs and feeds the PV MMA straight from TMEM.
// Softmax statistics are fp32 in the log2 domain; the running max used for
// P is only raised when the row max grows by more than 2^8, so O in TMEM is
// rescaled rarely (the final O / l is exact for any reference max).
//
// Masking follows the reference: keys >= kv_len are never loaded (the K/V
// tensor maps end at kv_len, TMA zero-fills past it), causal masks
// k_pos > q_pos with both sequences aligned at 0, kv blocks past kv_len or
// the causal diagonal are skipped (flash_attention.py:136-147), rows with no
// visible key write o = 0, lse = 0 (:150-159).
#include <cuda.h>
#include <algorithm>
#include <type_traits>
#include "common.cuh"
#include "kernels.h"
#include "sm100_util.cuh"

namespace pf {
namespace {

constexpr int kBM = 128;        // rows per query tile (= TMEM lanes)
constexpr int kBN = 128;        // keys per kv tile
constexpr int kThreads = 352;   // 11 warps: 0-7 softmax, 8 TMA, 9 MMA, 10 data certifier
constexpr float kRescaleThresh = 8.0f;  // log2 units

template <int D>
struct FwdCfg {
  static constexpr int kBoxes = D / 64;                  // 64-column (128 B) TMA boxes
  static constexpr int kTileBytes = kBM * D * 2;         // one 128 x D 16-bit tile
  // K and V rings are separate: a K tile is released as soon as both S
  // MMAs of its step have read it, so K runs further ahead than V.
  static constexpr int kKStages = D == 128 ? 3 : 4;
  static constexpr int kVStages = D == 128 ? 2 : 4;
  static constexpr int kQOff = 0;                        // Q0, Q1
  static constexpr int kKOff = 2 * kTileBytes;           // K stages
  static constexpr int kVOff = kKOff + kKStages * kTileBytes;
  static constexpr int kBarOff = kVOff + kVStages * kTileBytes;
  static constexpr int kSmem = kBarOff + 256 + 1024;     // + barriers + alignment slack
  // TMEM columns
  static constexpr uint32_t kS0 = 0, kS1 = 128, kO0 = 256, kO1 = 256 + D;
  static constexpr uint32_t kTmemCols = 512;
};

struct Bars {
  uint64_t q;
  uint64_t q_ready[2];  // RoPE: query tile w rotated in shared memory
  uint64_t k_full[4], v_full[4], k_empty[4], v_empty[4];
  uint64_t s_full[2], p_full[2], o_done[2];
  uint64_t p_half[2];   // P of the first 64 keys written (PV starts on it)
  uint64_t q_empty;     // an item's S MMAs have read the Q buffer (next item's Q may load)
  uint64_t o_free[2];   // an item's O has been read by the epilogue (next item's PV may start)
  uint64_t drained;     // follows every MMA of the CTA (committed after the issue loop)
  uint32_t tmem_base;
};
static_assert(sizeof(Bars) <= 256, "barrier block exceeds its shared-memory slot");

// Eight consecutive table entries [i, i + 8) as floats (16-byte aligned).
__device__ __forceinline__ void load8_table(const void* t, int dtype, long i, float (&o)[8]) {
  if (dtype == PF_F32) {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(t) + i);
    const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(t) + i + 4);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  } else {
    uint4 raw = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(t) + i);
    const uint16_t* h = reinterpret_cast<const uint16_t*>(&raw);
#pragma unroll
    for (int u = 0; u < 8; ++u)
      o[u] = dtype == PF_BF16 ? __bfloat162float(__ushort_as_bfloat16(h[u])) : __half2float(__ushort_as_half(h[u]));
  }
}

// Rotates one query row of a swizzled 128 x D tile in place:
// x*cos + rotate_half(x)*sin with table row `pos` (fused_rope.py:43-50, :75-78).
template <typename T, int D>
__device__ __forceinline__ void rope_row_in_smem(uint8_t* tile, int row, const void* cos_t, const void* sin_t,
                                                 int tbl_dtype, long pos) {
  constexpr int half = D / 2, NCH = half / 8;
  // The table loads of chunk ch+1 are issued before chunk ch is rotated, so
  // the row's eight (D = 128) global round trips overlap instead of queueing.
  float c0[2][8], s0[2][8], c1[2][8], s1[2][8];
  auto load = [&](int ch, int buf) {
    const int d0 = ch * 8, d1 = d0 + half;
    load8_table(cos_t, tbl_dtype, pos * D + d0, c0[buf]);
    load8_table(sin_t, tbl_dtype, pos * D + d0, s0[buf]);
    load8_table(cos_t, tbl_dtype, pos * D + d1, c1[buf]);
    load8_table(sin_t, tbl_dtype, pos * D + d1, s1[buf]);
  };
  load(0, 0);
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch) {
    if (ch + 1 < NCH) load(ch + 1, (ch + 1) & 1);
    const int buf = ch & 1;
    const int d0 = ch * 8, d1 = d0 + half;
    uint4* p0 = reinterpret_cast<uint4*>(tile + (d0 >> 6) * (kBM * 128) + row * 128 + ((((d0 & 63) >> 3) ^ (row & 7)) << 4));
    uint4* p1 = reinterpret_cast<uint4*>(tile + (d1 >> 6) * (kBM * 128) + row * 128 + ((((d1 & 63) >> 3) ^ (row & 7)) << 4));
    uint4 v0 = *p0, v1 = *p1;
    T* x0 = reinterpret_cast<T*>(&v0);
    T* x1 = reinterpret_cast<T*>(&v1);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float a = to_f(x0[u]), bb = to_f(x1[u]);
      x0[u] = from_f<T>(rope_lo(a, bb, c0[buf][u], s0[buf][u]));
      x1[u] = from_f<T>(rope_hi(a, bb, c1[buf][u], s1[buf][u]));
    }
    *p0 = v0;
    *p1 = v1;
  }
}

// One work item: two 128-row query tiles of one (batch, head).  Items are
// numbered heaviest first (the last query tiles, under causal), with the
// heads of one kv group adjacent so their shared K/V tiles meet in L2.
struct FwdItem {
  int b, h, bh, hk, q_start, kv_len, q_off, n_w[2], n_max;
};

__device__ __forceinline__ FwdItem fwd_item(int item, int B, int H, int Hkv, int Sq, int kv_len_max, int causal,
                                            int n_qtiles, const int32_t* kv_lens, const int32_t* q_offs) {
  FwdItem t;
  t.bh = item % (B * H);
  const int qt = n_qtiles - 1 - item / (B * H);
  t.b = t.bh / H;
  t.h = t.bh % H;
  t.hk = t.h / (H / Hkv);
  t.q_start = qt * 2 * kBM;
  // Keys of this sequence and the position of query row 0 (causal offset).
  t.kv_len = kv_lens ? max(0, min(kv_lens[t.b], kv_len_max)) : kv_len_max;
  t.q_off = q_offs ? q_offs[t.b] : 0;
  const int kvb = (t.kv_len + kBN - 1) / kBN;
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const int t0 = t.q_start + w * kBM;
    if (t0 >= Sq) {
      t.n_w[w] = 0;
    } else {
      const int last = min(t0 + kBM - 1, Sq - 1) + t.q_off;  // position of the tile's last query
      t.n_w[w] = causal ? (last < 0 ? 0 : min(kvb, last / kBN + 1)) : kvb;
    }
  }
  t.n_max = max(t.n_w[0], t.n_w[1]);
  return t;
}

// Persistent: one CTA per SM walks the items in serpentine rounds of
// gridDim.x.  Every role walks the same sequence and skips empty items
// the same way, so the K/V ring positions and the per-tile barrier phases
// continue across items.  At an item boundary the next item's K(0) and Q
// load under the current item's last tiles (Q once its S MMAs have read
// the buffer: q_empty), and its first S MMAs run under the softmax
// warpgroups' epilogue (its first PV waits only for O to be read: o_free).
template <typename T, int D, bool ROPE>
__global__ void __launch_bounds__(kThreads, 1)
fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, T* __restrict__ out,
                 float* __restrict__ lse, int B, int H, int Hkv, int Sq, int kv_len_max, int causal,
                 float scale_log2, int n_qtiles, const void* q_cos, const void* q_sin, int tbl_dtype,
                 const int32_t* __restrict__ kv_lens, const int32_t* __restrict__ q_offs) {
  using Cfg = FwdCfg<D>;
  constexpr int KS = Cfg::kKStages, VS = Cfg::kVStages;
  constexpr int fmt = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t idesc_qk = make_idesc_f16(fmt, kBM, kBN, 0, 0);
  constexpr uint32_t idesc_pv = make_idesc_f16(fmt, kBM, D, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + Cfg::kBarOff);
  const uint32_t sbase = smem_u32(smem);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_items = n_qtiles * B * H;
  // Round r of the item walk: left to right on even rounds, right to left on
  // odd ones, so that over the heaviest-first item order every CTA's total
  // work stays within about one item of the others.
  auto serpentine = [&](int r) {
    return r * (int)gridDim.x + ((r & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x);
  };
  auto item_at = [&](int item) {
    return fwd_item(item, B, H, Hkv, Sq, kv_len_max, causal, n_qtiles, kv_lens, q_offs);
  };

  if (threadIdx.x == 0) {
    mbar_init(&bars->q, 1);
    mbar_init(&bars->q_empty, 1);
    mbar_init(&bars->q_ready[0], kBM);
    mbar_init(&bars->q_ready[1], kBM);
    for (int s = 0; s < 4; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    mbar_init(&bars->drained, 1);
    for (int w = 0; w < 2; ++w) {
      mbar_init(&bars->s_full[w], 1);
      mbar_init(&bars->p_full[w], kBM + 1);  // softmax threads + the data certifier (K(j+1))
      mbar_init(&bars->p_half[w], kBM + 1);  // softmax threads + the data certifier (V(j))
      mbar_init(&bars->o_done[w], 1);
      mbar_init(&bars->o_free[w], kBM);
    }
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(&bars->tmem_base, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 8) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      // gk / gv: K / V tiles issued so far over all items (ring positions).
      int gk = 0, gv = 0, last_k = -1, last_v = -1, n_done = 0;
      bool okp = true;
      for (int r = 0; okp && r * (int)gridDim.x < n_items; ++r) {
        const int item = serpentine(r);
        if (item >= n_items) continue;
        const FwdItem t = item_at(item);
        if (t.n_max == 0) continue;
        const int kv_plane = t.b * Hkv + t.hk;
        auto load_k = [&](int j) -> bool {
          const int s = gk % KS;
          if (gk >= KS && !mbar_wait(&bars->k_empty[s], ((gk / KS) - 1) & 1)) return false;
          mbar_expect_tx(&bars->k_full[s], Cfg::kTileBytes);
          for (int c = 0; c < Cfg::kBoxes; ++c)
            tma_load_3d(smem + Cfg::kKOff + s * Cfg::kTileBytes + c * kBN * 128, &tm_k,
                        &bars->k_full[s], c * 64, j * kBN, kv_plane);
          last_k = gk++;
          trace(12, j);
          return true;
        };
        auto load_v = [&](int j) -> bool {
          const int s = gv % VS;
          if (gv >= VS && !mbar_wait(&bars->v_empty[s], ((gv / VS) - 1) & 1)) return false;
          mbar_expect_tx(&bars->v_full[s], Cfg::kTileBytes);
          for (int c = 0; c < Cfg::kBoxes; ++c)
            tma_load_3d(smem + Cfg::kVOff + s * Cfg::kTileBytes + c * kBN * 128, &tm_v,
                        &bars->v_full[s], c * 64, j * kBN, kv_plane);
          last_v = gv++;
          trace(13, j);
          return true;
        };
        okp = load_k(0);
        // The previous item's S MMAs must have read the Q buffer.
        if (okp && n_done > 0) okp = mbar_wait(&bars->q_empty, (n_done - 1) & 1);
        if (!okp) break;
        const int active = (t.n_w[0] > 0) + (t.n_w[1] > 0);
        mbar_expect_tx(&bars->q, active * Cfg::kTileBytes);
        for (int w = 0; w < 2; ++w) {
          if (t.n_w[w] == 0) continue;
          for (int c = 0; c < Cfg::kBoxes; ++c)
            tma_load_3d(smem + Cfg::kQOff + w * Cfg::kTileBytes + c * kBM * 128, &tm_q, &bars->q,
                        c * 64, t.q_start + w * kBM, t.bh);
        }
        ++n_done;
        // Issue order K0, K1, V0, K2, V1, ...: K one step ahead of V.
        for (int j = 1; okp && j <= t.n_max; ++j) {
          if (j < t.n_max) okp = load_k(j);
          okp = okp && load_v(j - 1);
        }
      }
      // Exit drain: no copy may land after the CTA is gone.
      if (n_done > 0) mbar_wait(&bars->q, (n_done - 1) & 1);
      drain_ring(bars->k_full, KS, last_k);
      drain_ring(bars->v_full, VS, last_v);
    }
  } else if (warp == 9) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0) {
      bool ok = true;
      // Descriptors are built once per tile; each k-step adds a constant.
      const uint64_t q_desc[2] = {desc_k_base<kBM>(sbase + Cfg::kQOff),
                                  desc_k_base<kBM>(sbase + Cfg::kQOff + Cfg::kTileBytes)};
      const uint32_t s_col[2] = {Cfg::kS0, Cfg::kS1};
      const uint32_t o_col[2] = {Cfg::kO0, Cfg::kO1};
      // Ring positions, S/P tiles per query-tile slot (barrier phases), and
      // items per slot (q_ready / o_free phases) over all items so far.
      int gk = 0, gv = 0, n_done = 0;
      int cnt[2] = {0, 0}, items_w[2] = {0, 0};
      for (int r = 0; ok && r * (int)gridDim.x < n_items; ++r) {
        const int item = serpentine(r);
        if (item >= n_items) continue;
        const FwdItem t = item_at(item);
        if (t.n_max == 0) continue;
        if (ROPE) {
          for (int w = 0; w < 2; ++w)
            if (t.n_w[w] > 0) ok = ok && mbar_wait(&bars->q_ready[w], items_w[w] & 1);
        } else {
          ok = mbar_wait(&bars->q, n_done & 1);
        }
        if (ok) ok = mbar_wait_spin(&bars->k_full[gk % KS], (gk / KS) & 1);
        tc_fence_after();
        auto issue_s = [&](int w, int j) {
          const uint64_t kd = desc_k_base<kBN>(sbase + Cfg::kKOff + ((gk + j) % KS) * Cfg::kTileBytes);
          const uint64_t qd = q_desc[w];
          const uint32_t dst = tmem + s_col[w];
          umma_ss(dst, qd, kd, idesc_qk, 0u);
#pragma unroll
          for (int kk = 1; kk < D / 16; ++kk) umma_ss_acc(dst, qd + koff<kBM>(kk), kd + koff<kBN>(kk), idesc_qk);
          umma_commit(&bars->s_full[w]);
        };
        // PV in two halves of the key axis: the first four k-steps start once
        // the softmax has written P for keys [0, 64) (p_half), the rest after
        // p_full.  The first PV of an item overwrites O, so it also waits
        // until the previous item's epilogue has read O (o_free).  Returns
        // false if a wait gave up.
        auto issue_pv = [&](int w, int j) -> bool {
          const uint64_t vd = desc_mn_base<kBN>(sbase + Cfg::kVOff + ((gv + j) % VS) * Cfg::kTileBytes);
          const uint32_t dst = tmem + o_col[w], src = tmem + s_col[w];
          const uint32_t ph = (cnt[w] + j) & 1;
          if (j == 0 && items_w[w] > 0 && !mbar_wait_spin(&bars->o_free[w], (items_w[w] - 1) & 1)) return false;
          if (!mbar_wait_spin(&bars->p_half[w], ph)) return false;
          tc_fence_after();
          umma_ts(dst, src, vd, idesc_pv, j > 0 ? 1u : 0u);
#pragma unroll
          for (int kk = 1; kk < kBN / 32; ++kk) umma_ts_acc(dst, src + kk * 8, vd + mnoff(kk), idesc_pv);
          if (!mbar_wait_spin(&bars->p_full[w], ph)) return false;
          tc_fence_after();
#pragma unroll
          for (int kk = kBN / 32; kk < kBN / 16; ++kk) umma_ts_acc(dst, src + kk * 8, vd + mnoff(kk), idesc_pv);
          umma_commit(&bars->o_done[w]);
          return true;
        };
        // Tile data is certified by warp 10 inside the softmax barrier phases:
        // p_half[w](j) completes only once V(j) is in shared memory and
        // p_full[w](j) once K(j+1) is, so apart from Q and K(0) of each item
        // this thread polls nothing but the softmax barriers (each poll it
        // waits on costs tensor-core time).
        const int n0 = t.n_w[0], n1 = t.n_w[1];
        for (int j = 0; ok && j <= t.n_max; ++j) {
          const int ks = (gk + j) % KS, vs = (gv + j) % VS;
          if (j < n0) {
            issue_s(0, j);
            trace(2, j);
            if (j >= n1) umma_commit(&bars->k_empty[ks]);  // only reader of K_j
          }
          if (j >= 1 && j - 1 < n1) {
            const int vp = (gv + j - 1) % VS;
            trace(3, j - 1);
            if (!(ok = issue_pv(1, j - 1))) break;
            umma_commit(&bars->v_empty[vp]);  // last reader of V_{j-1}
          }
          if (j < n1) {
            issue_s(1, j);
            trace(5, j);
            umma_commit(&bars->k_empty[ks]);  // last reader of K_j
          }
          if (j == t.n_max - 1) umma_commit(&bars->q_empty);  // the item's S MMAs are all issued
          if (j < n0) {
            trace(6, j);
            if (!(ok = issue_pv(0, j))) break;
            if (j >= n1) umma_commit(&bars->v_empty[vs]);
          }
        }
        gk += t.n_max;
        gv += t.n_max;
        for (int w = 0; w < 2; ++w) {
          cnt[w] += t.n_w[w];
          items_w[w] += t.n_w[w] > 0;
        }
        ++n_done;
      }
      umma_commit(&bars->drained);
    }
  } else if (warp == 10) {
    // --------------------------- data certifier ---------------------------
    // Adds one arrival to each softmax barrier phase once the tiles the MMA
    // issuer will read after that phase (V(j) after p_half(j), K(j+1) after
    // p_full(j)) have landed, then waits for the phases to complete so it
    // never arrives twice in one phase.
    if (lane == 0) {
      bool ok = true;
      int gk = 0, gv = 0, cnt[2] = {0, 0};
      for (int r = 0; ok && r * (int)gridDim.x < n_items; ++r) {
        const int item = serpentine(r);
        if (item >= n_items) continue;
        const FwdItem t = item_at(item);
        if (t.n_max == 0) continue;
        for (int j = 0; ok && j < t.n_max; ++j) {
          ok = mbar_wait(&bars->v_full[(gv + j) % VS], ((gv + j) / VS) & 1);
          if (!ok) break;
#pragma unroll
          for (int w = 0; w < 2; ++w)
            if (j < t.n_w[w]) mbar_arrive(&bars->p_half[w]);
          if (j + 1 < t.n_max) ok = mbar_wait(&bars->k_full[(gk + j + 1) % KS], ((gk + j + 1) / KS) & 1);
          if (!ok) break;
#pragma unroll
          for (int w = 0; w < 2; ++w)
            if (j < t.n_w[w]) mbar_arrive(&bars->p_full[w]);
#pragma unroll
          for (int w = 0; w < 2; ++w)
            if (ok && j < t.n_w[w])
              ok = mbar_wait(&bars->p_half[w], (cnt[w] + j) & 1) && mbar_wait(&bars->p_full[w], (cnt[w] + j) & 1);
        }
        gk += t.n_max;
        gv += t.n_max;
        cnt[0] += t.n_w[0];
        cnt[1] += t.n_w[1];
      }
    }
  } else if (warp < 8) {
    // ------------------------------ softmax -------------------------------
    const int w = warp / 4;                 // query tile of this warpgroup
    const int quad = warp % 4;              // TMEM lane quadrant
    const int row = quad * 32 + lane;       // row within the tile
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t s_addr = lane_base + (w == 0 ? Cfg::kS0 : Cfg::kS1);
    const uint32_t o_addr = lane_base + (w == 0 ? Cfg::kO0 : Cfg::kO1);
    bool ok = true;
    int cnt = 0, n_done = 0;  // S/P tiles of this slot and non-empty items so far
    bool rotated_ahead = false;  // this item's query tile was rotated before the previous epilogue
    for (int r = 0; ok && r * (int)gridDim.x < n_items; ++r) {
      const int item = serpentine(r);
      if (item >= n_items) continue;
      const FwdItem t = item_at(item);
      if (t.n_max == 0) continue;
      const int n = t.n_w[w];
      const int q_start = t.q_start, kv_len = t.kv_len, q_off = t.q_off;
      const int qpos = q_start + w * kBM + row;
      if (ROPE && n > 0 && !rotated_ahead) {
        // Rotate this warpgroup's query tile once, before any S MMA reads it.
        ok = mbar_wait(&bars->q, n_done & 1);
        if (ok && qpos < Sq)
          rope_row_in_smem<T, D>(smem + Cfg::kQOff + w * Cfg::kTileBytes, row, q_cos, q_sin, tbl_dtype, qpos);
        fence_proxy_async_smem();  // generic-proxy writes -> tensor-core (async proxy) reads
        mbar_arrive(&bars->q_ready[w]);
      }
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; ok && j < n; ++j) {
        if (!mbar_wait_spin(&bars->s_full[w], (cnt + j) & 1)) { ok = false; break; }
        if (threadIdx.x == 0 || threadIdx.x == 128) trace(8 + 2 * w, j);
        tc_fence_after();
        const int k0 = j * kBN;
        const bool edge = (k0 + kBN > kv_len) || (causal && k0 + kBN - 1 > q_start + w * kBM + q_off);
        // Visible-key count of this row in the tile: keys [k0, k0 + vis) survive
        // both the kv_len and the causal mask.
        int vis = kBN;
        if (edge) {
          vis = min(kBN, kv_len - k0);
          if (causal) vis = min(vis, qpos + q_off - k0 + 1);
          vis = max(vis, 0);
        }
        // Pass 1: row max.  All four 32-column loads are in flight before the
        // single wait; four independent three-input max chains.
        float mx;
        {
          uint32_t r[kBN / 32][32];
  #pragma unroll
          for (int c = 0; c < kBN / 32; ++c) tmem_ld32(s_addr + c * 32, r[c]);
          tmem_wait_ld();
          if (edge) {
  #pragma unroll
            for (int i = 0; i < kBN; ++i)
              if (i >= vis) r[i >> 5][i & 31] = __float_as_uint(-INFINITY);
          }
          float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  #pragma unroll
          for (int i = 0; i < kBN; i += 8) {
  #pragma unroll
            for (int u = 0; u < 4; ++u)
              mq[u] = fmax3(mq[u], __uint_as_float(r[(i + 2 * u) >> 5][(i + 2 * u) & 31]),
                            __uint_as_float(r[(i + 2 * u + 1) >> 5][(i + 2 * u + 1) & 31]));
          }
          mx = fmax3(mq[0], mq[1], fmaxf(mq[2], mq[3])) * scale_log2;
        }
        // Lazy rescale: raise the reference max only when it grew by > 2^8.
        const bool upd = mx > m_run + kRescaleThresh;
        const float alpha = upd ? fast_exp2(m_run - mx) : 1.f;  // 0 when m_run = -inf
        if (upd) {
          l_run *= alpha;
          m_run = mx;
        }
        if (j > 0 && __any_sync(0xffffffffu, upd)) {
          // PV of tile j-1 is complete: its commit preceded S_w(j)'s.
  #pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(o_addr + c * 32, o);
            tmem_wait_ld();
  #pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(o_addr + c * 32, o);
          }
        }
        // Pass 2: P = 2^(s*scale - m) in 64-column halves (two loads, one wait
        // each), packed to 16-bit pairs into the first half of the S columns
        // (a half's source columns are consumed before any store reaches them);
        // the row sum runs in four independent packed accumulators.
        const float msub = (m_run == -INFINITY) ? 0.f : m_run;
        const float2 sc2 = make_float2(scale_log2, scale_log2), nm2 = make_float2(-msub, -msub);
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                         make_float2(0.f, 0.f)};
  #pragma unroll
        for (int c = 0; c < kBN / 64; ++c) {
          uint32_t ra[2][32];
          tmem_ld32(s_addr + c * 64, ra[0]);
          tmem_ld32(s_addr + c * 64 + 32, ra[1]);
          tmem_wait_ld();
          uint32_t pk[32];
  #pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int cl = 2 * i, col = c * 64 + cl;
            const float2 x = fma2(make_float2(__uint_as_float(ra[cl >> 5][cl & 31]),
                                              __uint_as_float(ra[(cl + 1) >> 5][(cl + 1) & 31])), sc2, nm2);
            float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
            if (edge) {
              p.x = col < vis ? p.x : 0.f;
              p.y = col + 1 < vis ? p.y : 0.f;
            }
            acc[i & 3] = add2(acc[i & 3], p);
            pk[i] = (fmt == 1) ? pack_bf16x2(p.x, p.y) : pack_f16x2(p.x, p.y);
          }
          tmem_st32(s_addr + c * 32, pk);
          if (c == 0) {  // keys [0, 64) of P are in place: PV may start on them
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bars->p_half[w]);
          }
        }
        const float2 rs2 = add2(add2(acc[0], acc[1]), add2(acc[2], acc[3]));
        const float rowsum = rs2.x + rs2.y;
        l_run += rowsum;
        tmem_wait_st();
        tc_fence_before();
        if (threadIdx.x == 0 || threadIdx.x == 128) trace(9 + 2 * w, j);
        mbar_arrive(&bars->p_full[w]);
      }
      // RoPE: the next item's query tile lands once this item's S MMAs are done
      // (q_empty); rotating it now, before this item's epilogue, lets the
      // next item's first S MMAs run under the epilogue instead of after it.
      if (ROPE) {
        rotated_ahead = false;
        for (int r2 = r + 1; ok && r2 * (int)gridDim.x < n_items; ++r2) {
          const int item2 = serpentine(r2);
          if (item2 >= n_items) continue;
          const FwdItem t2 = item_at(item2);
          if (t2.n_max == 0) continue;
          if (t2.n_w[w] > 0) {
            ok = mbar_wait(&bars->q, (n_done + 1) & 1);
            const int qpos2 = t2.q_start + w * kBM + row;
            if (ok && qpos2 < Sq)
              rope_row_in_smem<T, D>(smem + Cfg::kQOff + w * Cfg::kTileBytes, row, q_cos, q_sin, tbl_dtype, qpos2);
            fence_proxy_async_smem();
            mbar_arrive(&bars->q_ready[w]);
            rotated_ahead = true;
          }
          break;
        }
      }
      // ---------------------------- epilogue ----------------------------
      if (n > 0) {
        if (ok && mbar_wait(&bars->o_done[w], (cnt + n - 1) & 1)) {
          tc_fence_after();
          const bool empty = (l_run == 0.f);
          const float inv = empty ? 0.f : 1.f / l_run;
          T* orow = out + ((long)t.bh * Sq + qpos) * D;
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(o_addr + c * 32, r);
            tmem_wait_ld();
            if (c == D / 32 - 1) {  // O is in registers: the next item's PV may overwrite it
              tc_fence_before();
              mbar_arrive(&bars->o_free[w]);
            }
            if (qpos < Sq) {
              uint32_t pk[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float a0 = __uint_as_float(r[2 * i]) * inv, a1 = __uint_as_float(r[2 * i + 1]) * inv;
                pk[i] = (fmt == 1) ? pack_bf16x2(a0, a1) : pack_f16x2(a0, a1);
              }
              uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
              for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
            }
          }
          if (lse != nullptr && qpos < Sq) lse[(long)t.bh * Sq + qpos] = empty ? 0.f : (m_run + log2f(l_run)) * kLn2;
        } else {
          ok = false;
        }
      }
      cnt += n;
      ++n_done;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    if (lane == 0) mbar_wait(&bars->drained, 0);  // no MMA may still write TMEM
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

template <typename T, int D, bool ROPE>
cudaError_t launch_t(const FwdArgs& a, const void* k_rot) {
  using Cfg = FwdCfg<D>;
  CUtensorMap tq, tk, tv;
  if (!make_tile_map(&tq, a.q, a.dtype, D, a.Sq, a.Sq, a.B * a.H, kBM) ||
      !make_tile_map(&tk, ROPE ? k_rot : a.k, a.dtype, D, a.kv_len, a.Sk, a.B * a.Hkv, kBN) ||
      !make_tile_map(&tv, a.v, a.dtype, D, a.kv_len, a.Sk, a.B * a.Hkv, kBN))
    return cudaErrorInvalidValue;
  auto kern = fwd_sm100_kernel<T, D, ROPE>;
  cudaError_t e = ensure_smem(kern, Cfg::kSmem);
  if (e != cudaSuccess) return e;
  const int n_qtiles = (a.Sq + 2 * kBM - 1) / (2 * kBM);
  // Persistent (one CTA per SM) when every sequence has the same length: the
  // serpentine walk over the heaviest-first order balances the CTAs.  With
  // per-sequence lengths (kv_lens) item costs no longer follow that order, so
  // each item gets its own CTA and the hardware balances them as CTAs retire.
  const int n_items = n_qtiles * a.B * a.H;
  dim3 grid((unsigned)(a.kv_lens != nullptr ? n_items : std::min(n_items, sm_count())));
  const float scale_log2 = a.sm_scale * kLog2e;
  kern<<<grid, kThreads, Cfg::kSmem, a.stream>>>(tq, tk, tv, (T*)a.o, a.lse, a.B, a.H, a.Hkv, a.Sq,
                                                 a.kv_len, a.causal, scale_log2, n_qtiles, a.q_cos, a.q_sin,
                                                 a.tbl_dtype, a.kv_lens, a.q_offs);
  return cudaGetLastError();
}


// K rotated once per row into `out` ([B*Hkv, Sk, D], rows < kv_len), so the
// attention kernel streams pre-rotated keys: each key row is rotated once
// instead of once per (query head, query tile) that reads it.
template <typename T, int D>
__global__ void rope_rows_kernel(const T* __restrict__ x, T* __restrict__ out, const void* cos_t,
                                 const void* sin_t, int tbl_dtype, int Sk, int kv_len, long n_items) {
  constexpr int half = D / 2, per_row = half / 8;
  for (long it = (long)blockIdx.x * blockDim.x + threadIdx.x; it < n_items; it += (long)gridDim.x * blockDim.x) {
    const long row = it / per_row;            // over planes * kv_len
    const int d0 = (int)(it % per_row) * 8, d1 = d0 + half;
    const long plane = row / kv_len;
    const int pos = (int)(row % kv_len);
    const long base = (plane * Sk + pos) * D;
    uint4 v0 = *reinterpret_cast<const uint4*>(x + base + d0);
    uint4 v1 = *reinterpret_cast<const uint4*>(x + base + d1);
    T* x0 = reinterpret_cast<T*>(&v0);
    T* x1 = reinterpret_cast<T*>(&v1);
    float c0[8], s0[8], c1[8], s1[8];
    load8_table(cos_t, tbl_dtype, (long)pos * D + d0, c0);
    load8_table(sin_t, tbl_dtype, (long)pos * D + d0, s0);
    load8_table(cos_t, tbl_dtype, (long)pos * D + d1, c1);
    load8_table(sin_t, tbl_dtype, (long)pos * D + d1, s1);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float a = to_f(x0[u]), bb = to_f(x1[u]);
      x0[u] = from_f<T>(rope_lo(a, bb, c0[u], s0[u]));
      x1[u] = from_f<T>(rope_hi(a, bb, c1[u], s1[u]));
    }
    *reinterpret_cast<uint4*>(out + base + d0) = v0;
    *reinterpret_cast<uint4*>(out + base + d1) = v1;
  }
}

template <typename T, int D>
cudaError_t launch_rope_t(const FwdArgs& a, void* k_rot) {
  const long n_items = (long)a.B * a.Hkv * a.kv_len * (D / 16);
  const int threads = 256;
  const long blocks = (n_items + threads - 1) / threads;
  rope_rows_kernel<T, D><<<(unsigned)(blocks < 148L * 32 ? blocks : 148L * 32), threads, 0, a.stream>>>(
      (const T*)a.k, (T*)k_rot, a.k_cos, a.k_sin, a.tbl_dtype, a.Sk, a.kv_len, n_items);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_t<T, D, true>(a, k_rot);
}

}  // namespace

bool fwd_sm100_supported(int dtype, int D) {
  return (dtype == PF_BF16 || dtype == PF_F16) && (D == 64 || D == 128);
}

cudaError_t launch_fwd_sm100(const FwdArgs& a) {
  if (a.dtype == PF_BF16)
    return a.D == 128 ? launch_t<__nv_bfloat16, 128, false>(a, nullptr) : launch_t<__nv_bfloat16, 64, false>(a, nullptr);
  return a.D == 128 ? launch_t<__half, 128, false>(a, nullptr) : launch_t<__half, 64, false>(a, nullptr);
}

size_t rope_fwd_sm100_workspace(int dtype, int B, int Hkv, int Sk, int D) {
  (void)dtype;
  return ((size_t)B * Hkv * Sk * D * 2 + 255) / 256 * 256;
}

cudaError_t launch_rope_fwd_sm100(const FwdArgs& a, void* k_rot) {
  if (a.dtype == PF_BF16)
    return a.D == 128 ? launch_rope_t<__nv_bfloat16, 128>(a, k_rot) : launch_rope_t<__nv_bfloat16, 64>(a, k_rot);
  return a.D == 128 ? launch_rope_t<__half, 128>(a, k_rot) : launch_rope_t<__half, 64>(a, k_rot);
}

}  // namespace pf
