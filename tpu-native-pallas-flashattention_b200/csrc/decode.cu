// decode.cu -- single-query (decode) attention over a fixed or paged KV cache,
// and the cache bookkeeping kernels.
//
// Decode is HBM-bound: every cached key and value is read once per step and
// each (4 B K + V) x D byte row supports only ~4 FLOP per byte.  The kernel
// therefore streams K/V with bulk asynchronous copies (cp.async.bulk, 16-byte
// aligned rows straight into shared memory, completion on an mbarrier) into a
// per-warp multi-stage ring, and one CTA serves every query head of a kv head
// group so K/V cross HBM once, not once per query head as in the reference's
// (batch, head, page) grid (paged.py:164-178).
//
// Split-KV: the cached positions of each (sequence, kv head) are cut into
// fixed-size splits (grid.x), each producing an un-normalised partial
// (acc, m, l) per query head; a combine kernel merges them.  Positions are
// assigned to splits / warps / lanes purely by absolute position, so a paged
// cache and the same cache laid out contiguously produce bit-identical
// results.
//
// Reference semantics: flash_attention_decode (flash_attention.py:555-589):
// attend positions [0, cache_len); paged_flash_attention (paged.py:45-99):
// position pos of sequence b is row pos % ps of page block_tables[b, pos/ps],
// positions >= context_lens[b] are masked and their pages never read.
#include "common.cuh"
#include "kernels.h"

namespace pf {
namespace {

constexpr int kKeysPerWarp = 32;
constexpr int kSplitQuantum = 128;   // split lengths are multiples of this
constexpr int kMaxSplitLen = 4096;
constexpr int kSingleSplitLen = 1024;  // caches up to this length decode in one split

template <typename T, int D>
struct DecodeCfg {
  static constexpr int kRowBytes = D * (int)sizeof(T);
  static constexpr int kWarpStageBytes = 2 * kKeysPerWarp * kRowBytes;  // K + V
  // Aim for ~192 KB of ring per CTA: 4 warps when rows are <= 256 bytes.
  static constexpr int kWarps = kRowBytes <= 256 ? 4 : (kRowBytes <= 512 ? 2 : 1);
  static constexpr int kStages = 3;
  static constexpr int kSmemRing = kWarps * kStages * kWarpStageBytes;
  static constexpr int kChunks = kRowBytes / 16;  // 16-byte chunks per row
  static constexpr int kElemsPerChunk = 16 / (int)sizeof(T);
  static constexpr int kNPL = D / 32;             // output dims per lane
};

template <int N, typename T> __device__ __forceinline__ void load_row_part(const T* p, float (&out)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = to_f(p[i]);
}

// One CTA = one split of one (sequence, kv head, head chunk).
// grid = (num_splits, Hkv * head_chunks, B); block = kWarps * 32.
template <typename T, int D, int GC>
__global__ void __launch_bounds__(DecodeCfg<T, D>::kWarps * 32)
decode_split_kernel(DecodeArgs a, int head_chunks) {
  using Cfg = DecodeCfg<T, D>;
  constexpr int W = Cfg::kWarps, S = Cfg::kStages, NPL = Cfg::kNPL;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem;                                            // [W][S][K|V][32][D]
  float* sQ = reinterpret_cast<float*>(smem + Cfg::kSmemRing);     // [GC][D]
  float* sRed = sQ + GC * D;                                       // [W][GC][D + 2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRed + W * GC * (D + 2));  // [W][S]

  const int split = blockIdx.x;
  const int hk = blockIdx.y / head_chunks;
  const int hchunk = blockIdx.y % head_chunks;
  const int b = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int G = a.H / a.Hkv;
  const int h0 = hk * G + hchunk * GC;
  const int gcount = min(GC, hk * G + G - h0);

  int len = a.context_lens ? a.context_lens[b] : a.fixed_len;
  if (a.block_tables != nullptr && len > a.pages_per_seq * a.page_size) {
    if (threadIdx.x == 0) flag_status(PF_DEV_BAD_PAGE);
    len = a.pages_per_seq * a.page_size;
  }
  // A length beyond the call's promised maximum would lose the keys past the
  // planned splits: record it (once per sequence and head group) instead of
  // silently attending a prefix.
  if (len > a.max_len && split == 0 && threadIdx.x == 0) flag_status(PF_DEV_LEN_OVER_MAX);
  const int k_begin = split * a.split_len;
  const int k_end = min(len, k_begin + a.split_len);
  if (k_begin >= k_end) return;  // the combine kernel ignores this split

  // q rows of this head chunk, pre-scaled so that exp2 applies directly.
  const float qscale = a.sm_scale * kLog2e;
  for (int i = threadIdx.x; i < GC * D; i += blockDim.x) {
    const int g = i / D;
    sQ[i] = g < gcount ? to_f(static_cast<const T*>(a.q)[((long)b * a.H + h0 + g) * D + i % D]) * qscale : 0.f;
  }
  uint64_t* wbar = bars + warp * S;
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
  }
  __syncthreads();

  const T* ksrc = static_cast<const T*>(a.k_src);
  const T* vsrc = static_cast<const T*>(a.v_src);
  uint8_t* wring = ring + (size_t)warp * S * Cfg::kWarpStageBytes;
  const int n_tiles = (k_end - k_begin + W * kKeysPerWarp - 1) / (W * kKeysPerWarp);
  // Tiles of this warp: t = 0..n_tiles-1, keys [tile_key(t), +32).
  auto tile_key = [&](int t) { return k_begin + (t * W + warp) * kKeysPerWarp; };
  auto tile_valid = [&](int t) { return max(0, min(kKeysPerWarp, k_end - tile_key(t))); };

  // Issues the copies of tile t into stage t % S (lane 0 only).
  auto issue = [&](int t) {
    const int kt = tile_key(t);
    const int nv = tile_valid(t);
    if (nv <= 0) return;
    uint64_t* bar = &wbar[t % S];
    uint8_t* kdst = wring + (size_t)(t % S) * Cfg::kWarpStageBytes;
    uint8_t* vdst = kdst + kKeysPerWarp * Cfg::kRowBytes;
    mbar_expect_tx(bar, (uint32_t)(2 * nv * Cfg::kRowBytes));
    int pos = kt;
    while (pos < kt + nv) {
      long row;   // row index into [*, D] of the source
      int run;    // consecutive rows available in this page
      if (a.block_tables == nullptr) {
        row = ((long)b * a.Hkv + hk) * a.cache_rows + pos;
        run = kt + nv - pos;
      } else {
        const int lp = pos / a.page_size, off = pos % a.page_size;
        int page = a.block_tables[(long)b * a.pages_per_seq + lp];
        if (page < 0 || page >= a.num_pages) {
          flag_status(PF_DEV_BAD_PAGE);
          page = 0;
        }
        row = ((long)page * a.Hkv + hk) * a.page_size + off;
        run = min(kt + nv - pos, a.page_size - off);
      }
      const int r = pos - kt;
      bulk_load(kdst + r * Cfg::kRowBytes, ksrc + row * D, run * Cfg::kRowBytes, bar);
      bulk_load(vdst + r * Cfg::kRowBytes, vsrc + row * D, run * Cfg::kRowBytes, bar);
      pos += run;
    }
  };

  if (lane == 0)
    for (int t = 0; t < S && t < n_tiles; ++t) issue(t);
  __syncwarp();

  float m[GC], l[GC], acc[GC][NPL];
#pragma unroll
  for (int g = 0; g < GC; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i) acc[g][i] = 0.f;
  }

  bool ok_all = true;
  int t_stop = 0;  // first tile not consumed
  for (int t = 0; t < n_tiles; ++t, t_stop = t) {
    const int nv = tile_valid(t);
    if (nv <= 0) break;  // later tiles of this warp are empty too
    if (!mbar_wait(&wbar[t % S], (t / S) & 1)) { ok_all = false; break; }
    const uint8_t* kbuf = wring + (size_t)(t % S) * Cfg::kWarpStageBytes;
    const uint8_t* vbuf = kbuf + kKeysPerWarp * Cfg::kRowBytes;

    // Scores: lane j owns key j; chunks are visited in a lane-rotated order
    // so the 16-byte shared loads of a quarter-warp hit distinct banks.
    float s[GC];
#pragma unroll
    for (int g = 0; g < GC; ++g) s[g] = 0.f;
    if (lane < nv) {
      const uint8_t* krow = kbuf + lane * Cfg::kRowBytes;
#pragma unroll 4
      for (int i = 0; i < Cfg::kChunks; ++i) {
        const int c = (lane + i) % Cfg::kChunks;
        const uint4 raw = *reinterpret_cast<const uint4*>(krow + c * 16);
        const T* e = reinterpret_cast<const T*>(&raw);
        float kf[Cfg::kElemsPerChunk];
#pragma unroll
        for (int u = 0; u < Cfg::kElemsPerChunk; ++u) kf[u] = to_f(e[u]);
#pragma unroll
        for (int g = 0; g < GC; ++g) {
          const float* qg = sQ + g * D + c * Cfg::kElemsPerChunk;
#pragma unroll
          for (int u = 0; u < Cfg::kElemsPerChunk; ++u) s[g] = fmaf(qg[u], kf[u], s[g]);
        }
      }
    }
    float p[GC];
#pragma unroll
    for (int g = 0; g < GC; ++g) {
      const float sv = lane < nv ? s[g] : -INFINITY;
      const float mn = fmaxf(m[g], warp_max(sv));  // finite: nv >= 1
      p[g] = lane < nv ? exp2f(sv - mn) : 0.f;
      const float alpha = exp2f(m[g] - mn);
      l[g] = l[g] * alpha + warp_sum(p[g]);
      m[g] = mn;
#pragma unroll
      for (int i = 0; i < NPL; ++i) acc[g][i] *= alpha;
    }
    // P.V: lane owns dims [lane*NPL, lane*NPL + NPL); only valid rows are read
    // (rows past the valid count may hold stale or uninitialised bytes).
    for (int j = 0; j < nv; ++j) {
      float vf[NPL];
      load_row_part<NPL>(reinterpret_cast<const T*>(vbuf + j * Cfg::kRowBytes) + lane * NPL, vf);
#pragma unroll
      for (int g = 0; g < GC; ++g) {
        const float pj = __shfl_sync(0xffffffffu, p[g], j);
#pragma unroll
        for (int i = 0; i < NPL; ++i) acc[g][i] = fmaf(pj, vf[i], acc[g][i]);
      }
    }
    __syncwarp();
    if (lane == 0 && t + S < n_tiles) issue(t + S);
    __syncwarp();
  }
  // Exit drain (only a timed-out wait leaves copies in flight): tiles
  // [0, t_stop + S) were issued, those before t_stop consumed.
  if (lane == 0)
    for (int u = t_stop; u < t_stop + S && u < n_tiles; ++u)
      if (tile_valid(u) > 0) mbar_wait(&wbar[u % S], (u / S) & 1);
  __syncwarp();

  // Merge the warps' states, then write this split's partial.
  float* myred = sRed + warp * GC * (D + 2);
#pragma unroll
  for (int g = 0; g < GC; ++g) {
#pragma unroll
    for (int i = 0; i < NPL; ++i) myred[g * (D + 2) + lane * NPL + i] = acc[g][i];
    if (lane == 0) {
      myred[g * (D + 2) + D] = m[g];
      myred[g * (D + 2) + D + 1] = l[g];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < gcount * D; e += blockDim.x) {
    const int g = e / D, d = e % D;
    float M = -INFINITY;
    for (int w = 0; w < W; ++w) M = fmaxf(M, sRed[(w * GC + g) * (D + 2) + D]);
    float L = 0.f, A = 0.f;
    for (int w = 0; w < W; ++w) {
      const float* r = sRed + (w * GC + g) * (D + 2);
      if (r[D] == -INFINITY) continue;
      const float sc = exp2f(r[D] - M);
      L += r[D + 1] * sc;
      A += r[d] * sc;
    }
    float* out = a.partial + (((long)b * a.H + h0 + g) * a.num_splits + split) * (D + 2);
    out[d] = A;
    if (d == 0) {
      out[D] = M;
      out[D + 1] = L;
    }
  }
  (void)ok_all;
}

// Merges the splits of each (sequence, q head) into the output row.
// grid = B * H, block = D threads (one per output dim).
template <typename T>
__global__ void decode_combine_kernel(DecodeArgs a) {
  const int bh = blockIdx.x;
  const int b = bh / a.H;
  const int D = a.D;
  int len = a.context_lens ? a.context_lens[b] : a.fixed_len;
  if (a.block_tables != nullptr) len = min(len, a.pages_per_seq * a.page_size);
  const int ns = min(a.num_splits, (len + a.split_len - 1) / a.split_len);
  const float* base = a.partial + (long)bh * a.num_splits * (D + 2);
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, base[s * (D + 2) + D]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.f, A = 0.f;
    for (int s = 0; s < ns; ++s) {
      const float* r = base + s * (D + 2);
      if (r[D] == -INFINITY) continue;
      const float sc = exp2f(r[D] - M);
      L += r[D + 1] * sc;
      A += r[d] * sc;
    }
    static_cast<T*>(a.o)[(long)bh * D + d] = from_f<T>(L == 0.f ? 0.f : A / L);
  }
}

template <typename T, int D, int GC>
cudaError_t launch_decode_t(const DecodeArgs& a) {
  using Cfg = DecodeCfg<T, D>;
  const int G = a.H / a.Hkv;
  const int head_chunks = (G + GC - 1) / GC;
  const size_t smem = Cfg::kSmemRing + (size_t)GC * D * 4 + (size_t)Cfg::kWarps * GC * (D + 2) * 4 +
                      (size_t)Cfg::kWarps * Cfg::kStages * 8;
  auto kern = decode_split_kernel<T, D, GC>;
  cudaError_t e = ensure_smem(kern, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.num_splits, a.Hkv * head_chunks, a.B);
  kern<<<grid, Cfg::kWarps * 32, smem, a.stream>>>(a, head_chunks);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_decode_combine(a);
}

template <typename T, int D>
cudaError_t launch_decode_gc(const DecodeArgs& a) {
  const int G = a.H / a.Hkv;
  if (G <= 1) return launch_decode_t<T, D, 1>(a);
  if (G <= 2) return launch_decode_t<T, D, 2>(a);
  if (G <= 4) return launch_decode_t<T, D, 4>(a);
  return launch_decode_t<T, D, 8>(a);
}

template <typename T>
cudaError_t launch_decode_d(const DecodeArgs& a) {
  switch (a.D) {
    case 64: return launch_decode_gc<T, 64>(a);
    case 128: return launch_decode_gc<T, 128>(a);
    default: return launch_decode_gc<T, 256>(a);
  }
}

// ---------------------------------------------------------------------------
// Cache bookkeeping
// ---------------------------------------------------------------------------
// One token per sequence into its page (paged.py:205-223).  The physical page
// index is clamped into [0, num_pages) the way dynamic_update_slice clamps.
template <typename T>
__global__ void paged_write_kernel(T* kp, T* vp, const T* k, const T* v, const int32_t* tables,
                                   const int32_t* positions, int Hkv, int num_pages, int ps,
                                   int pages_per_seq, int D) {
  const int b = blockIdx.y, hk = blockIdx.x;
  const int pos = positions[b];
  int lp = pos / ps;
  lp = min(max(lp, 0), pages_per_seq - 1);
  const int off = pos - (pos / ps) * ps;
  int page = tables[(long)b * pages_per_seq + lp];
  page = min(max(page, 0), num_pages - 1);
  const long dst = (((long)page * Hkv + hk) * ps + off) * D;
  const long src = ((long)b * Hkv + hk) * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    kp[dst + d] = k[src + d];
    vp[dst + d] = v[src + d];
  }
}

// One decode token per sequence: Q rotated in place and K rotated, at table
// row rope_pos[b], then K and V written into page block_tables[b,
// positions[b] / ps] at offset positions[b] % ps -- the step before the decode
// kernel (model.py:338-342 RoPE + _cache_write, paged.py:205-223), one launch
// instead of two RoPE expressions and a cache write.  Rotation
// y = x*cos + rotate_half(x)*sin in fp32 with one rounding; an out-of-range
// page (or logical page, or table row) is clamped like the page write above.
// grid = (H + Hkv, B), block = D/2 threads (one rotation pair each).
// Sequence b's q heads start at q_in + b * q_bs (written to q_out, contiguous
// [B, H, D]; q_out may equal q_in when q_bs = H * D), its k / v heads at
// k / v + b * kv_bs: separate tensors, or the slices of one fused projection row.
template <typename T>
__global__ void rope_paged_write_kernel(const T* q_in, long q_bs, T* q_out, T* kp, T* vp, const T* k, const T* v,
                                        long kv_bs, const void* cos_t, const void* sin_t, int tdtype,
                                        int table_rows, const int32_t* tables, const int32_t* positions,
                                        const int32_t* rope_pos, int H, int Hkv, int num_pages, int ps,
                                        int pages_per_seq, int D) {
  const int b = blockIdx.y, head = blockIdx.x, i = threadIdx.x, half = D / 2;
  if (i >= half) return;
  const long r = min(max(rope_pos[b], 0), table_rows - 1);
  const float c1 = load_any(cos_t, tdtype, r * D + i), s1 = load_any(sin_t, tdtype, r * D + i);
  const float c2 = load_any(cos_t, tdtype, r * D + i + half), s2 = load_any(sin_t, tdtype, r * D + i + half);
  if (head < H) {
    const T* x = q_in + (long)b * q_bs + (long)head * D;
    T* y = q_out + ((long)b * H + head) * D;
    const float x1 = to_f(x[i]), x2 = to_f(x[i + half]);
    y[i] = from_f<T>(rope_lo(x1, x2, c1, s1));
    y[i + half] = from_f<T>(rope_hi(x1, x2, c2, s2));
    return;
  }
  const int hk = head - H;
  const int pos = positions[b];
  const int lp = min(max(pos / ps, 0), pages_per_seq - 1);
  const int off = pos - (pos / ps) * ps;
  int page = tables[(long)b * pages_per_seq + lp];
  page = min(max(page, 0), num_pages - 1);
  const long dst = (((long)page * Hkv + hk) * ps + off) * D;
  const long src = (long)b * kv_bs + (long)hk * D;
  const float x1 = to_f(k[src + i]), x2 = to_f(k[src + i + half]);
  kp[dst + i] = from_f<T>(rope_lo(x1, x2, c1, s1));
  kp[dst + i + half] = from_f<T>(rope_hi(x1, x2, c2, s2));
  vp[dst + i] = v[src + i];
  vp[dst + i + half] = v[src + i + half];
}

// Paged prefill, step 1: the context of every sequence as contiguous rows
// [B, Hkv, T, D] (T = the longest context) plus the causal offsets
// q_offs[b] = context_lens[b] - L of the L-query chunk.  Only the rows the
// attention can load are produced: [0, context_lens[b]) from the pages and
// zeros up to the next 128-row tile boundary (the last tile is read whole;
// zeros keep 0 * V finite there).  Later rows are never loaded: every
// prefill kernel stops at the sequence's key length.  grid.x = B * Hkv
// planes, grid.y = chunks of a plane's 16-byte words (32-bit index math);
// an out-of-range page is flagged and read as page 0.
constexpr int kGatherTile = 128;
__global__ void paged_ctx_gather_kernel(const uint4* __restrict__ kpages, const uint4* __restrict__ vpages,
                                        const int32_t* __restrict__ tables, const int32_t* __restrict__ ctx,
                                        uint4* __restrict__ kout, uint4* __restrict__ vout, int32_t* q_offs,
                                        int L, int B, int Hkv, int num_pages, int ps, int pps, int T, int vec) {
  if (blockIdx.x == 0 && blockIdx.y == 0)
    for (int b = threadIdx.x; b < B; b += blockDim.x) q_offs[b] = ctx[b] - L;
  const int plane = blockIdx.x, b = plane / Hkv, hk = plane % Hkv;
  const int len = max(0, min(min(ctx[b], T), pps * ps));                  // rows with data
  const int lim = min(T, (max(0, min(ctx[b], T)) + kGatherTile - 1) / kGatherTile * kGatherTile);
  const int total = lim * vec;
  const int32_t* trow = tables + (long)b * pps;
  uint4* ko = kout + (long)plane * T * vec;
  uint4* vo = vout + (long)plane * T * vec;
  for (int w = blockIdx.y * blockDim.x + threadIdx.x; w < total; w += gridDim.y * blockDim.x) {
    const int t = w / vec, c = w - t * vec;
    uint4 kw = make_uint4(0, 0, 0, 0), vw = kw;
    if (t < len) {
      int page = trow[t / ps];
      if (page < 0 || page >= num_pages) {
        flag_status(PF_DEV_BAD_PAGE);
        page = 0;
      }
      const long src = (((long)page * Hkv + hk) * ps + t % ps) * vec + c;
      kw = kpages[src];
      vw = vpages[src];
    }
    ko[w] = kw;
    vo[w] = vw;
  }
}

// L tokens into slots (start + i) % C  (model.py:257-262 fixed cache,
// model.py:434-449 / :475-487 ring buffer).
template <typename T>
__global__ void cache_write_kernel(T* kc, T* vc, const T* k, const T* v, int Hkv, int C, int L,
                                   int D, int start) {
  const long row = blockIdx.x;  // over B * Hkv * L
  const int i = (int)(row % L);
  const long bh = row / L;
  const int slot = (int)(((long)start + i) % C);
  const long dst = (bh * C + slot) * D;
  const long src = row * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    kc[dst + d] = k[src + d];
    vc[dst + d] = v[src + d];
  }
}

// out[b, h, t] = pages[table[b, t / ps], h, t % ps]: byte copy of 16-bit or
// 32-bit words (the block-table index map of paged.py:158-159, materialised).
__global__ void paged_gather_kernel(const uint16_t* pages, const int32_t* tables, uint16_t* out,
                                    int Hkv, int num_pages, int ps, int pages_per_seq, int words) {
  const long row = blockIdx.x;  // over B * Hkv * pages_per_seq * ps
  const int T_ = pages_per_seq * ps;
  const int t = (int)(row % T_);
  const long bh = row / T_;
  const int hk = (int)(bh % Hkv);
  const long b = bh / Hkv;
  int page = tables[b * pages_per_seq + t / ps];
  if (page < 0 || page >= num_pages) {
    if (threadIdx.x == 0) flag_status(PF_DEV_BAD_PAGE);
    return;
  }
  const long src = (((long)page * Hkv + hk) * ps + t % ps) * words;
  for (int w = threadIdx.x; w < words; w += blockDim.x) out[row * words + w] = pages[src + w];
}

}  // namespace

bool decode_supported(int D) { return D == 64 || D == 128 || D == 256; }

void decode_plan(int max_len, int B, int Hkv, int* num_splits, int* split_len) {
  if (max_len <= kSingleSplitLen) {
    // Short caches (the generation decode step): one split, whose kernel writes
    // the output itself, saves the combine launch on a launch-bound step.
    *num_splits = 1;
    *split_len = (max_len + kSplitQuantum - 1) / kSplitQuantum * kSplitQuantum;
    return;
  }
  const int units = B * Hkv;
  const int target = 4 * 148;
  int splits = (target + units - 1) / units;
  splits = max(splits, (max_len + kMaxSplitLen - 1) / kMaxSplitLen);
  const int max_splits = max(1, (max_len + kSplitQuantum - 1) / kSplitQuantum);
  splits = max(1, min(splits, max_splits));
  int sl = (max_len + splits - 1) / splits;
  sl = (sl + kSplitQuantum - 1) / kSplitQuantum * kSplitQuantum;
  *split_len = sl;
  *num_splits = (max_len + sl - 1) / sl;
}

cudaError_t launch_decode_combine(const DecodeArgs& a) {
  const int th = a.D < 128 ? a.D : 128;
  switch (a.dtype) {
    case PF_F32: decode_combine_kernel<float><<<a.B * a.H, th, 0, a.stream>>>(a); break;
    case PF_BF16: decode_combine_kernel<__nv_bfloat16><<<a.B * a.H, th, 0, a.stream>>>(a); break;
    default: decode_combine_kernel<__half><<<a.B * a.H, th, 0, a.stream>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launch_decode(const DecodeArgs& a) {
  const bool paged = a.block_tables != nullptr;
  const long rows = paged ? (long)a.num_pages * a.Hkv * a.page_size : 0;
  if (decode_tc_supported(a.dtype, a.D, a.page_size, paged, rows)) return launch_decode_tc(a);
  switch (a.dtype) {
    case PF_F32: return launch_decode_d<float>(a);
    case PF_BF16: return launch_decode_d<__nv_bfloat16>(a);
    default: return launch_decode_d<__half>(a);
  }
}

cudaError_t launch_paged_write(void* k_pages, void* v_pages, const void* k, const void* v,
                               const int32_t* block_tables, const int32_t* positions, int dtype,
                               int B, int Hkv, int num_pages, int page_size, int pages_per_seq,
                               int D, cudaStream_t stream) {
  dim3 grid(Hkv, B);
  const int th = D < 256 ? D : 256;
#define PF_PW(T) paged_write_kernel<T><<<grid, th, 0, stream>>>((T*)k_pages, (T*)v_pages, (const T*)k, (const T*)v, block_tables, positions, Hkv, num_pages, page_size, pages_per_seq, D)
  if (dtype == PF_F32) PF_PW(float);
  else if (dtype == PF_BF16) PF_PW(__nv_bfloat16);
  else PF_PW(__half);
#undef PF_PW
  return cudaGetLastError();
}

cudaError_t launch_paged_ctx_gather(const void* k_pages, const void* v_pages, const int32_t* block_tables,
                                    const int32_t* context_lens, void* kout, void* vout, int32_t* q_offs, int L,
                                    int B, int Hkv, int num_pages, int page_size, int pages_per_seq, int T,
                                    int row_bytes, cudaStream_t stream) {
  const int vec = row_bytes / 16;
  const long planes = (long)B * Hkv;
  if (planes <= 0) return cudaSuccess;
  // ~8 words per thread, and enough blocks over all planes to fill the GPU.
  const long per_plane = (long)T * vec;
  long chunks = (per_plane + 256 * 8 - 1) / (256 * 8);
  const long min_chunks = ((long)sm_count() * 8 + planes - 1) / planes;
  if (chunks < min_chunks) chunks = min(min_chunks, (per_plane + 255) / 256);
  if (chunks < 1) chunks = 1;
  if (chunks > 65535) chunks = 65535;
  const dim3 grid((unsigned)planes, (unsigned)chunks);
  paged_ctx_gather_kernel<<<grid, 256, 0, stream>>>((const uint4*)k_pages, (const uint4*)v_pages, block_tables,
                                                      context_lens, (uint4*)kout, (uint4*)vout, q_offs, L, B, Hkv,
                                                      num_pages, page_size, pages_per_seq, T, vec);
  return cudaGetLastError();
}

cudaError_t launch_rope_paged_write(const void* q_in, long q_bs, void* q_out, void* k_pages, void* v_pages,
                                    const void* k, const void* v, long kv_bs, const void* cos_t, const void* sin_t,
                                    int tdtype, int table_rows, const int32_t* block_tables,
                                    const int32_t* positions, const int32_t* rope_pos, int dtype, int B, int H,
                                    int Hkv, int num_pages, int page_size, int pages_per_seq, int D,
                                    cudaStream_t stream) {
  const dim3 grid(H + Hkv, B);
  const int th = ((D / 2 + 31) / 32) * 32;
#define PF_RPW(T)                                                                                               \
  rope_paged_write_kernel<T><<<grid, th, 0, stream>>>((const T*)q_in, q_bs, (T*)q_out, (T*)k_pages, (T*)v_pages, \
                                                      (const T*)k, (const T*)v, kv_bs, cos_t, sin_t, tdtype,     \
                                                      table_rows, block_tables, positions, rope_pos, H, Hkv,     \
                                                      num_pages, page_size, pages_per_seq, D)
  if (dtype == PF_F32) PF_RPW(float);
  else if (dtype == PF_BF16) PF_RPW(__nv_bfloat16);
  else PF_RPW(__half);
#undef PF_RPW
  return cudaGetLastError();
}

cudaError_t launch_cache_write(void* k_cache, void* v_cache, const void* k, const void* v,
                               int dtype, int B, int Hkv, int C, int L, int D, int start,
                               cudaStream_t stream) {
  const long rows = (long)B * Hkv * L;
  if (rows == 0) return cudaSuccess;
  const int th = D < 256 ? D : 256;
#define PF_CW(T) cache_write_kernel<T><<<(unsigned)rows, th, 0, stream>>>((T*)k_cache, (T*)v_cache, (const T*)k, (const T*)v, Hkv, C, L, D, start)
  if (dtype == PF_F32) PF_CW(float);
  else if (dtype == PF_BF16) PF_CW(__nv_bfloat16);
  else PF_CW(__half);
#undef PF_CW
  return cudaGetLastError();
}

cudaError_t launch_paged_gather(const void* pages, const int32_t* block_tables, void* out,
                                int dtype, int B, int Hkv, int num_pages, int page_size,
                                int pages_per_seq, int D, cudaStream_t stream) {
  const long rows = (long)B * Hkv * pages_per_seq * page_size;
  if (rows == 0) return cudaSuccess;
  const int words = D * dtype_size(dtype) / 2;
  paged_gather_kernel<<<(unsigned)rows, 64, 0, stream>>>((const uint16_t*)pages, block_tables,
                                                         (uint16_t*)out, Hkv, num_pages, page_size,
                                                         pages_per_seq, words);
  return cudaGetLastError();
}

}  // namespace pf
