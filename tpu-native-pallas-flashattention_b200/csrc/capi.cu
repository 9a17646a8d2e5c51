// capi.cu -- the extern "C" boundary of libpallas_flash_b200.so.
//
// Validates arguments with the reference's rules (the ValueError checks of
// flash_attention.py:527-545, fused_rope.py:154-181, paged.py:129-149),
// picks the kernel family and launches on the caller's stream.  Nothing here
// allocates device memory; scratch comes from the caller's workspace.
#include <climits>
#include <cstdio>
#include <cstring>
#include <cstdarg>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

using namespace pf;

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return PF_OK;
  return fail(PF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool valid_dtype(int d) { return d == PF_F32 || d == PF_BF16 || d == PF_F16; }
size_t elem_bytes(int d) { return d == PF_F32 ? 4 : 2; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_attn_shapes(const char* fn, const void* q, const void* k, const void* v, int dtype,
                      int B, int H, int Hkv, int Sq, int Sk, int D, int kv_len) {
  if (!valid_dtype(dtype)) return fail(PF_ERR_INVALID, "%s: unknown dtype %d", fn, dtype);
  if (q == nullptr || k == nullptr || v == nullptr) return fail(PF_ERR_INVALID, "%s: null input", fn);
  if (B <= 0 || H <= 0 || Sq <= 0 || Sk <= 0 || D <= 0)
    return fail(PF_ERR_INVALID, "%s: shapes must be positive (B=%d H=%d Sq=%d Sk=%d D=%d)", fn, B, H, Sq, Sk, D);
  if (Hkv <= 0 || H % Hkv != 0)
    return fail(PF_ERR_INVALID,
                "%s: num_heads (%d) must be a multiple of num_kv_heads (%d) for grouped-query attention",
                fn, H, Hkv);
  if (kv_len <= 0 || kv_len > Sk)
    return fail(PF_ERR_INVALID, "%s: kv_len must be in (0, %d], got %d", fn, Sk, kv_len);
  if (D > 256) return fail(PF_ERR_UNSUPPORTED, "%s: head_dim %d > 256 is not built", fn, D);
  return PF_OK;
}

}  // namespace

namespace pf {
int set_last_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}
// One CTA waits (bounded) on an mbarrier that nothing ever arrives on: the
// wait gives up after g_wait_limit_ns, records PF_DEV_WAIT_TIMEOUT and the
// kernel returns.  Exercises the timeout path that every pipelined kernel
// relies on, without any other kernel misbehaving.
__global__ void wait_timeout_selftest_kernel() {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0);
  __syncthreads();
}
}  // namespace pf

extern "C" {

const char* pf_last_error(void) { return g_err; }
const char* pf_version(void) { return "0.1.0+sm100a"; }

int pf_device_status(int* bits_out, int reset) {
  int v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "pf_device_status");
  e = cudaMemcpyFromSymbol(&v, g_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "pf_device_status");
  if (bits_out) *bits_out = v;
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_status, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "pf_device_status");
  }
  return PF_OK;
}

int pf_set_wait_limit_ns(unsigned long long ns) {
  const unsigned long long v = ns == 0 ? (unsigned long long)kWaitLimitNs : ns;
  return cuda_status(cudaMemcpyToSymbol(g_wait_limit_ns, &v, sizeof(v)), "pf_set_wait_limit_ns");
}

int pf_selftest_wait_timeout(void* stream) {
  wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>();
  return cuda_status(cudaGetLastError(), "pf_selftest_wait_timeout");
}

#ifdef PF_TRACE
// Development builds only: copies the phase trace out and clears it.
int pf_trace_read(unsigned long long* dst, unsigned int* counts) {
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(dst, g_trace, sizeof(unsigned long long) * kTraceCtas * kTraceEvents);
  cudaMemcpyFromSymbol(counts, g_trace_n, sizeof(unsigned int) * kTraceCtas);
  void* p = nullptr;
  cudaGetSymbolAddress(&p, g_trace);
  return cuda_status(cudaMemset(p, 0, sizeof(unsigned long long) * kTraceCtas * kTraceEvents), "pf_trace_read");
}
#endif

int pf_fwd_kernel_kind(int dtype, int head_dim) { return fwd_sm100_supported(dtype, head_dim) ? 1 : 0; }

int pf_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int dtype, int B,
           int H, int Hkv, int Sq, int Sk, int D, int causal, float sm_scale, int kv_len,
           void* stream) {
  int st = check_attn_shapes("pf_fwd", q, k, v, dtype, B, H, Hkv, Sq, Sk, D, kv_len);
  if (st != PF_OK) return st;
  if (o == nullptr) return fail(PF_ERR_INVALID, "pf_fwd: null output");
  FwdArgs a{};
  a.q = q; a.k = k; a.v = v; a.o = o; a.lse = lse;
  a.dtype = dtype; a.B = B; a.H = H; a.Hkv = Hkv; a.Sq = Sq; a.Sk = Sk; a.D = D;
  a.causal = causal != 0; a.kv_len = kv_len; a.sm_scale = sm_scale;
  a.stream = static_cast<cudaStream_t>(stream);
  if (fwd_sm100_supported(dtype, D) && aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o))
    return cuda_status(launch_fwd_sm100(a), "pf_fwd (tcgen05)");
  return cuda_status(launch_fwd_simt(a), "pf_fwd (simt)");
}

size_t pf_rope_fwd_workspace_size(int dtype, int B, int Hkv, int Sk, int D) {
  if (!fwd_sm100_supported(dtype, D) || B <= 0 || Hkv <= 0 || Sk <= 0) return 0;
  return rope_fwd_sm100_workspace(dtype, B, Hkv, Sk, D);
}

int pf_rope_fwd(const void* q, const void* k, const void* v, const void* q_cos, const void* q_sin,
                const void* k_cos, const void* k_sin, int tbl_dtype, void* o, int dtype, int B,
                int H, int Hkv, int Sq, int Sk, int D, int causal, float sm_scale, int kv_len,
                void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_attn_shapes("pf_rope_fwd", q, k, v, dtype, B, H, Hkv, Sq, Sk, D, kv_len);
  if (st != PF_OK) return st;
  if (D % 2 != 0) return fail(PF_ERR_INVALID, "pf_rope_fwd: head_dim must be even for RoPE, got %d", D);
  if (!valid_dtype(tbl_dtype)) return fail(PF_ERR_INVALID, "pf_rope_fwd: unknown table dtype %d", tbl_dtype);
  if (!q_cos || !q_sin || !k_cos || !k_sin) return fail(PF_ERR_INVALID, "pf_rope_fwd: null rope table");
  if (o == nullptr) return fail(PF_ERR_INVALID, "pf_rope_fwd: null output");
  FwdArgs a{};
  a.q = q; a.k = k; a.v = v; a.o = o; a.lse = nullptr;
  a.dtype = dtype; a.B = B; a.H = H; a.Hkv = Hkv; a.Sq = Sq; a.Sk = Sk; a.D = D;
  a.causal = causal != 0; a.kv_len = kv_len; a.sm_scale = sm_scale;
  a.q_cos = q_cos; a.q_sin = q_sin; a.k_cos = k_cos; a.k_sin = k_sin; a.tbl_dtype = tbl_dtype;
  a.stream = static_cast<cudaStream_t>(stream);
  if (fwd_sm100_supported(dtype, D) && aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o)) {
    const size_t need = rope_fwd_sm100_workspace(dtype, B, Hkv, Sk, D);
    if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
      return fail(PF_ERR_WORKSPACE, "pf_rope_fwd: workspace of %zu bytes required, got %zu", need, workspace_bytes);
    return cuda_status(launch_rope_fwd_sm100(a, workspace), "pf_rope_fwd (tcgen05)");
  }
  return cuda_status(launch_fwd_simt(a), "pf_rope_fwd (simt)");
}

int pf_bwd_preprocess(const void* o, const void* dout, float* delta, int dtype, int B, int H,
                      int Sq, int D, void* stream) {
  if (!valid_dtype(dtype) || !o || !dout || !delta) return fail(PF_ERR_INVALID, "pf_bwd_preprocess: bad argument");
  return cuda_status(launch_bwd_preprocess(o, dout, delta, dtype, (long)B * H * Sq, D,
                                           static_cast<cudaStream_t>(stream)),
                     "pf_bwd_preprocess");
}

// Tensor-core backward: 16-bit inputs, head_dim 64/128, 16-byte aligned operands.
static bool use_tc_bwd(const BwdArgs& a) {
  return bwd_sm100_supported(a.dtype, a.D) && aligned16(a.q) && aligned16(a.k) && aligned16(a.v) &&
         aligned16(a.dout) && (a.dq == nullptr || aligned16(a.dq)) && (a.dk == nullptr || aligned16(a.dk)) &&
         (a.dv == nullptr || aligned16(a.dv));
}

static int fill_bwd(BwdArgs* a, const char* fn, const void* q, const void* k, const void* v,
                    const void* dout, const float* lse, const float* delta, int dtype, int B,
                    int H, int Hkv, int Sq, int Sk, int D, int causal, float sm_scale, int kv_len,
                    void* stream) {
  int st = check_attn_shapes(fn, q, k, v, dtype, B, H, Hkv, Sq, Sk, D, kv_len);
  if (st != PF_OK) return st;
  if (!dout || !lse || !delta) return fail(PF_ERR_INVALID, "%s: null dout/lse/delta", fn);
  *a = BwdArgs{};
  a->q = q; a->k = k; a->v = v; a->dout = dout; a->lse = lse; a->delta = delta;
  a->dtype = dtype; a->B = B; a->H = H; a->Hkv = Hkv; a->Sq = Sq; a->Sk = Sk; a->D = D;
  a->causal = causal != 0; a->sm_scale = sm_scale; a->kv_len = kv_len;
  a->stream = static_cast<cudaStream_t>(stream);
  return PF_OK;
}

int pf_bwd_dq(const void* q, const void* k, const void* v, const void* dout, const float* lse,
              const float* delta, void* dq, int dtype, int B, int H, int Hkv, int Sq, int Sk,
              int D, int causal, float sm_scale, int kv_len, void* stream) {
  BwdArgs a;
  int st = fill_bwd(&a, "pf_bwd_dq", q, k, v, dout, lse, delta, dtype, B, H, Hkv, Sq, Sk, D,
                    causal, sm_scale, kv_len, stream);
  if (st != PF_OK) return st;
  if (!dq) return fail(PF_ERR_INVALID, "pf_bwd_dq: null dq");
  a.dq = dq;
  if (use_tc_bwd(a)) return cuda_status(launch_bwd_dq_sm100(a), "pf_bwd_dq (tcgen05)");
  return cuda_status(launch_bwd_dq_simt(a), "pf_bwd_dq");
}

int pf_bwd_dkv(const void* q, const void* k, const void* v, const void* dout, const float* lse,
               const float* delta, void* dk, void* dv, int dtype, int B, int H, int Hkv, int Sq,
               int Sk, int D, int causal, float sm_scale, int kv_len, void* stream) {
  BwdArgs a;
  int st = fill_bwd(&a, "pf_bwd_dkv", q, k, v, dout, lse, delta, dtype, B, H, Hkv, Sq, Sk, D,
                    causal, sm_scale, kv_len, stream);
  if (st != PF_OK) return st;
  if (!dk || !dv) return fail(PF_ERR_INVALID, "pf_bwd_dkv: null dk/dv");
  a.dk = dk; a.dv = dv;
  if (use_tc_bwd(a)) return cuda_status(launch_bwd_dkv_sm100(a), "pf_bwd_dkv (tcgen05)");
  return cuda_status(launch_bwd_dkv_simt(a), "pf_bwd_dkv");
}

static size_t bwd_delta_bytes(int B, int H, int Sq) {
  return ((size_t)B * H * Sq * sizeof(float) + 255) / 256 * 256;
}

size_t pf_bwd_workspace_size(int dtype, int B, int H, int Hkv, int Sq, int Sk, int D, int causal,
                             int kv_len) {
  (void)Hkv;
  if (B <= 0 || H <= 0 || Sq <= 0 || Sk <= 0) return 0;
  const size_t delta = bwd_delta_bytes(B, H, Sq);
  if (!bwd_sm100_supported(dtype, D)) return delta;
  if (kv_len <= 0 || kv_len > Sk) kv_len = Sk;
  return delta + bwd_ds_spill_bytes(B, H, Sq, kv_len, causal != 0) +
         bwd_dkv_part_bytes(B, Hkv, Sk, D, bwd_dkv_head_parts(B, H, Hkv, Sk));
}

int pf_bwd_head_parts(int B, int H, int Hkv, int Sk) { return bwd_dkv_head_parts(B, H, Hkv, Sk); }

int pf_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
           const float* lse, void* dq, void* dk, void* dv, int dtype, int B, int H, int Hkv,
           int Sq, int Sk, int D, int causal, float sm_scale, int kv_len, void* workspace,
           size_t workspace_bytes, void* stream) {
  if (B <= 0 || H <= 0 || Sq <= 0) return fail(PF_ERR_INVALID, "pf_bwd: shapes must be positive");
  const size_t need = bwd_delta_bytes(B, H, Sq);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(PF_ERR_WORKSPACE, "pf_bwd: workspace of at least %zu bytes required, got %zu", need,
                workspace_bytes);
  if (!o) return fail(PF_ERR_INVALID, "pf_bwd: null o");
  float* delta = static_cast<float*>(workspace);
  BwdArgs a;
  int st = fill_bwd(&a, "pf_bwd", q, k, v, dout, lse, delta, dtype, B, H, Hkv, Sq, Sk, D, causal,
                    sm_scale, kv_len, stream);
  if (st != PF_OK) return st;
  if (!dq || !dk || !dv) return fail(PF_ERR_INVALID, "pf_bwd: null gradient output");
  a.dq = dq; a.dk = dk; a.dv = dv;
  st = cuda_status(launch_bwd_preprocess(o, dout, delta, dtype, (long)B * H * Sq, D, a.stream), "pf_bwd (delta)");
  if (st != PF_OK) return st;
  if (use_tc_bwd(a)) {
    // With room for the dS spill: dK/dV writes every dS tile and dQ is one GEMM
    // over them (5 tile GEMMs per key/query tile pair); otherwise the dQ kernel
    // recomputes S and dP (7).
    const size_t spill = bwd_ds_spill_bytes(B, H, Sq, kv_len, a.causal);
    if (workspace_bytes >= need + spill) {
      a.ds_buf = reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(workspace) + need);
      // Small problems (fewer key-tile CTAs than SMs): split each kv group's q heads over
      // several CTAs when the workspace also holds their f32 partial dK/dV.
      const int parts = bwd_dkv_head_parts(B, H, Hkv, Sk);
      const size_t part_bytes = bwd_dkv_part_bytes(B, Hkv, Sk, D, parts);
      if (parts > 1 && workspace_bytes >= need + spill + part_bytes) {
        a.dkv_part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + need + spill);
        a.head_parts = parts;
      }
      // Measured and dropped: chunking the units and overlapping each chunk's dQ
      // GEMM (side stream, small grid) with the next chunk's dK/dV -- a chunk of
      // dK/dV CTAs is bound by its heaviest key tile, so the chunks' tails cost
      // more than the overlap gains (2.2 vs 1.65 ms at config 2).
      st = cuda_status(launch_bwd_dkv_sm100(a), "pf_bwd (dkv + dS spill, tcgen05)");
      if (st != PF_OK) return st;
      return cuda_status(launch_bwd_dq_gemm_sm100(a), "pf_bwd (dq gemm, tcgen05)");
    }
    st = cuda_status(launch_bwd_dkv_sm100(a), "pf_bwd (dkv, tcgen05)");
    if (st != PF_OK) return st;
    return cuda_status(launch_bwd_dq_sm100(a), "pf_bwd (dq, tcgen05)");
  }
  st = cuda_status(launch_bwd_dq_simt(a), "pf_bwd (dq)");
  if (st != PF_OK) return st;
  return cuda_status(launch_bwd_dkv_simt(a), "pf_bwd (dkv)");
}

// ------------------------------- decode --------------------------------------
static size_t decode_ws(int B, int H, int Hkv, int max_len, int D) {
  int ns, sl;
  decode_plan(max_len, B, Hkv, &ns, &sl);
  return (size_t)B * H * ns * (D + 2) * sizeof(float);
}

size_t pf_decode_workspace_size(int B, int H, int Hkv, int C, int D) {
  if (B <= 0 || H <= 0 || Hkv <= 0 || C <= 0 || D <= 0) return 0;
  return decode_ws(B, H, Hkv, C, D);
}

int pf_decode(const void* q, const void* k_cache, const void* v_cache, void* o, int dtype, int B,
              int H, int Hkv, int C, int D, int cache_len, float sm_scale, void* workspace,
              size_t workspace_bytes, void* stream) {
  int st = check_attn_shapes("pf_decode", q, k_cache, v_cache, dtype, B, H, Hkv, 1, C, D, cache_len);
  if (st != PF_OK) return st;
  if (!o) return fail(PF_ERR_INVALID, "pf_decode: null output");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!decode_supported(D) || !aligned16(k_cache) || !aligned16(v_cache)) {
    // Odd head sizes: the general forward kernel with one query row.
    FwdArgs a{};
    a.q = q; a.k = k_cache; a.v = v_cache; a.o = o; a.lse = nullptr;
    a.dtype = dtype; a.B = B; a.H = H; a.Hkv = Hkv; a.Sq = 1; a.Sk = C; a.D = D;
    a.causal = 0; a.kv_len = cache_len; a.sm_scale = sm_scale; a.stream = s;
    return cuda_status(launch_fwd_simt(a), "pf_decode (simt)");
  }
  DecodeArgs a{};
  a.q = q; a.k_src = k_cache; a.v_src = v_cache; a.block_tables = nullptr; a.context_lens = nullptr;
  a.fixed_len = cache_len; a.o = o; a.dtype = dtype; a.B = B; a.H = H; a.Hkv = Hkv; a.D = D;
  a.page_size = 1; a.cache_rows = C; a.max_len = C; a.sm_scale = sm_scale; a.stream = s;
  decode_plan(C, B, Hkv, &a.num_splits, &a.split_len);
  const size_t need = (size_t)B * H * a.num_splits * (D + 2) * sizeof(float);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(PF_ERR_WORKSPACE, "pf_decode: workspace of %zu bytes required, got %zu", need, workspace_bytes);
  a.partial = static_cast<float*>(workspace);
  return cuda_status(launch_decode(a), "pf_decode");
}

size_t pf_paged_decode_workspace_size(int B, int H, int Hkv, int page_size, int max_context_len, int D) {
  (void)page_size;
  if (B <= 0 || H <= 0 || Hkv <= 0 || max_context_len <= 0 || D <= 0) return 0;
  return decode_ws(B, H, Hkv, max_context_len, D);
}

int pf_paged_decode(const void* q, const void* k_pages, const void* v_pages,
                    const int32_t* block_tables, const int32_t* context_lens, void* o, int dtype,
                    int B, int H, int Hkv, int num_pages, int page_size, int pages_per_seq, int D,
                    int max_context_len, float sm_scale, void* workspace, size_t workspace_bytes,
                    void* stream) {
  if (!valid_dtype(dtype)) return fail(PF_ERR_INVALID, "pf_paged_decode: unknown dtype %d", dtype);
  if (!q || !k_pages || !v_pages || !block_tables || !context_lens || !o)
    return fail(PF_ERR_INVALID, "pf_paged_decode: null argument");
  if (B <= 0 || H <= 0 || D <= 0 || num_pages <= 0 || page_size <= 0 || pages_per_seq <= 0)
    return fail(PF_ERR_INVALID, "pf_paged_decode: shapes must be positive");
  if (Hkv <= 0 || H % Hkv != 0)
    return fail(PF_ERR_INVALID, "pf_paged_decode: num_heads (%d) must be a multiple of num_kv_heads (%d)", H, Hkv);
  if (!decode_supported(D))
    return fail(PF_ERR_UNSUPPORTED, "pf_paged_decode: head_dim %d not built (64, 128, 256)", D);
  if (!aligned16(k_pages) || !aligned16(v_pages))
    return fail(PF_ERR_INVALID, "pf_paged_decode: page pools must be 16-byte aligned");
  const long long cap = (long long)pages_per_seq * page_size;
  if (cap > INT_MAX)
    return fail(PF_ERR_INVALID, "pf_paged_decode: pages_per_seq * page_size = %lld exceeds INT_MAX", cap);
  if (max_context_len <= 0 || max_context_len > cap) max_context_len = (int)cap;
  DecodeArgs a{};
  a.q = q; a.k_src = k_pages; a.v_src = v_pages; a.block_tables = block_tables;
  a.context_lens = context_lens; a.o = o; a.dtype = dtype; a.B = B; a.H = H; a.Hkv = Hkv; a.D = D;
  a.num_pages = num_pages; a.page_size = page_size; a.pages_per_seq = pages_per_seq;
  a.max_len = max_context_len; a.sm_scale = sm_scale; a.stream = static_cast<cudaStream_t>(stream);
  decode_plan(max_context_len, B, Hkv, &a.num_splits, &a.split_len);
  const size_t need = (size_t)B * H * a.num_splits * (D + 2) * sizeof(float);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(PF_ERR_WORKSPACE, "pf_paged_decode: workspace of %zu bytes required, got %zu", need, workspace_bytes);
  a.partial = static_cast<float*>(workspace);
  return cuda_status(launch_decode(a), "pf_paged_decode");
}

int pf_paged_write(void* k_pages, void* v_pages, const void* k, const void* v,
                   const int32_t* block_tables, const int32_t* positions, int dtype, int B, int Hkv,
                   int num_pages, int page_size, int pages_per_seq, int D, void* stream) {
  if (!valid_dtype(dtype) || !k_pages || !v_pages || !k || !v || !block_tables || !positions)
    return fail(PF_ERR_INVALID, "pf_paged_write: bad argument");
  if (B <= 0 || Hkv <= 0 || num_pages <= 0 || page_size <= 0 || pages_per_seq <= 0 || D <= 0)
    return fail(PF_ERR_INVALID, "pf_paged_write: shapes must be positive");
  return cuda_status(launch_paged_write(k_pages, v_pages, k, v, block_tables, positions, dtype, B, Hkv,
                                        num_pages, page_size, pages_per_seq, D,
                                        static_cast<cudaStream_t>(stream)),
                     "pf_paged_write");
}

int pf_cache_write(void* k_cache, void* v_cache, const void* k, const void* v, int dtype, int B,
                   int Hkv, int C, int L, int D, int start, void* stream) {
  if (!valid_dtype(dtype) || !k_cache || !v_cache || !k || !v)
    return fail(PF_ERR_INVALID, "pf_cache_write: bad argument");
  if (B <= 0 || Hkv <= 0 || C <= 0 || L < 0 || D <= 0 || start < 0)
    return fail(PF_ERR_INVALID, "pf_cache_write: bad shape");
  if (L > C) return fail(PF_ERR_INVALID, "pf_cache_write: %d tokens do not fit a %d-slot cache", L, C);
  return cuda_status(launch_cache_write(k_cache, v_cache, k, v, dtype, B, Hkv, C, L, D, start,
                                        static_cast<cudaStream_t>(stream)),
                     "pf_cache_write");
}

int pf_paged_gather(const void* pages, const int32_t* block_tables, void* out, int dtype, int B,
                    int Hkv, int num_pages, int page_size, int pages_per_seq, int D, void* stream) {
  if (!valid_dtype(dtype) || !pages || !block_tables || !out)
    return fail(PF_ERR_INVALID, "pf_paged_gather: bad argument");
  if (B <= 0 || Hkv <= 0 || num_pages <= 0 || page_size <= 0 || pages_per_seq <= 0 || D <= 0)
    return fail(PF_ERR_INVALID, "pf_paged_gather: shapes must be positive");
  return cuda_status(launch_paged_gather(pages, block_tables, out, dtype, B, Hkv, num_pages, page_size,
                                         pages_per_seq, D, static_cast<cudaStream_t>(stream)),
                     "pf_paged_gather");
}

int pf_rope_apply(const void* x, const void* cos_t, const void* sin_t, int table_dtype, void* out, int dtype,
                  int B, int H, int S, int D, int inverse, void* stream) {
  if (!valid_dtype(dtype) || !valid_dtype(table_dtype) || !x || !cos_t || !sin_t || !out)
    return fail(PF_ERR_INVALID, "pf_rope_apply: bad argument");
  if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(PF_ERR_INVALID, "pf_rope_apply: shapes must be positive");
  if (D % 2 != 0) return fail(PF_ERR_INVALID, "pf_rope_apply: head_dim must be even for RoPE");
  return cuda_status(launch_rope_apply(x, cos_t, sin_t, table_dtype, out, dtype, (long)B * H * S, S, D,
                                       inverse != 0, static_cast<cudaStream_t>(stream)),
                     "pf_rope_apply");
}

int pf_add_rms_norm(const void* x, const void* residual, const void* weight, void* x_out, void* h, int dtype,
                    long rows, int dim, float eps, void* stream) {
  if (!valid_dtype(dtype) || !x || !weight || !h || (residual && !x_out))
    return fail(PF_ERR_INVALID, "pf_add_rms_norm: bad argument");
  if (rows < 0 || dim <= 0) return fail(PF_ERR_INVALID, "pf_add_rms_norm: shapes must be positive");
  if (!(eps >= 0.f)) return fail(PF_ERR_INVALID, "pf_add_rms_norm: eps must be >= 0");
  return cuda_status(launch_add_rms_norm(x, residual, weight, x_out, h, dtype, rows, dim, eps,
                                         static_cast<cudaStream_t>(stream)),
                     "pf_add_rms_norm");
}

int pf_rows_linear(const void* x, const void* norm_weight, float eps, const void* wt, const void* residual,
                   void* y, int dtype, int M, int K, int N, int mode, void* stream) {
  if (!valid_dtype(dtype) || !x || !wt || !y || (mode == 1 && !residual))
    return fail(PF_ERR_INVALID, "pf_rows_linear: bad argument");
  if (!(eps >= 0.f)) return fail(PF_ERR_INVALID, "pf_rows_linear: eps must be >= 0");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(wt) | reinterpret_cast<uintptr_t>(norm_weight)) & 15u)
    return fail(PF_ERR_INVALID, "pf_rows_linear: x, wt and norm_weight must be 16-byte aligned");
  if (!rows_linear_supported(dtype, M, K, N, mode))
    return fail(PF_ERR_UNSUPPORTED,
                "pf_rows_linear: needs bf16/f16, 1 <= M <= 16, K a multiple of 32 up to 2048, N a multiple of %d, "
                "mode 0-2 (got dtype %d, M %d, K %d, N %d, mode %d)",
                mode == 2 ? 16 : 32, dtype, M, K, N, mode);
  return cuda_status(launch_rows_linear(x, norm_weight, eps, wt, residual, y, dtype, M, K, N, mode,
                                        static_cast<cudaStream_t>(stream)),
                     "pf_rows_linear");
}

int pf_rows_linear_rope_write(const void* x, const void* norm_weight, float eps, const void* wt, void* q_out,
                              void* k_pages, void* v_pages, const void* cos_t, const void* sin_t, int table_dtype,
                              int table_rows, const int32_t* block_tables, const int32_t* positions,
                              const int32_t* rope_positions, int dtype, int B, int K, int H, int Hkv, int num_pages,
                              int page_size, int pages_per_seq, int D, void* stream) {
  const char* fn = "pf_rows_linear_rope_write";
  if (!valid_dtype(dtype) || !valid_dtype(table_dtype) || !x || !wt || !q_out || !k_pages || !v_pages || !cos_t ||
      !sin_t || !block_tables || !positions || !rope_positions)
    return fail(PF_ERR_INVALID, "%s: bad argument", fn);
  if (!(eps >= 0.f)) return fail(PF_ERR_INVALID, "%s: eps must be >= 0", fn);
  if (B <= 0 || H <= 0 || Hkv <= 0 || num_pages <= 0 || page_size <= 0 || pages_per_seq <= 0 || D <= 0 ||
      table_rows <= 0)
    return fail(PF_ERR_INVALID, "%s: shapes must be positive", fn);
  if (H % Hkv != 0) return fail(PF_ERR_INVALID, "%s: num_heads must be a multiple of num_kv_heads", fn);
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(wt) | reinterpret_cast<uintptr_t>(norm_weight)) & 15u)
    return fail(PF_ERR_INVALID, "%s: x, wt and norm_weight must be 16-byte aligned", fn);
  if (!rows_linear_rope_supported(dtype, B, K, H, Hkv, D))
    return fail(PF_ERR_UNSUPPORTED,
                "%s: needs bf16/f16, 1 <= B <= 16, K a multiple of 32 up to 2048, head_dim a multiple of 32 "
                "(got dtype %d, B %d, K %d, head_dim %d)", fn, dtype, B, K, D);
  return cuda_status(launch_rows_linear_rope_write(x, norm_weight, eps, wt, q_out, k_pages, v_pages, cos_t, sin_t,
                                                   table_dtype, table_rows, block_tables, positions, rope_positions,
                                                   dtype, B, K, H, Hkv, num_pages, page_size, pages_per_seq, D,
                                                   static_cast<cudaStream_t>(stream)),
                     fn);
}

int pf_silu_mul(const void* gate, const void* up, void* out, int dtype, long rows, int cols, long in_stride,
                void* stream) {
  if (!valid_dtype(dtype) || !gate || !up || !out) return fail(PF_ERR_INVALID, "pf_silu_mul: bad argument");
  if (rows < 0 || cols < 0 || in_stride < cols) return fail(PF_ERR_INVALID, "pf_silu_mul: bad shape");
  return cuda_status(launch_silu_mul(gate, up, out, dtype, rows, cols, in_stride, static_cast<cudaStream_t>(stream)),
                     "pf_silu_mul");
}

int pf_argmax_embed(const void* logits, long row_stride, int vocab, int rows, int64_t* token, const void* embed,
                    void* x, int dim, int dtype, void* stream) {
  if (!valid_dtype(dtype) || !logits || !token || (embed && !x))
    return fail(PF_ERR_INVALID, "pf_argmax_embed: bad argument");
  if (rows < 0 || vocab <= 0 || row_stride < vocab || (embed && dim <= 0))
    return fail(PF_ERR_INVALID, "pf_argmax_embed: bad shape");
  return cuda_status(launch_argmax_embed(logits, row_stride, vocab, rows, token, embed, x, dim, dtype,
                                         static_cast<cudaStream_t>(stream)),
                     "pf_argmax_embed");
}

int pf_decode_positions(int64_t* pos, int capacity, int32_t* slots, int32_t* lens, int32_t* rope_rows, int B,
                        void* stream) {
  if (!pos || !slots || !lens || !rope_rows) return fail(PF_ERR_INVALID, "pf_decode_positions: bad argument");
  if (capacity <= 0 || B <= 0) return fail(PF_ERR_INVALID, "pf_decode_positions: capacity and B must be positive");
  return cuda_status(launch_decode_positions(pos, capacity, slots, lens, rope_rows, B,
                                             static_cast<cudaStream_t>(stream)),
                     "pf_decode_positions");
}

int pf_rope_paged_write(void* q, void* k_pages, void* v_pages, const void* k, const void* v, const void* cos_t,
                        const void* sin_t, int table_dtype, int table_rows, const int32_t* block_tables,
                        const int32_t* positions, const int32_t* rope_positions, int dtype, int B, int H, int Hkv,
                        int num_pages, int page_size, int pages_per_seq, int D, void* stream) {
  if (!valid_dtype(dtype) || !valid_dtype(table_dtype) || !q || !k_pages || !v_pages || !k || !v || !cos_t ||
      !sin_t || !block_tables || !positions || !rope_positions)
    return fail(PF_ERR_INVALID, "pf_rope_paged_write: bad argument");
  if (B <= 0 || H <= 0 || Hkv <= 0 || num_pages <= 0 || page_size <= 0 || pages_per_seq <= 0 || D <= 0 ||
      table_rows <= 0)
    return fail(PF_ERR_INVALID, "pf_rope_paged_write: shapes must be positive");
  if (D % 2 != 0 || D > 1024) return fail(PF_ERR_INVALID, "pf_rope_paged_write: head_dim must be even and <= 1024");
  if (H % Hkv != 0) return fail(PF_ERR_INVALID, "pf_rope_paged_write: num_heads must be a multiple of num_kv_heads");
  return cuda_status(launch_rope_paged_write(q, (long)H * D, q, k_pages, v_pages, k, v, (long)Hkv * D, cos_t, sin_t,
                                             table_dtype, table_rows, block_tables, positions, rope_positions, dtype,
                                             B, H, Hkv, num_pages, page_size, pages_per_seq, D,
                                             static_cast<cudaStream_t>(stream)),
                     "pf_rope_paged_write");
}

int pf_rope_paged_write_qkv(const void* qkv, long row_stride, void* q_out, void* k_pages, void* v_pages,
                            const void* cos_t, const void* sin_t, int table_dtype, int table_rows,
                            const int32_t* block_tables, const int32_t* positions, const int32_t* rope_positions,
                            int dtype, int B, int H, int Hkv, int num_pages, int page_size, int pages_per_seq, int D,
                            void* stream) {
  if (!valid_dtype(dtype) || !valid_dtype(table_dtype) || !qkv || !q_out || !k_pages || !v_pages || !cos_t ||
      !sin_t || !block_tables || !positions || !rope_positions)
    return fail(PF_ERR_INVALID, "pf_rope_paged_write_qkv: bad argument");
  if (B <= 0 || H <= 0 || Hkv <= 0 || num_pages <= 0 || page_size <= 0 || pages_per_seq <= 0 || D <= 0 ||
      table_rows <= 0)
    return fail(PF_ERR_INVALID, "pf_rope_paged_write_qkv: shapes must be positive");
  if (D % 2 != 0 || D > 1024)
    return fail(PF_ERR_INVALID, "pf_rope_paged_write_qkv: head_dim must be even and <= 1024");
  if (H % Hkv != 0)
    return fail(PF_ERR_INVALID, "pf_rope_paged_write_qkv: num_heads must be a multiple of num_kv_heads");
  if (row_stride < (long)(H + 2 * Hkv) * D)
    return fail(PF_ERR_INVALID, "pf_rope_paged_write_qkv: row_stride %ld < (H + 2*Hkv) * D", row_stride);
  const size_t elt = dtype_size(dtype);
  const char* base = static_cast<const char*>(qkv);
  return cuda_status(launch_rope_paged_write(qkv, row_stride, q_out, k_pages, v_pages, base + (size_t)H * D * elt,
                                             base + (size_t)(H + Hkv) * D * elt, row_stride, cos_t, sin_t,
                                             table_dtype, table_rows, block_tables, positions, rope_positions, dtype,
                                             B, H, Hkv, num_pages, page_size, pages_per_seq, D,
                                             static_cast<cudaStream_t>(stream)),
                     "pf_rope_paged_write_qkv");
}

size_t pf_paged_prefill_workspace_size(int dtype, int B, int Hkv, int max_context_len, int D) {
  if (!valid_dtype(dtype) || B <= 0 || Hkv <= 0 || max_context_len <= 0 || D <= 0) return 0;
  const size_t plane = (size_t)B * Hkv * max_context_len * D * elem_bytes(dtype);
  const size_t aligned = (plane + 255) & ~(size_t)255;
  return 2 * aligned + (size_t)B * sizeof(int32_t);
}

int pf_paged_prefill(const void* q, const void* k_pages, const void* v_pages, const int32_t* block_tables,
                     const int32_t* context_lens, void* o, int dtype, int B, int H, int Hkv, int L, int num_pages,
                     int page_size, int pages_per_seq, int D, int max_context_len, float sm_scale,
                     void* workspace, size_t workspace_bytes, void* stream) {
  if (!valid_dtype(dtype) || !q || !k_pages || !v_pages || !block_tables || !context_lens || !o)
    return fail(PF_ERR_INVALID, "pf_paged_prefill: bad argument");
  if (B <= 0 || H <= 0 || Hkv <= 0 || L <= 0 || num_pages <= 0 || page_size <= 0 || pages_per_seq <= 0 || D <= 0 ||
      max_context_len <= 0)
    return fail(PF_ERR_INVALID, "pf_paged_prefill: shapes must be positive");
  if (H % Hkv != 0) return fail(PF_ERR_INVALID, "pf_paged_prefill: num_heads must be a multiple of num_kv_heads");
  const int row_bytes = D * (int)elem_bytes(dtype);
  if (row_bytes % 16 != 0)
    return fail(PF_ERR_UNSUPPORTED, "pf_paged_prefill: head_dim * element size must be a multiple of 16 bytes");
  const int T = max_context_len < pages_per_seq * page_size ? max_context_len : pages_per_seq * page_size;
  if ((long)T * (row_bytes / 16) >= (1l << 31))
    return fail(PF_ERR_UNSUPPORTED, "pf_paged_prefill: context of %d rows x %d bytes exceeds 2^31 16-byte words", T,
                row_bytes);
  const size_t need = pf_paged_prefill_workspace_size(dtype, B, Hkv, T, D);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    return fail(PF_ERR_WORKSPACE, "pf_paged_prefill: workspace of %zu bytes required, got %zu", need,
                workspace_bytes);
  const size_t plane = (((size_t)B * Hkv * T * row_bytes) + 255) & ~(size_t)255;
  char* ws = static_cast<char*>(workspace);
  int32_t* q_offs = reinterpret_cast<int32_t*>(ws + 2 * plane);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_paged_ctx_gather(k_pages, v_pages, block_tables, context_lens, ws, ws + plane, q_offs, L, B,
                                          Hkv, num_pages, page_size, pages_per_seq, T, row_bytes, st);
  if (e != cudaSuccess) return cuda_status(e, "pf_paged_prefill (gather)");
  FwdArgs a{};
  a.q = q; a.k = ws; a.v = ws + plane; a.o = o; a.lse = nullptr;
  a.dtype = dtype; a.B = B; a.H = H; a.Hkv = Hkv; a.Sq = L; a.Sk = T; a.D = D;
  a.causal = 1; a.kv_len = T; a.sm_scale = sm_scale;
  a.stream = st;
  a.kv_lens = context_lens; a.q_offs = q_offs;
  if (fwd_sm100_supported(dtype, D) && aligned16(q) && aligned16(o))
    return cuda_status(launch_fwd_sm100(a), "pf_paged_prefill (tcgen05)");
  return cuda_status(launch_fwd_simt(a), "pf_paged_prefill (simt)");
}

}  // extern "C"
