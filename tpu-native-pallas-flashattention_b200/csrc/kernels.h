// kernels.h -- internal launch interface between the C ABI (capi.cu) and the
// kernel translation units.  Not part of the public ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace pf {

struct FwdArgs {
  const void *q, *k, *v;
  void* o;
  float* lse;  // may be null
  int dtype, B, H, Hkv, Sq, Sk, D, causal, kv_len;
  float sm_scale;
  // fused RoPE tables (all null when RoPE is off)
  const void *q_cos, *q_sin, *k_cos, *k_sin;
  int tbl_dtype;
  cudaStream_t stream;
  // Optional per-sequence key lengths (clamped to kv_len, which stays the
  // extent of the K/V tensors) and causal query offsets: with them, query row
  // i of sequence b sits at position q_offs[b] + i and sees keys
  // [0, min(kv_lens[b], q_offs[b] + i]) (the chunked-prefill mask).  Null: the
  // scalar kv_len and offset 0 (both sequences aligned at 0).
  const int32_t* kv_lens;
  const int32_t* q_offs;
};

struct BwdArgs {
  const void *q, *k, *v, *dout;
  const float *lse, *delta;
  void *dq, *dk, *dv;
  int dtype, B, H, Hkv, Sq, Sk, D, causal, kv_len;
  float sm_scale;
  float* dq_accum;  // f32 [B,H,Sq,D] scratch (tensor-core path)
  uint16_t* ds_buf;  // dS spill of the dK/dV kernel for the dQ GEMM (null: not written)
  int dq_ctas;       // CTAs of the persistent dQ GEMM (0: one per SM)
  float* dkv_part;   // head-split f32 partial dK/dV (null: no split)
  int head_parts;    // q-head parts per key tile when dkv_part is set
  cudaStream_t stream;
};

// Split-KV decode over a page source.  A fixed cache is described as pages of
// `page_size` rows with an implicit identity table (block_tables == null):
// page p of sequence b is rows [p*ps, (p+1)*ps) of cache (b, hkv).
struct DecodeArgs {
  const void* q;
  const void *k_src, *v_src;
  const int32_t* block_tables;   // null -> fixed cache
  const int32_t* context_lens;   // null -> every sequence has `fixed_len`
  int fixed_len;
  void* o;
  int dtype, B, H, Hkv, D;
  int num_pages, page_size, pages_per_seq;  // pages: source [num_pages, Hkv, ps, D]
  long cache_rows;                          // fixed cache capacity C
  int max_len;                              // upper bound of the lengths
  float sm_scale;
  float* partial;   // workspace: [B, H, num_splits, D + 2] f32
  int num_splits, split_len;
  cudaStream_t stream;
};

cudaError_t launch_fwd_simt(const FwdArgs& a);
cudaError_t launch_bwd_dq_simt(const BwdArgs& a);
cudaError_t launch_bwd_dkv_simt(const BwdArgs& a);
cudaError_t launch_bwd_preprocess(const void* o, const void* dout, float* delta, int dtype,
                                  long rows, int D, cudaStream_t stream);

// tcgen05 tensor-core forward (bf16/f16, D in {64, 128}).
bool fwd_sm100_supported(int dtype, int D);
cudaError_t launch_fwd_sm100(const FwdArgs& a);
// Fused-RoPE forward: Q rotated in shared memory, K rotated once per row into
// k_rot (rope_fwd_sm100_workspace bytes) and streamed from there.
size_t rope_fwd_sm100_workspace(int dtype, int B, int Hkv, int Sk, int D);
cudaError_t launch_rope_fwd_sm100(const FwdArgs& a, void* k_rot);

// tcgen05 tensor-core backward (same dtypes / head dims as the forward).
bool bwd_sm100_supported(int dtype, int D);
cudaError_t launch_bwd_dkv_sm100(const BwdArgs& a);
// Bytes of the dS spill (16-bit 128 x 128 tiles of every live key/query tile pair).
size_t bwd_ds_spill_bytes(int B, int H, int Sq, int kv_len, int causal);
// q-head parts per key tile of the tensor-core dK/dV kernel (1: no split):
// doubled while the grid has fewer CTAs than SMs and the group divides.
int bwd_dkv_head_parts(int B, int H, int Hkv, int Sk);
// f32 partial dK/dV bytes of a head split into `parts` (0 when parts == 1).
size_t bwd_dkv_part_bytes(int B, int Hkv, int Sk, int D, int parts);
// dQ as one GEMM over the spilled dS tiles (after launch_bwd_dkv_sm100 with ds_buf set).
cudaError_t launch_bwd_dq_gemm_sm100(const BwdArgs& a);
cudaError_t launch_bwd_dq_sm100(const BwdArgs& a);

// Split-KV decode.
void decode_plan(int max_len, int B, int Hkv, int* num_splits, int* split_len);
bool decode_supported(int D);
cudaError_t launch_decode(const DecodeArgs& a);
cudaError_t launch_decode_combine(const DecodeArgs& a);
// Tensor-core decode (bf16/f16, D 64/128); launch_decode dispatches to it.
bool decode_tc_supported(int dtype, int D, int page_size, bool paged, long rows);
cudaError_t launch_decode_tc(const DecodeArgs& a);

cudaError_t launch_paged_write(void* k_pages, void* v_pages, const void* k, const void* v,
                               const int32_t* block_tables, const int32_t* positions, int dtype,
                               int B, int Hkv, int num_pages, int page_size, int pages_per_seq,
                               int D, cudaStream_t stream);
cudaError_t launch_cache_write(void* k_cache, void* v_cache, const void* k, const void* v,
                               int dtype, int B, int Hkv, int C, int L, int D, int start,
                               cudaStream_t stream);
cudaError_t launch_add_rms_norm(const void* x, const void* res, const void* w, void* x_out, void* h, int dtype,
                                long rows, int dim, float eps, cudaStream_t st);
cudaError_t launch_silu_mul(const void* g, const void* u, void* out, int dtype, long rows, int cols, long in_stride,
                            cudaStream_t st);
// Projection of <= 16 rows with an optional RMSNorm prologue and a plain /
// residual-add / SwiGLU epilogue (rows_linear.cu).
bool rows_linear_supported(int dtype, int M, int K, int N, int mode);
size_t rows_linear_smem(int K);
cudaError_t launch_rows_linear(const void* x, const void* norm_w, float eps, const void* wt, const void* res, void* y,
                               int dtype, int M, int K, int N, int mode, cudaStream_t st);
bool rows_linear_rope_supported(int dtype, int M, int K, int H, int Hkv, int D);
cudaError_t launch_rows_linear_rope_write(const void* x, const void* norm_w, float eps, const void* wt, void* q_out,
                                          void* k_pages, void* v_pages, const void* cos_t, const void* sin_t,
                                          int tdtype, int table_rows, const int32_t* tables,
                                          const int32_t* positions, const int32_t* rope_pos, int dtype, int M, int K,
                                          int H, int Hkv, int num_pages, int page_size, int pages_per_seq, int D,
                                          cudaStream_t st);
cudaError_t launch_argmax_embed(const void* logits, long row_stride, int vocab, int rows, int64_t* token,
                                const void* embed, void* x, int dim, int dtype, cudaStream_t st);
cudaError_t launch_decode_positions(int64_t* pos, int C, int32_t* slots, int32_t* lens, int32_t* rope_rows, int B,
                                    cudaStream_t st);
cudaError_t launch_rope_apply(const void* x, const void* cos_t, const void* sin_t, int tdtype, void* out, int dtype,
                              long rows, int S, int D, bool inverse, cudaStream_t st);
cudaError_t launch_rope_paged_write(const void* q_in, long q_bs, void* q_out, void* k_pages, void* v_pages,
                                    const void* k, const void* v, long kv_bs, const void* cos_t, const void* sin_t,
                                    int tdtype, int table_rows, const int32_t* block_tables,
                                    const int32_t* positions, const int32_t* rope_pos, int dtype, int B, int H,
                                    int Hkv, int num_pages, int page_size, int pages_per_seq, int D,
                                    cudaStream_t stream);
cudaError_t launch_paged_ctx_gather(const void* k_pages, const void* v_pages, const int32_t* block_tables,
                                    const int32_t* context_lens, void* kout, void* vout, int32_t* q_offs, int L,
                                    int B, int Hkv, int num_pages, int page_size, int pages_per_seq, int T,
                                    int row_bytes, cudaStream_t stream);
cudaError_t launch_paged_gather(const void* pages, const int32_t* block_tables, void* out,
                                int dtype, int B, int Hkv, int num_pages, int page_size,
                                int pages_per_seq, int D, cudaStream_t stream);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device):
// later launches -- including ones recorded into a CUDA graph -- skip the call.
cudaError_t set_smem_once(const void* kernel, int bytes);
template <typename K>
inline cudaError_t ensure_smem(K kernel, int bytes) {
  return set_smem_once(reinterpret_cast<const void*>(kernel), bytes);
}

// Streaming multiprocessors of the current device (cached per device): the
// grid size of the persistent kernels.
int sm_count();

// Records the message returned by pf_last_error() and returns `code`.
int set_last_error(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

inline int dtype_size(int dtype) { return dtype == 0 ? 4 : 2; }

}  // namespace pf
