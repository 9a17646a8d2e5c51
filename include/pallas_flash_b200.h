/*
 * pallas_flash_b200.h -- C ABI of libpallas_flash_b200.so, the sm_100a (B200)
 * attention kernels behind the pallas_flash Python API.
 *
 * Every entry point takes raw device pointers, plain integer shapes, scalars
 * and the CUDA stream to launch on.  Nothing here allocates device memory:
 * where a kernel needs scratch space (split-KV partials, the dQ accumulator)
 * the caller passes a workspace and asks for its size first with the matching
 * *_workspace_size function.  All tensors are dense row-major with the
 * shapes stated below (the layouts of the reference's jax.Array operands).
 *
 * Return value: PF_OK (0) or one of the PF_ERR_* codes; pf_last_error()
 * returns a static, human readable message for the most recent failure on
 * the calling thread.
 *
 * Reference interfaces replaced (paths inside aabhimittal/TPU-Native-Pallas-
 * FlashAttention):
 *   pf_fwd              src/pallas_flash/flash_attention.py:162-227  (_flash_attention_call)
 *   pf_bwd_preprocess   src/pallas_flash/flash_attention.py:363-365  (delta)
 *   pf_bwd_dq           src/pallas_flash/flash_attention.py:276-311,379-398
 *   pf_bwd_dkv          src/pallas_flash/flash_attention.py:314-351,403-436 (+ group_sum)
 *   pf_bwd              src/pallas_flash/flash_attention.py:354-442  (_flash_attention_bwd_call)
 *   pf_decode           src/pallas_flash/flash_attention.py:555-589  (flash_attention_decode)
 *   pf_rope_fwd         src/pallas_flash/fused_rope.py:116-213       (flash_attention_rope)
 *   pf_paged_decode     src/pallas_flash/paged.py:102-192            (paged_flash_attention)
 *   pf_paged_write      src/pallas_flash/paged.py:205-223            (write_to_paged_cache)
 *   pf_cache_write      src/pallas_flash/model.py:257-262,446-449    (_cache_write / ring slots)
 *   pf_paged_gather     src/pallas_flash/paged.py:158-159            (the block-table index map)
 *   pf_rope_paged_write src/pallas_flash/model.py:338-342 + paged.py:205-223 (RoPE of the decode
 *                       token's q/k fused with the k/v page write)
 *   pf_rope_paged_write_qkv  the same, reading q/k/v from one fused projection row
 *                       (model.py:80-88 project_qkv as a single matmul)
 *   pf_paged_prefill    extension of src/pallas_flash/paged.py:102-192 to an L-query chunk
 *                       (the reference pages single-query decode only)
 *   pf_rope_apply       src/pallas_flash/fused_rope.py:43-50, model.py:41-67 (apply_rope; and its
 *                       inverse, for the gradient of the RoPE-fused attention)
 *   pf_add_rms_norm     src/pallas_flash/model.py:34-38 (rms_norm) + the residual add before it
 *   pf_silu_mul         src/pallas_flash/model.py:70-74 (the silu(gate) * up of swiglu_mlp)
 *   pf_rows_linear      src/pallas_flash/model.py:90-101, 120-124, 70-74, 307-356 (a decode
 *                       step's x @ W projections with the rms_norm before them, the residual
 *                       add after them, or the SwiGLU activation between them)
 *   pf_rows_linear_rope_write  the same step's q/k/v projection (model.py:90-101) with
 *                       rope (model.py:41-67) and the cache write (model.py:307-356,
 *                       paged.py:205-223) as its epilogue
 *   pf_decode_positions src/pallas_flash/model.py:434-449, 475-476 (slot, kv_len and RoPE row
 *                       of a decode step, computed on the device)
 *   pf_argmax_embed     src/pallas_flash/model.py:377-383, 520-528 (greedy argmax) + :333, 478
 *                       (the next step's embedding lookup)
 */
#ifndef PALLAS_FLASH_B200_H_
#define PALLAS_FLASH_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of q/k/v/o and of the cos/sin tables. */
enum pf_dtype { PF_F32 = 0, PF_BF16 = 1, PF_F16 = 2 };

/* Status codes. */
enum pf_status {
  PF_OK = 0,
  PF_ERR_INVALID = 1,     /* bad shape / argument: the reference raises ValueError */
  PF_ERR_UNSUPPORTED = 2, /* valid request this build has no kernel for           */
  PF_ERR_CUDA = 3,        /* a CUDA runtime / driver call failed                   */
  PF_ERR_DEVICE = 4,      /* a kernel recorded a device-side status (see below)    */
  PF_ERR_WORKSPACE = 5    /* workspace pointer missing or too small                */
};

/* Device-side status bits, accumulated in a per-device word by the kernels
 * instead of trapping; read (and optionally clear) with pf_device_status. */
enum pf_device_bits {
  PF_DEV_WAIT_TIMEOUT = 1, /* a bounded mbarrier wait gave up                     */
  PF_DEV_BAD_PAGE = 2,     /* a block-table entry was outside [0, num_pages)      */
  PF_DEV_SMEM_LAYOUT = 4,  /* dynamic shared memory was not 1024-byte aligned     */
  PF_DEV_LEN_OVER_MAX = 8  /* a context length exceeded the call's max_context_len:
                              keys past the planned splits were not attended     */
};

const char* pf_last_error(void);
/* Library version string, e.g. "0.1.0+sm100a". */
const char* pf_version(void);
/* Reads the device status word of the current device (synchronises the
 * device); clears it when reset != 0. */
int pf_device_status(int* bits_out, int reset);
/* Sets the wall-time bound of every bounded in-kernel wait (mbarrier phases
 * of the TMA/tcgen05 pipelines), in ns, on the current device; 0 restores the
 * 2 s default.  A wait that runs out records PF_DEV_WAIT_TIMEOUT and its
 * kernel returns.  No counterpart in the reference (its Pallas kernels have no
 * device-side waits); provided so the timeout path can be tested. */
int pf_set_wait_limit_ns(unsigned long long ns);
/* Launches one CTA that waits on an mbarrier nothing arrives on: after the
 * wait limit it records PF_DEV_WAIT_TIMEOUT and returns.  A self-test of the
 * timeout path (no counterpart in the reference). */
int pf_selftest_wait_timeout(void* stream);
/* Which forward kernel family pf_fwd would use for these arguments:
 * 1 = tcgen05/TMEM tensor-core kernel, 0 = fp32 SIMT kernel. */
int pf_fwd_kernel_kind(int dtype, int head_dim);

/* ---------------------------------------------------------------------------
 * Prefill forward with saved log-sum-exp.
 *   q   [B, H,   Sq, D]   k, v [B, Hkv, Sk, D]   o [B, H, Sq, D] (dtype of q)
 *   lse [B, H, Sq] float32 (the reference's [B,H,Sq,1]); may be NULL.
 * H % Hkv == 0 (query head h reads kv head h / (H/Hkv)).  Keys at positions
 * >= kv_len (1 <= kv_len <= Sk) are masked and never read; causal applies
 * q_pos >= k_pos with both sequences aligned at position 0.  Rows with no
 * visible key give o = 0 and lse = 0.
 * ------------------------------------------------------------------------- */
int pf_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
           int dtype, int B, int H, int Hkv, int Sq, int Sk, int D,
           int causal, float sm_scale, int kv_len, void* stream);

/* Forward with RoPE fused in: q and k are rotated with x*cos +
 * rotate_half(x)*sin, q by rows of (q_cos, q_sin) [Sq, D] and k by rows of
 * (k_cos, k_sin) [Sk, D] (table dtype tbl_dtype).  No lse output.  On the
 * tensor-core path each query tile is rotated once in shared memory and each
 * key row once into the workspace (pf_rope_fwd_workspace_size bytes; 0 for
 * the fp32 path, which rotates both operands as it loads them). */
size_t pf_rope_fwd_workspace_size(int dtype, int B, int Hkv, int Sk, int D);
int pf_rope_fwd(const void* q, const void* k, const void* v,
                const void* q_cos, const void* q_sin,
                const void* k_cos, const void* k_sin, int tbl_dtype,
                void* o, int dtype, int B, int H, int Hkv, int Sq, int Sk,
                int D, int causal, float sm_scale, int kv_len,
                void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Backward.  delta [B,H,Sq] f32 = sum_d o*do.
 * dq like q, dk/dv like k/v (already summed over each GQA group).
 * ------------------------------------------------------------------------- */
int pf_bwd_preprocess(const void* o, const void* dout, float* delta,
                      int dtype, int B, int H, int Sq, int D, void* stream);

int pf_bwd_dq(const void* q, const void* k, const void* v, const void* dout,
              const float* lse, const float* delta, void* dq,
              int dtype, int B, int H, int Hkv, int Sq, int Sk, int D,
              int causal, float sm_scale, int kv_len, void* stream);

int pf_bwd_dkv(const void* q, const void* k, const void* v, const void* dout,
               const float* lse, const float* delta, void* dk, void* dv,
               int dtype, int B, int H, int Hkv, int Sq, int Sk, int D,
               int causal, float sm_scale, int kv_len, void* stream);

/* Whole backward (preprocess + dQ + dK/dV) in one call.  The workspace holds
 * delta (B*H*Sq f32) and, on the tensor-core path, the dS spill: every 16-bit
 * 128 x 128 dS tile the dK/dV kernel computes, from which dQ is one GEMM per
 * query tile instead of a kernel that recomputes S and dP.
 * For problems with fewer key tiles (B*Hkv*ceil(Sk/128)) than the device has
 * SMs, the dK/dV kernel splits each kv group's q heads over
 * pf_bwd_head_parts() CTAs per key tile; the workspace then also holds their
 * f32 partial dK/dV (summed in a fixed order, so results stay deterministic).
 * pf_bwd_workspace_size returns the size with the spill and the partials (for
 * these causal / kv_len arguments; kv_len <= 0 means Sk); pf_bwd accepts any
 * workspace of at least the delta size, recomputes when the spill does not
 * fit and does not split when the partials do not. */
size_t pf_bwd_workspace_size(int dtype, int B, int H, int Hkv, int Sq, int Sk,
                             int D, int causal, int kv_len);
/* q-head parts per key tile of that split on the current device (1: none).
 * No reference counterpart: the Pallas grid has no analogue of this
 * small-problem load balancing. */
int pf_bwd_head_parts(int B, int H, int Hkv, int Sk);
int pf_bwd(const void* q, const void* k, const void* v, const void* o,
           const void* dout, const float* lse, void* dq, void* dk, void* dv,
           int dtype, int B, int H, int Hkv, int Sq, int Sk, int D,
           int causal, float sm_scale, int kv_len,
           void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Single-query decode over a fixed-capacity cache.
 *   q [B, H, 1, D]   k_cache, v_cache [B, Hkv, C, D]   o [B, H, 1, D]
 * Attends cache positions [0, cache_len) (1 <= cache_len <= C); cache_len is
 * a runtime scalar.  Split-KV: partial results go to the workspace.
 * ------------------------------------------------------------------------- */
size_t pf_decode_workspace_size(int B, int H, int Hkv, int C, int D);
int pf_decode(const void* q, const void* k_cache, const void* v_cache, void* o,
              int dtype, int B, int H, int Hkv, int C, int D, int cache_len,
              float sm_scale, void* workspace, size_t workspace_bytes,
              void* stream);

/* ---------------------------------------------------------------------------
 * Paged decode.
 *   q [B, H, 1, D]   k_pages, v_pages [num_pages, Hkv, page_size, D]
 *   block_tables [B, pages_per_seq] int32   context_lens [B] int32 (device)
 * Logical page p of sequence b lives in physical page block_tables[b, p];
 * positions >= context_lens[b] are masked and their pages never read.
 * max_context_len bounds context_lens (it sizes the split grid); pass
 * pages_per_seq * page_size when unknown.
 * ------------------------------------------------------------------------- */
size_t pf_paged_decode_workspace_size(int B, int H, int Hkv, int page_size,
                                      int max_context_len, int D);
int pf_paged_decode(const void* q, const void* k_pages, const void* v_pages,
                    const int32_t* block_tables, const int32_t* context_lens,
                    void* o, int dtype, int B, int H, int Hkv, int num_pages,
                    int page_size, int pages_per_seq, int D,
                    int max_context_len, float sm_scale, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Paged decode without a caller workspace.  No counterpart in the reference:
 * it exists for callers that cannot allocate device memory (a host that
 * manages device memory as fixed arenas, or a call site handed only its
 * input and output buffers, where cudaMalloc -- which also synchronises the
 * device -- is not allowed).  Same arguments and results as pf_paged_decode;
 * the split-KV scratch is a fixed 16 MiB __device__ array inside the library
 * (held by every GPU that loads it until exit).  The first call on a device
 * resolves that array's address; make it before any stream capture.  Calls
 * that overlap on the GPU race on the shared scratch.  Requests needing more
 * than 16 MiB of partials even at one split per sequence (B*H*(D+2)*4 bytes)
 * return PF_ERR_WORKSPACE. */
int pf_paged_decode_noalloc(const void* q, const void* k_pages, const void* v_pages,
                            const int32_t* block_tables, const int32_t* context_lens,
                            void* o, int dtype, int B, int H, int Hkv, int num_pages,
                            int page_size, int pages_per_seq, int D,
                            int max_context_len, float sm_scale, void* stream);

/* ---------------------------------------------------------------------------
 * Cache bookkeeping.
 * pf_paged_write: for each sequence b of the batch, write one token's k/v
 *   ([B, Hkv, 1, D] each) into page block_tables[b, positions[b] / page_size]
 *   at offset positions[b] % page_size.  A physical page index outside
 *   [0, num_pages) is clamped, as jax.lax.dynamic_update_slice clamps.
 * pf_cache_write: write L tokens k/v [B, Hkv, L, D] into cache slots
 *   (start + i) % C of k_cache/v_cache [B, Hkv, C, D] (a fixed cache when
 *   start + L <= C, a ring buffer otherwise).
 * pf_paged_gather: out[b, h, t, :] = pages[block_tables[b, t / ps], h,
 *   t % ps, :] for t < pages_per_seq * ps (byte-exact copy; debug/oracle aid).
 * ------------------------------------------------------------------------- */
int pf_paged_write(void* k_pages, void* v_pages, const void* k, const void* v,
                   const int32_t* block_tables, const int32_t* positions,
                   int dtype, int B, int Hkv, int num_pages, int page_size,
                   int pages_per_seq, int D, void* stream);

int pf_cache_write(void* k_cache, void* v_cache, const void* k, const void* v,
                   int dtype, int B, int Hkv, int C, int L, int D, int start,
                   void* stream);

int pf_paged_gather(const void* pages, const int32_t* block_tables, void* out,
                    int dtype, int B, int Hkv, int num_pages, int page_size,
                    int pages_per_seq, int D, void* stream);

/* pf_paged_prefill: chunked prefill over a page pool.  q [B, H, L, D] holds the
 *   last L positions of every sequence (query row i of sequence b sits at
 *   position context_lens[b] - L + i; its k/v are already in the pages) and
 *   attends causally to keys [0, position] of its own context, read through
 *   block_tables as in pf_paged_decode; out like q.  The contexts are first
 *   gathered into the workspace (pf_paged_prefill_workspace_size bytes,
 *   16-byte aligned; max_context_len bounds context_lens), then the prefill
 *   kernels run with per-sequence lengths and causal offsets.  Requires
 *   D * element size to be a multiple of 16 bytes.
 */
size_t pf_paged_prefill_workspace_size(int dtype, int B, int Hkv, int max_context_len, int D);
int pf_paged_prefill(const void* q, const void* k_pages, const void* v_pages,
                     const int32_t* block_tables, const int32_t* context_lens, void* out,
                     int dtype, int B, int H, int Hkv, int L, int num_pages, int page_size,
                     int pages_per_seq, int D, int max_context_len, float sm_scale,
                     void* workspace, size_t workspace_bytes, void* stream);

/* pf_rope_paged_write: the step before decode attention, for one token per
 *   sequence: q [B, H, 1, D] is rotated in place and k [B, Hkv, 1, D] rotated,
 *   both at row rope_positions[b] of the [table_rows, D] cos/sin tables
 *   (clamped into range), then rotated k and v are written like
 *   pf_paged_write at slot positions[b] (for a ring cache the slot differs
 *   from the rotation position).  Rotation in fp32, one rounding.
 */
int pf_rope_paged_write(void* q, void* k_pages, void* v_pages, const void* k,
                        const void* v, const void* cos, const void* sin,
                        int table_dtype, int table_rows, const int32_t* block_tables,
                        const int32_t* positions, const int32_t* rope_positions,
                        int dtype, int B, int H, int Hkv, int num_pages, int page_size,
                        int pages_per_seq, int D, void* stream);

/* pf_rope_paged_write_qkv: pf_rope_paged_write on the output of one fused
 *   q/k/v projection: row b of qkv (row_stride elements apart, >= (H+2*Hkv)*D)
 *   holds sequence b's H query heads, then its Hkv key heads, then its Hkv
 *   value heads, D elements each.  Rotated q goes to q_out [B, H, 1, D]
 *   (contiguous, not aliasing qkv); rotated k and v go to the pages as above.
 */
int pf_rope_paged_write_qkv(const void* qkv, long row_stride, void* q_out, void* k_pages,
                            void* v_pages, const void* cos, const void* sin, int table_dtype,
                            int table_rows, const int32_t* block_tables, const int32_t* positions,
                            const int32_t* rope_positions, int dtype, int B, int H, int Hkv,
                            int num_pages, int page_size, int pages_per_seq, int D, void* stream);

/* ---------------------------------------------------------------------------
 * Rotary embedding.
 * pf_rope_apply: out = x*cos + rotate_half(x)*sin over rows x[B, H, S, D]
 *   (rotate_half([x1, x2]) = [-x2, x1]); row s of the [S, D] cos/sin tables
 *   (table_dtype) belongs to position s.  inverse != 0 applies the transpose
 *   (sin negated): the gradient map of the rotation.  fp32 arithmetic; out may
 *   alias x.  D must be even.
 * ------------------------------------------------------------------------- */
int pf_rope_apply(const void* x, const void* cos, const void* sin, int table_dtype,
                  void* out, int dtype, int B, int H, int S, int D, int inverse,
                  void* stream);

/* ---------------------------------------------------------------------------
 * Decoder-block elementwise steps (the tiny-LLaMA decode step is a chain of
 * small launches at batch 16; these fold ~8 launches per norm into one).
 * pf_add_rms_norm: x' = x + residual (rounded to dtype; written to x_out, which
 *   may alias x; skipped when residual is NULL, x_out then unused), then
 *   h = (x' * rsqrt(mean(x'^2) + eps)) * weight over `rows` rows of `dim`.
 *   Replaces rms_norm (src/pallas_flash/model.py:34-38) and the residual add
 *   before it (model.py:120-124, 298-301).  fp32 arithmetic; roundings where
 *   the unfused expression rounds.
 * pf_silu_mul: out[r, c] = silu(gate[r, c]) * up[r, c] over rows x cols, silu
 *   rounded to dtype before the product -- the activation of swiglu_mlp
 *   (model.py:70-74).  gate/up rows are in_stride elements apart (>= cols), so
 *   both halves of one fused [rows, 2*cols] projection can be passed; out is
 *   contiguous [rows, cols].
 * pf_decode_positions: for a decode step at p = *pos (int64, device), writes
 *   slots[b] = p % capacity, lens[b] = min(p + 1, capacity), rope_rows[b] = p
 *   for b < B, then *pos = p + 1 -- the per-step slot / live-length / RoPE-row
 *   arithmetic of model.py:434-449, 475-476, on the device so that one
 *   captured decode step serves every position.
 * ------------------------------------------------------------------------- */
int pf_add_rms_norm(const void* x, const void* residual, const void* weight,
                    void* x_out, void* h, int dtype, long rows, int dim, float eps,
                    void* stream);
int pf_silu_mul(const void* gate, const void* up, void* out, int dtype, long rows,
                int cols, long in_stride, void* stream);
/* pf_rows_linear: y = epilogue(prologue(x) @ W) for 1 <= M <= 16 rows (a
 *   decode step's batch), bf16 or f16.  x is [M, K] (16-byte aligned, K a
 *   multiple of 32, at most 2048); W is passed transposed, wt = W^T [N_w, K]
 *   row-major.  Prologue: when norm_weight ([K]) is not NULL each row is
 *   replaced by round((x * rsqrt(mean(x^2) + eps)) * norm_weight), the output
 *   of pf_add_rms_norm without a residual.  Epilogue by `mode`:
 *     0: y[M, N] = round(x W)                                  (N_w = N)
 *     1: y[M, N] = round(residual + round(x W)); residual [M, N] may alias y
 *     2: y[M, N] = round(round(silu(round(g))) * round(u)) with g = x W[:, :N],
 *        u = x W[:, N:2N] (N_w = 2N) -- pf_silu_mul of the fused projection.
 *   N must be a multiple of 32 (16 in mode 2).  fp32 accumulation; the sum
 *   over K is done in a fixed order (deterministic).  Replaces the matmul and
 *   its neighbouring pf_add_rms_norm / pf_silu_mul launches of a decode step
 *   (src/pallas_flash/model.py:90-101, 120-124, 70-74 as called by
 *   decode_step, :307-356).  PF_ERR_UNSUPPORTED outside those shapes.
 */
int pf_rows_linear(const void* x, const void* norm_weight, float eps, const void* wt,
                   const void* residual, void* y, int dtype, int M, int K, int N, int mode,
                   void* stream);
/* pf_rows_linear_rope_write: one decode token per sequence through the fused
 *   q/k/v projection, RoPE and the K/V cache write, in one launch.  The
 *   projection is pf_rows_linear mode 0 (M = B rows of x [B, K], optional
 *   RMSNorm prologue) with wt = [W_q | W_k | W_v]^T [(H + 2*Hkv) * D, K]; its
 *   rounded output then goes exactly where pf_rope_paged_write_qkv sends a
 *   [B, (H + 2*Hkv) * D] projection: q heads rotated into q_out [B, H, 1, D],
 *   k heads rotated and v heads copied into page
 *   block_tables[b][positions[b] / page_size], row positions[b] % page_size,
 *   with the RoPE table row rope_positions[b] (clamped to the table).  head_dim
 *   must be a multiple of 32; other limits as pf_rows_linear.
 */
int pf_rows_linear_rope_write(const void* x, const void* norm_weight, float eps, const void* wt,
                              void* q_out, void* k_pages, void* v_pages, const void* cos_t,
                              const void* sin_t, int table_dtype, int table_rows,
                              const int32_t* block_tables, const int32_t* positions,
                              const int32_t* rope_positions, int dtype, int B, int K, int H,
                              int Hkv, int num_pages, int page_size, int pages_per_seq, int D,
                              void* stream);
int pf_decode_positions(int64_t* pos, int capacity, int32_t* slots, int32_t* lens,
                        int32_t* rope_rows, int B, void* stream);
/* pf_argmax_embed: the end of a greedy decode step.  For each of `rows` rows of
 *   logits (row_stride elements apart, `vocab` used): token[b] (int64) = the
 *   first index of the row's maximum, a NaN ranking above every number (the
 *   argmax rule of jnp.argmax at model.py:377-383, 520-528); then, when embed
 *   [vocab_rows, dim] is not NULL, x[b, :] = embed[token[b], :], the next
 *   step's input (the embedding lookup of model.py:333, 478).
 */
int pf_argmax_embed(const void* logits, long row_stride, int vocab, int rows, int64_t* token,
                    const void* embed, void* x, int dim, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PALLAS_FLASH_B200_H_ */
