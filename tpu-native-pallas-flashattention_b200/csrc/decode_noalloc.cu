// decode_noalloc.cu -- paged decode for callers that cannot allocate device memory.
//
// pf_paged_decode needs a scratch buffer for its split-KV partial results and
// asks the caller for it.  Some callers have no way to provide one: a C host
// that embeds this library and manages device memory as fixed arenas, or a
// plugin-style call site that is handed only its declared input and output
// buffers and may not call cudaMalloc (which also synchronises the device).
// pf_paged_decode_noalloc serves them: its scratch is a file-scope __device__
// array of kNoallocScratchBytes that every GPU which loads the library holds
// until the process exits.  The caller still passes q, the page pools, the
// tables, the lengths and the output.
//
// Host code never hands the array's name to a kernel (in host code it is only
// a stand-in symbol, not a device address).  The first call on each device
// resolves the real address with cudaGetSymbolAddress while that device is
// current, checks the result and caches it for the life of the process; that
// first call should come before any stream capture.  A cudaDeviceReset (or any
// other teardown of the primary context) reloads the module and can move the
// array, so a process that resets a device must not call this entry point
// again on that device.  All calls share the one array and nothing in it
// needs clearing (every partial the combine step reads is written earlier in
// the same call), but calls that overlap on the GPU -- e.g. on two streams of
// one device -- race on it.  Requests whose partials cannot fit even with a
// single split per sequence are rejected with PF_ERR_WORKSPACE.
#include <climits>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace pf {
namespace {

constexpr size_t kNoallocScratchBytes = 16u << 20;  // 16 MiB per device
constexpr int kMaxDevices = 64;
constexpr int kQuantum = 128;  // split lengths are multiples of this (as in decode.cu)

static __device__ __align__(256) float g_noalloc_scratch[kNoallocScratchBytes / sizeof(float)];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (set up once per device).
cudaError_t scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace pf

using namespace pf;

extern "C" int pf_paged_decode_noalloc(const void* q, const void* k_pages, const void* v_pages,
                                       const int32_t* block_tables, const int32_t* context_lens,
                                       void* o, int dtype, int B, int H, int Hkv, int num_pages,
                                       int page_size, int pages_per_seq, int D,
                                       int max_context_len, float sm_scale, void* stream) {
  const char* fn = "pf_paged_decode_noalloc";
  if (!(dtype == PF_F32 || dtype == PF_BF16 || dtype == PF_F16))
    return set_last_error(PF_ERR_INVALID, "%s: unknown dtype %d", fn, dtype);
  if (!q || !k_pages || !v_pages || !block_tables || !context_lens || !o)
    return set_last_error(PF_ERR_INVALID, "%s: null argument", fn);
  if (B <= 0 || H <= 0 || D <= 0 || num_pages <= 0 || page_size <= 0 || pages_per_seq <= 0)
    return set_last_error(PF_ERR_INVALID, "%s: shapes must be positive", fn);
  if (Hkv <= 0 || H % Hkv != 0)
    return set_last_error(PF_ERR_INVALID, "%s: num_heads (%d) must be a multiple of num_kv_heads (%d)", fn, H,
                          Hkv);
  if (!decode_supported(D))
    return set_last_error(PF_ERR_UNSUPPORTED, "%s: head_dim %d not built (64, 128, 256)", fn, D);
  if ((reinterpret_cast<uintptr_t>(k_pages) & 15u) || (reinterpret_cast<uintptr_t>(v_pages) & 15u))
    return set_last_error(PF_ERR_INVALID, "%s: page pools must be 16-byte aligned", fn);
  const long long cap = (long long)pages_per_seq * page_size;
  if (cap > INT_MAX)
    return set_last_error(PF_ERR_INVALID, "%s: pages_per_seq * page_size = %lld exceeds INT_MAX", fn, cap);
  if (max_context_len <= 0 || max_context_len > cap) max_context_len = (int)cap;

  // One split per sequence needs B*H*(D+2) floats; use more splits only while they fit.
  const size_t per_split = (size_t)B * H * (D + 2) * sizeof(float);
  if (per_split > kNoallocScratchBytes)
    return set_last_error(PF_ERR_WORKSPACE,
                          "%s: B=%d H=%d D=%d needs %zu bytes of split-KV partials, above the fixed "
                          "%zu-byte scratch; call pf_paged_decode with a workspace instead",
                          fn, B, H, D, per_split, kNoallocScratchBytes);
  DecodeArgs a{};
  a.q = q; a.k_src = k_pages; a.v_src = v_pages; a.block_tables = block_tables;
  a.context_lens = context_lens; a.o = o; a.dtype = dtype; a.B = B; a.H = H; a.Hkv = Hkv; a.D = D;
  a.num_pages = num_pages; a.page_size = page_size; a.pages_per_seq = pages_per_seq;
  a.max_len = max_context_len; a.sm_scale = sm_scale; a.stream = static_cast<cudaStream_t>(stream);
  decode_plan(max_context_len, B, Hkv, &a.num_splits, &a.split_len);
  const int max_ns = (int)(kNoallocScratchBytes / per_split);
  if (a.num_splits > max_ns) {
    int sl = (max_context_len + max_ns - 1) / max_ns;
    sl = (sl + kQuantum - 1) / kQuantum * kQuantum;
    a.split_len = sl;
    a.num_splits = (max_context_len + sl - 1) / sl;
  }
  void* scratch = nullptr;
  const cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess)
    return set_last_error(PF_ERR_CUDA, "%s: cudaGetSymbolAddress: %s", fn, cudaGetErrorString(e));
  a.partial = static_cast<float*>(scratch);
  const cudaError_t le = launch_decode(a);
  if (le != cudaSuccess) return set_last_error(PF_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(le));
  return PF_OK;
}
