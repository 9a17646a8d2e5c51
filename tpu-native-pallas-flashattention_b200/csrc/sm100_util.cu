// sm100_util.cu -- host side of sm100_util.cuh: TMA tensor maps, encoded
// through the driver entry point so the library needs no -lcuda.
#include "sm100_util.cuh"
#include "kernels.h"

#include <mutex>
#include <map>
#include <set>
#include <utility>

namespace pf {
namespace {
// --------------------------------------------------------------------------
// Host side: tensor maps through the driver entry point (no -lcuda needed).
// --------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace

cudaError_t set_smem_once(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kernel, dev})) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.insert({kernel, dev});
  return e;
}

int sm_count() {
  static std::mutex mu;
  static std::map<int, int> counts;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  auto it = counts.find(dev);
  if (it != counts.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  counts[dev] = n;
  return n;
}

bool make_tile_map(CUtensorMap* m, const void* base, int dtype, int D, int rows,
                   long row_stride_rows, int planes, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return false;
  const CUtensorMapDataType dt =
      dtype == PF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)rows, (cuuint64_t)planes};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)row_stride_rows * D * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A paged pool of D = 128 rows viewed so that one TMA box brings both 64-column
// halves of `box_rows` consecutive rows: dims (64 columns, rows at 256 B, 2
// halves at 128 B), box {64, box_rows, 2}; the box lands in shared memory as
// [half][row][64 columns], the layout two {64, box_rows} boxes give.
bool make_paged_pair_map(CUtensorMap* m, const void* base, int dtype, long rows, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return false;
  const CUtensorMapDataType dt =
      dtype == PF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, 2};
  cuuint64_t strides[2] = {256, 128};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 2};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace pf
