// sm100_util.cuh -- host and device helpers shared by the tcgen05 kernels:
// TMA tensor maps over [planes, rows, D] 16-bit tensors and the UMMA shared-
// memory descriptors of the tiles those maps produce.
//
// Every tile is stored as D/64 "boxes" of `rows` x 64 elements (128-byte rows,
// 128-byte swizzle, 1024-byte swizzle atoms of 8 rows).  One physical layout
// serves two operand roles:
//   K-major  (rows = M or N, contiguous 64-element chunks along K = d):
//            k-step kk (16 elements) starts 32*(kk%4) bytes into box kk/4;
//   MN-major (rows = K, contiguous chunks along N = d):
//            k-step kk (16 rows) starts 16*128*kk bytes in; the next 64
//            columns are one box further (LBO), 8-row groups 1024 B apart (SBO).
#pragma once

#include <cuda.h>
#include "common.cuh"

namespace pf {

template <int ROWS>
__device__ __forceinline__ uint64_t desc_k(uint32_t tile_addr, int kk) {
  const uint32_t addr = tile_addr + (kk >> 2) * (ROWS * 128) + (kk & 3) * 32;
  return smem_desc_sw128(addr, 16, 1024);
}

template <int ROWS>
__device__ __forceinline__ uint64_t desc_mn(uint32_t tile_addr, int kk) {
  return smem_desc_sw128(tile_addr + kk * 16 * 128, ROWS * 128, 1024);
}

// Cheap per-MMA descriptors: the start-address field is linear (address/16 in
// bits 0-13, and shared addresses stay below 256 KB, so it never carries), so
// the descriptor of k-step kk is the tile's base descriptor plus a
// compile-time constant.  The MMA-issuing thread shares its scheduler with
// busy elementwise warps; every instruction it spends between two MMAs
// delays the tensor core, so descriptors are built once per tile.
template <int ROWS>
__device__ __forceinline__ uint64_t desc_k_base(uint32_t tile_addr) {
  return smem_desc_sw128(tile_addr, 16, 1024);
}
template <int ROWS>
__device__ __forceinline__ uint64_t desc_mn_base(uint32_t tile_addr) {
  return smem_desc_sw128(tile_addr, ROWS * 128, 1024);
}
template <int ROWS>
constexpr uint64_t koff(int kk) {
  return (uint64_t)(((kk >> 2) * (ROWS * 128) + (kk & 3) * 32) >> 4);
}
constexpr uint64_t mnoff(int kk) { return (uint64_t)(kk * 16 * 128 >> 4); }

// TMEM column of k-step kk (16 values of K) of a 16-bit operand packed by the
// elementwise warps: each 32-column chunk c of an f32 tile holds its 32 values
// as 16 packed pairs in columns [32c, 32c + 16).
__device__ __forceinline__ uint32_t split_packed_col(int kk) {
  return (uint32_t)((kk >> 1) * 32 + (kk & 1) * 8);
}

// 16-bit [planes, row_stride_rows, D] tensor exposing `rows` rows per plane,
// box = 64 columns x box_rows rows, 128-byte swizzle, zero fill past `rows`.
bool make_tile_map(CUtensorMap* m, const void* base, int dtype, int D, int rows,
                   long row_stride_rows, int planes, int box_rows);
// A D = 128 paged pool as (64 columns, rows, 2 halves): one box of
// {64, box_rows, 2} brings both column halves of box_rows rows.
bool make_paged_pair_map(CUtensorMap* m, const void* base, int dtype, long rows, int box_rows);

}  // namespace pf
