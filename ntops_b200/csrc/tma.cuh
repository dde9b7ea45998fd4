// Host-side TMA descriptor encoding through the driver entry point (no libcuda link needed).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "ntb_common.cuh"

namespace ntb {
namespace tma {

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Encodes a rank-3 (x innermost, y, z) tiled map with 128-byte swizzle and zero OOB fill.
// strides_bytes[0] is the y stride, [1] the z stride; both must be multiples of 16.
inline int encode_3d(CUtensorMap* map, CUtensorMapDataType dtype, void* base, uint64_t dx, uint64_t dy,
                     uint64_t dz, uint64_t sy_bytes, uint64_t sz_bytes, uint32_t bx, uint32_t by,
                     CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  NTB_REQUIRE(fn != nullptr, NTB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {dx, dy, dz};
  cuuint64_t strides[2] = {sy_bytes, sz_bytes};
  cuuint32_t box[3] = {bx, by, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  NTB_REQUIRE(r == CUDA_SUCCESS, NTB_ERR_CUDA,
              "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu x %llu, strides %llu %llu, box %u x %u",
              (int)r, (unsigned long long)dx, (unsigned long long)dy, (unsigned long long)dz,
              (unsigned long long)sy_bytes, (unsigned long long)sz_bytes, bx, by);
  return NTB_OK;
}

// Rank-4 variant (x, y, z, w), box {bx, by, 1, 1}.
inline int encode_4d(CUtensorMap* map, CUtensorMapDataType dtype, void* base, uint64_t dx, uint64_t dy,
                     uint64_t dz, uint64_t dw, uint64_t sy_bytes, uint64_t sz_bytes, uint64_t sw_bytes,
                     uint32_t bx, uint32_t by, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  NTB_REQUIRE(fn != nullptr, NTB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[4] = {dx, dy, dz, dw};
  cuuint64_t strides[3] = {sy_bytes, sz_bytes, sw_bytes};
  cuuint32_t box[4] = {bx, by, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, dtype, 4, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  NTB_REQUIRE(r == CUDA_SUCCESS, NTB_ERR_CUDA, "cuTensorMapEncodeTiled (4-D) failed (%d)", (int)r);
  return NTB_OK;
}

inline PFN_cuTensorMapEncodeIm2col_v12000 encode_im2col_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(p);
  });
  return fn;
}

// im2col map over an activation [N, H, W, C] (channels innermost; C, W, H, N as dims 0..3) with
// 128-byte swizzle and zero OOB fill.  The pixel box of window origins runs from (lower_w,
// lower_h) to (W - 1 + upper_w, H - 1 + upper_h) stepping by (step_w, step_h); each load
// copies `pixels` pixels of `channels` channels.
inline int encode_im2col_4d(CUtensorMap* map, CUtensorMapDataType dtype, void* base, uint64_t C, uint64_t W,
                            uint64_t H, uint64_t N, uint64_t sw_bytes, uint64_t sh_bytes, uint64_t sn_bytes,
                            int lower_w, int lower_h, int upper_w, int upper_h, uint32_t channels, uint32_t pixels,
                            uint32_t step_w, uint32_t step_h) {
  auto fn = encode_im2col_fn();
  NTB_REQUIRE(fn != nullptr, NTB_ERR_CUDA, "cuTensorMapEncodeIm2col is not available from the driver");
  cuuint64_t dims[4] = {C, W, H, N};
  cuuint64_t strides[3] = {sw_bytes, sh_bytes, sn_bytes};
  int lower[2] = {lower_w, lower_h};
  int upper[2] = {upper_w, upper_h};
  cuuint32_t estr[4] = {1, step_w, step_h, 1};
  CUresult r = fn(map, dtype, 4, base, dims, strides, lower, upper, channels, pixels, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  NTB_REQUIRE(r == CUDA_SUCCESS, NTB_ERR_CUDA,
              "cuTensorMapEncodeIm2col failed (%d): C %llu W %llu H %llu N %llu, box (%d, %d) .. (%d, %d)", (int)r,
              (unsigned long long)C, (unsigned long long)W, (unsigned long long)H, (unsigned long long)N, lower_w,
              lower_h, upper_w, upper_h);
  return NTB_OK;
}

// A TMA stride must be a positive multiple of 16 bytes below 2^40.
inline bool stride_ok(int64_t bytes) { return bytes > 0 && bytes % 16 == 0 && bytes < (1LL << 40); }

}  // namespace tma
}  // namespace ntb
