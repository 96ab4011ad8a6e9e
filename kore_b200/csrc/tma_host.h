// Host-side helpers: TMA tensor-map encoding through the driver entry point
// (no link-time dependency on libcuda), and device property caching.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <stdexcept>
#include <string>

namespace kore {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_tiled();
int num_sms(int device);

// 2-D tile map over a row-major matrix: `inner` contiguous elements per row,
// `outer` rows, rows `row_stride_elems` apart. Box = box_inner x box_outer.
CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                         uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                         uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// 3-D variant (inner, mid, outer) with explicit strides in elements.
CUtensorMap make_tmap_3d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                         uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_elems,
                         uint64_t stride2_elems, uint32_t b0, uint32_t b1, uint32_t b2,
                         CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Reads and clears the device-side error word (1 = barrier wait timeout,
// 2 = peer flag timeout). Synchronizes the current device.
int read_and_clear_device_error();

}  // namespace kore
