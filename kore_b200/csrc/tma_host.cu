#include "tma_host.h"
#include "common.cuh"

#include <mutex>
#include <vector>

namespace kore {

static std::vector<int (*)()>& error_readers() {
  static std::vector<int (*)()> v;
  return v;
}
void register_error_reader(int (*fn)()) { error_readers().push_back(fn); }

EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q),
               "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    if (q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int num_sms(int device) {
  static std::vector<int> cache(64, 0);
  if (device < 0 || device >= 64) throw std::runtime_error("bad device index");
  if (cache[device] == 0) {
    int v = 0;
    check_cuda(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device),
               "cudaDeviceGetAttribute(SM count)");
    cache[device] = v;
  }
  return cache[device];
}

CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                         uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                         uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  if ((strides[0] & 15) != 0) throw std::runtime_error("TMA row stride must be a multiple of 16 B");
  CUresult r = get_encode_tiled()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed (2d), code " + std::to_string(r));
  return m;
}

CUtensorMap make_tmap_3d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0,
                         uint64_t d1, uint64_t d2, uint64_t stride1_elems, uint64_t stride2_elems,
                         uint32_t b0, uint32_t b1, uint32_t b2, CUtensorMapSwizzle swizzle) {
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_elems * (uint64_t)elem_bytes,
                           stride2_elems * (uint64_t)elem_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  if ((strides[0] & 15) != 0 || (strides[1] & 15) != 0)
    throw std::runtime_error("TMA strides must be multiples of 16 B");
  CUresult r = get_encode_tiled()(&m, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed (3d), code " + std::to_string(r));
  return m;
}

int read_and_clear_device_error() {
  check_cuda(cudaDeviceSynchronize(), "sync before error read");
  int v = 0;
  for (auto fn : error_readers()) {
    int e = fn();
    if (e != 0) v = e;
  }
  return v;
}

}  // namespace kore
