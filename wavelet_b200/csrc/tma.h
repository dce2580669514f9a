// Host-side TMA descriptor construction (cuTensorMapEncodeTiled through the
// runtime's driver entry point, so the extension needs no -lcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace wb {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
      throw std::runtime_error("wavelet_b200: cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D row-major matrix of `outer` rows x `inner` contiguous elements with a
// row pitch of `ld` elements.  Box = box_inner x box_outer elements.
inline CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                                uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                                uint32_t box_outer, CUtensorMapSwizzle swz) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    throw std::runtime_error("wavelet_b200: TMA base address must be 16-byte aligned");
  if ((ld * elem_bytes) % 16 != 0)
    throw std::runtime_error("wavelet_b200: TMA row pitch must be a multiple of 16 bytes (ld=" +
                             std::to_string(ld) + ")");
  if ((box_inner * elem_bytes) % 16 != 0)
    throw std::runtime_error("wavelet_b200: TMA box inner extent must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * static_cast<uint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("wavelet_b200: cuTensorMapEncodeTiled failed (" + std::to_string(r) +
                             ")");
  return m;
}

inline int num_sms(int device) {
  static int cached[64] = {0};
  if (device < 0 || device >= 64) device = 0;
  if (!cached[device]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
    cached[device] = v > 0 ? v : 148;
  }
  return cached[device];
}

}  // namespace wb
