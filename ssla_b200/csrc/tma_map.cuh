// Host-side TMA tensor-map encoding (cuTensorMapEncodeTiled through the runtime's driver entry
// point, so the library links only against the CUDA runtime).
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace ssla {
namespace tma {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiled encode_fn() {
  static EncodeTiled fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}

// Tiled map, unit element strides, out-of-range elements read as zero.
inline int encode(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
                  const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw, const char* who) {
  const EncodeTiled enc = encode_fn();
  if (!enc) {
    set_error("%s: cuTensorMapEncodeTiled is unavailable", who);
    return SSLA_ERR_CUDA;
  }
  const cuuint32_t es[3] = {1u, 1u, 1u};
  const CUresult r = enc(m, dt, rank, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("%s: cuTensorMapEncodeTiled failed (%d)", who, (int)r);
    return SSLA_ERR_CUDA;
  }
  return SSLA_OK;
}

}  // namespace tma
}  // namespace ssla
