// Tensor-core (tcgen05) kernels of the chunked GLA path.  Not yet enabled: tc_supported()
// reports no coverage, so every shape runs on the CUDA-core kernels of chunk_gla.cu.
#include "chunk_gla.cuh"

namespace ssla {
namespace chunk {

int tc_supported(int, int, int64_t, int64_t) { return 0; }
int tc_local_state(int, int, int, const void*, const void*, const void*, const int64_t*,
                   const int64_t*, int64_t, int64_t, int64_t, float, float*, float*, cudaStream_t) {
  return SSLA_ERR_UNSUPPORTED;
}
int tc_fwd_o(int, int, const void*, const void*, const void*, const void*, const int64_t*,
             const int64_t*, int64_t, int64_t, int64_t, float, const float*, void*, cudaStream_t) {
  return SSLA_ERR_UNSUPPORTED;
}
int tc_bwd(int, int, const void*, const void*, const void*, const void*, const int64_t*,
           const int64_t*, int64_t, int64_t, int64_t, float, const float*, const float*,
           const void*, void*, void*, void*, float*, cudaStream_t) {
  return SSLA_ERR_UNSUPPORTED;
}

}  // namespace chunk
}  // namespace ssla
