// Shared device helpers for the ssla_b200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include <utility>

#include "../../include/ssla_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "ssla_b200 kernels target sm_100a (Blackwell) only"
#endif

namespace ssla {

// Last error message, per host thread; read through ssla_last_error().
void set_error(const char* fmt, ...);
const char* get_error();

#define SSLA_CHECK_ARG(cond, ...)                  \
  do {                                             \
    if (!(cond)) {                                 \
      ::ssla::set_error(__VA_ARGS__);              \
      return SSLA_ERR_INVALID_ARG;                 \
    }                                              \
  } while (0)

#define SSLA_CHECK_LAUNCH(name)                                                  \
  do {                                                                           \
    cudaError_t e__ = cudaGetLastError();                                        \
    if (e__ != cudaSuccess) {                                                    \
      ::ssla::set_error("%s: launch failed: %s", name, cudaGetErrorString(e__)); \
      return SSLA_ERR_CUDA;                                                      \
    }                                                                            \
  } while (0)

template <typename T> struct Io;
template <> struct Io<float> {
  static __device__ __forceinline__ float ld(const float* p) { return *p; }
  static __device__ __forceinline__ void st(float* p, float x) { *p = x; }
};
template <> struct Io<__nv_bfloat16> {
  static __device__ __forceinline__ float ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }
};
template <> struct Io<__half> {
  static __device__ __forceinline__ float ld(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ void st(__half* p, float x) { *p = __float2half_rn(x); }
};

template <typename T> __device__ __forceinline__ float ldf(const T* p) { return Io<T>::ld(p); }
template <typename T> __device__ __forceinline__ void stf(T* p, float x) { Io<T>::st(p, x); }

// Programmatic dependent launch (chunk path).  A kernel launched with launch_pdl may start
// while its stream predecessor is still running: it calls griddep_launch_dependents() early
// (letting its own successor launch once all of its CTAs have started) and griddep_wait()
// after its prologue, before reading anything a predecessor wrote or writing anything a
// predecessor may still read.  Both are no-ops for an ordinary launch.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

inline size_t dtype_size(int dt) { return dt == SSLA_F32 ? 4 : 2; }
inline bool dtype_ok(int dt) { return dt == SSLA_F32 || dt == SSLA_BF16 || dt == SSLA_F16; }

// Dispatch a generic lambda over one runtime dtype code.
#define SSLA_DISPATCH_DTYPE(code, TYPE, ...)                          \
  [&]() -> int {                                                      \
    switch (code) {                                                   \
      case SSLA_F32: { using TYPE = float; return __VA_ARGS__(); }    \
      case SSLA_BF16: { using TYPE = __nv_bfloat16; return __VA_ARGS__(); } \
      case SSLA_F16: { using TYPE = __half; return __VA_ARGS__(); }   \
      default: ::ssla::set_error("unsupported dtype code %d", code); return SSLA_ERR_INVALID_ARG; \
    }                                                                 \
  }()

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

constexpr int kNumSMs = 148;

}  // namespace ssla
