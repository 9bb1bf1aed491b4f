// Vectorised global loads/stores of VEC consecutive elements converted to/from fp32.
#pragma once
#include "common.cuh"

namespace ssla {

template <typename T, int VEC> struct Vec;

template <typename T> struct Vec<T, 1> {
  static __device__ __forceinline__ void load(const T* p, float* x) { x[0] = ldf(p); }
  static __device__ __forceinline__ void store(T* p, const float* x) { stf(p, x[0]); }
};

template <> struct Vec<float, 4> {
  static __device__ __forceinline__ void load(const float* p, float* x) {
    float4 v = __ldg(reinterpret_cast<const float4*>(p));
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  }
  static __device__ __forceinline__ void store(float* p, const float* x) {
    *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
  }
};

template <> struct Vec<__nv_bfloat16, 4> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float* x) {
    uint2 r = __ldg(reinterpret_cast<const uint2*>(p));
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&r.x);
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&r.y);
    x[0] = __low2float(a); x[1] = __high2float(a); x[2] = __low2float(b); x[3] = __high2float(b);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float* x) {
    __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(x[2], x[3]);
    uint2 r;
    r.x = *reinterpret_cast<uint32_t*>(&a);
    r.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = r;
  }
};

template <> struct Vec<__half, 4> {
  static __device__ __forceinline__ void load(const __half* p, float* x) {
    uint2 r = __ldg(reinterpret_cast<const uint2*>(p));
    __half2 a = *reinterpret_cast<__half2*>(&r.x);
    __half2 b = *reinterpret_cast<__half2*>(&r.y);
    x[0] = __low2float(a); x[1] = __high2float(a); x[2] = __low2float(b); x[3] = __high2float(b);
  }
  static __device__ __forceinline__ void store(__half* p, const float* x) {
    __half2 a = __floats2half2_rn(x[0], x[1]);
    __half2 b = __floats2half2_rn(x[2], x[3]);
    uint2 r;
    r.x = *reinterpret_cast<uint32_t*>(&a);
    r.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = r;
  }
};

// 16-byte vectors of 16-bit types (8 elements).
template <typename T2> struct Pair16;
template <> struct Pair16<__nv_bfloat16> {
  using P = __nv_bfloat162;
  static __device__ __forceinline__ P pack(float a, float b) { return __floats2bfloat162_rn(a, b); }
};
template <> struct Pair16<__half> {
  using P = __half2;
  static __device__ __forceinline__ P pack(float a, float b) { return __floats2half2_rn(a, b); }
};

template <typename T> struct Vec8x16 {
  using P = typename Pair16<T>::P;
  static __device__ __forceinline__ void load(const T* p, float* x) {
    uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
    unpack(r, x);
  }
  static __device__ __forceinline__ void unpack(uint4 r, float* x) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      P a = *reinterpret_cast<const P*>(&w[i]);
      x[2 * i] = __low2float(a);
      x[2 * i + 1] = __high2float(a);
    }
  }
  static __device__ __forceinline__ void store(T* p, const float* x) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      P a = Pair16<T>::pack(x[2 * i], x[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&a);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
};
template <> struct Vec<__nv_bfloat16, 8> : Vec8x16<__nv_bfloat16> {};
template <> struct Vec<__half, 8> : Vec8x16<__half> {};

inline bool aligned_to(const void* p, size_t a) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace ssla
