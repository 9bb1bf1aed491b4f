// Token-by-token gated linear attention (fused_recurrent_gla forward), the streaming path:
//   S_t = diag(exp(g_t)) S_{t-1} + k_t v_t^T ,   o_t = (scale q_t)^T S_t
// with the update before the read-out, as in naive_gla_recurrent (ops/gla/naive.py:93-98).
//
// The step is HBM-bound: per (sequence, head) the fp32 state [K,V] is read and written once
// per call, the token vectors are tiny.  Fast path: one warp owns a 32-column slice of one
// (sequence, head) state; lane = 8*r + c holds rows {r, r+4, r+8, ...} of columns
// [4c, 4c+4) as float4 registers, so each warp-wide 16-byte load/store moves four full
// 128-byte state rows (fully coalesced).  q/k/exp(g) are loaded once per warp and
// broadcast with shuffles; the read-out over K is an in-register partial sum followed by a
// two-step xor-shuffle reduction over the four row phases.  The state stays in registers
// across the tokens of a sequence, so multi-token sequences touch HBM state only once.
#include "common.cuh"
#include "vec.cuh"

namespace ssla {
namespace {

template <typename T, typename Tg, int K>
__global__ void __launch_bounds__(256) recurrent_gla_fwd_fast(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const Tg* __restrict__ g, const int64_t* __restrict__ cu, int64_t n_seqs, int H, int V,
    float scale, const float* __restrict__ h0, T* __restrict__ o, float* __restrict__ ht) {
  constexpr int KR = K / 4;          // rows held per lane
  constexpr int KL = (K + 31) / 32;  // token-vector elements loaded per lane
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int VB = V / 32;
  if (warp >= n_seqs * H * VB) return;
  const int64_t sh = warp / VB;  // (seq, head)
  const int vb = (int)(warp - sh * VB);
  const int64_t seq = sh / H;
  const int head = (int)(sh - seq * H);
  const int r = lane >> 3, c = lane & 7;
  const int col = vb * 32 + c * 4;
  const int64_t bos = cu[seq], eos = cu[seq + 1];

  float4 S[KR];
  const size_t sbase = (size_t)sh * K * V + col;
  if (h0) {
#pragma unroll
    for (int i = 0; i < KR; ++i)
      S[i] = __ldg(reinterpret_cast<const float4*>(h0 + sbase + (size_t)(r + 4 * i) * V));
  } else {
#pragma unroll
    for (int i = 0; i < KR; ++i) S[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  for (int64_t t = bos; t < eos; ++t) {
    const size_t tk = ((size_t)t * H + head) * K;
    float xq[KL], xk[KL], xd[KL];
#pragma unroll
    for (int j = 0; j < KL; ++j) {
      const int kk = lane + 32 * j;
      if (kk < K) {
        xq[j] = ldf(q + tk + kk) * scale;
        xk[j] = ldf(k + tk + kk);
        xd[j] = expf(ldf(g + tk + kk));
      } else {
        xq[j] = xk[j] = xd[j] = 0.f;
      }
    }
    float xv[4];
    Vec<T, 4>::load(v + ((size_t)t * H + head) * V + col, xv);
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll
    for (int i = 0; i < KR; ++i) {
      const int kk = r + 4 * i;
      const float d = __shfl_sync(0xffffffffu, xd[kk / 32], kk % 32);
      const float kv = __shfl_sync(0xffffffffu, xk[kk / 32], kk % 32);
      const float qq = __shfl_sync(0xffffffffu, xq[kk / 32], kk % 32);
      S[i].x = fmaf(d, S[i].x, kv * xv[0]);
      S[i].y = fmaf(d, S[i].y, kv * xv[1]);
      S[i].z = fmaf(d, S[i].z, kv * xv[2]);
      S[i].w = fmaf(d, S[i].w, kv * xv[3]);
      o0 = fmaf(qq, S[i].x, o0);
      o1 = fmaf(qq, S[i].y, o1);
      o2 = fmaf(qq, S[i].z, o2);
      o3 = fmaf(qq, S[i].w, o3);
    }
#pragma unroll
    for (int m = 8; m <= 16; m <<= 1) {
      o0 += __shfl_xor_sync(0xffffffffu, o0, m);
      o1 += __shfl_xor_sync(0xffffffffu, o1, m);
      o2 += __shfl_xor_sync(0xffffffffu, o2, m);
      o3 += __shfl_xor_sync(0xffffffffu, o3, m);
    }
    if (r == 0) {
      const float ov[4] = {o0, o1, o2, o3};
      Vec<T, 4>::store(o + ((size_t)t * H + head) * V + col, ov);
    }
  }
  if (ht) {
#pragma unroll
    for (int i = 0; i < KR; ++i)
      *reinterpret_cast<float4*>(ht + sbase + (size_t)(r + 4 * i) * V) = S[i];
  }
}

// Generic shapes: one thread per (sequence, head, column), state column in registers.
template <typename T, typename Tg, int KMAX>
__global__ void __launch_bounds__(128) recurrent_gla_fwd_generic(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const Tg* __restrict__ g, const int64_t* __restrict__ cu, int64_t n_seqs, int H, int K,
    int V, float scale, const float* __restrict__ h0, T* __restrict__ o, float* __restrict__ ht) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_seqs * H * V) return;
  const int64_t sh = idx / V;
  const int col = (int)(idx - sh * V);
  const int64_t seq = sh / H;
  const int head = (int)(sh - seq * H);
  const int64_t bos = cu[seq], eos = cu[seq + 1];
  float S[KMAX];
  const size_t sbase = (size_t)sh * K * V + col;
#pragma unroll
  for (int i = 0; i < KMAX; ++i) S[i] = (i < K && h0) ? h0[sbase + (size_t)i * V] : 0.f;
  for (int64_t t = bos; t < eos; ++t) {
    const size_t tk = ((size_t)t * H + head) * K;
    const float xv = ldf(v + ((size_t)t * H + head) * V + col);
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < KMAX; ++i) {
      if (i < K) {
        S[i] = fmaf(expf(ldf(g + tk + i)), S[i], ldf(k + tk + i) * xv);
        acc = fmaf(ldf(q + tk + i) * scale, S[i], acc);
      }
    }
    stf(o + ((size_t)t * H + head) * V + col, acc);
  }
  if (ht) {
#pragma unroll
    for (int i = 0; i < KMAX; ++i)
      if (i < K) ht[sbase + (size_t)i * V] = S[i];
  }
}

template <typename T, typename Tg>
int launch(const void* q, const void* k, const void* v, const void* g, const int64_t* cu,
           int64_t N, int H, int K, int V, float scale, const float* h0, void* o, float* ht,
           cudaStream_t s) {
  const bool fast = (V % 32 == 0) && (K == 16 || K == 32 || K == 64 || K == 128) &&
                    aligned_to(v, 4 * sizeof(T)) && aligned_to(o, 4 * sizeof(T)) &&
                    aligned_to(h0, 16) && aligned_to(ht, 16);
  if (fast) {
    const int64_t threads = N * H * (V / 32) * 32;
    const int grid = ceil_div(threads, 256);
#define SSLA_RG_FAST(KK)                                                                      \
  recurrent_gla_fwd_fast<T, Tg, KK><<<grid, 256, 0, s>>>((const T*)q, (const T*)k, (const T*)v, \
                                                         (const Tg*)g, cu, N, H, V, scale, h0,  \
                                                         (T*)o, ht)
    switch (K) {
      case 16: SSLA_RG_FAST(16); break;
      case 32: SSLA_RG_FAST(32); break;
      case 64: SSLA_RG_FAST(64); break;
      default: SSLA_RG_FAST(128); break;
    }
#undef SSLA_RG_FAST
  } else {
    const int64_t threads = N * H * V;
    const int grid = ceil_div(threads, 128);
#define SSLA_RG_GEN(KK)                                                                          \
  recurrent_gla_fwd_generic<T, Tg, KK><<<grid, 128, 0, s>>>((const T*)q, (const T*)k, (const T*)v, \
                                                            (const Tg*)g, cu, N, H, K, V, scale, \
                                                            h0, (T*)o, ht)
    if (K <= 32) SSLA_RG_GEN(32);
    else if (K <= 64) SSLA_RG_GEN(64);
    else if (K <= 128) SSLA_RG_GEN(128);
    else SSLA_RG_GEN(256);
#undef SSLA_RG_GEN
  }
  SSLA_CHECK_LAUNCH("ssla_recurrent_gla_fwd");
  return SSLA_OK;
}

}  // namespace
}  // namespace ssla

using namespace ssla;

extern "C" int ssla_recurrent_gla_fwd(const void* q, const void* k, const void* v, const void* g,
                                      int dtype, int dtype_g, const int64_t* cu_seqlens,
                                      int64_t n_seqs, int64_t T, int64_t H, int64_t K, int64_t V,
                                      float scale, const float* h0, void* o, float* ht,
                                      ssla_stream_t stream) {
  SSLA_CHECK_ARG(dtype_ok(dtype) && dtype_ok(dtype_g), "ssla_recurrent_gla_fwd: bad dtype");
  SSLA_CHECK_ARG(n_seqs >= 0 && T >= 0 && H >= 0 && K >= 0 && V >= 0,
                 "ssla_recurrent_gla_fwd: negative size");
  SSLA_CHECK_ARG(K <= 256, "ssla_recurrent_gla_fwd: K=%lld > 256 is not supported", (long long)K);
  if (n_seqs == 0 || H == 0 || V == 0) return SSLA_OK;
  SSLA_CHECK_ARG(cu_seqlens, "ssla_recurrent_gla_fwd: null cu_seqlens");
  SSLA_CHECK_ARG(T == 0 || (q && k && v && g && o), "ssla_recurrent_gla_fwd: null pointer");
  SSLA_CHECK_ARG(K > 0, "ssla_recurrent_gla_fwd: K must be positive");
  cudaStream_t s = (cudaStream_t)stream;
  return SSLA_DISPATCH_DTYPE(dtype, T_, [&] {
    return SSLA_DISPATCH_DTYPE(dtype_g, Tg, [&] {
      return launch<T_, Tg>(q, k, v, g, cu_seqlens, n_seqs, (int)H, (int)K, (int)V, scale, h0, o,
                            ht, s);
    });
  });
}
