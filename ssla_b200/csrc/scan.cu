// Element-wise gated scan h_t = g_t * h_{t-1} + u_t over packed variable-length sequences
// (the recurrence MosAttention / LinearAttention run, ops/common/scan.py:11-86), and the
// scalar-state GLA recurrence (ops/gla/naive_scalar.py:7-66) that backs chunk_gla_scalar.
//
// Design: the work is HBM-bound and the sequences are short (1-11 events on average in
// the model), so one thread owns VEC adjacent channels of one sequence and walks its tokens
// in order.  Channel vectors are loaded 16 B (fp32) / 8 B (16-bit) at a time; consecutive
// threads cover consecutive channels of the same rows, so a warp reads whole rows.
// Arithmetic is fp32 with one rounding per multiply and per add (no FMA contraction), the
// same operation order as the reference, so results are bit-identical to a CPU fp32 scan.
#include "common.cuh"
#include "vec.cuh"

namespace ssla {
namespace {

template <typename Tu, typename Tg, int VEC>
__global__ void __launch_bounds__(256) scan_fwd_kernel(const Tu* __restrict__ u,
                                                       const Tg* __restrict__ g,
                                                       Tu* __restrict__ h,
                                                       const int64_t* __restrict__ cu,
                                                       int64_t n_seqs, int64_t C) {
  const int64_t CV = C / VEC;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_seqs * CV) return;
  const int64_t seq = idx / CV;
  const int64_t c = (idx - seq * CV) * VEC;
  const int64_t bos = cu[seq], eos = cu[seq + 1];
  float acc[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) acc[i] = 0.f;
  // tokens in batches of U: the batch's loads are issued together (they do not depend on the
  // running value), so a sequence costs one memory round trip per U tokens, not per token
  constexpr int U = 4;
  for (int64_t t0 = bos; t0 < eos; t0 += U) {
    float xu[U][VEC], xg[U][VEC];
#pragma unroll
    for (int j = 0; j < U; ++j)
      if (t0 + j < eos) {
        Vec<Tu, VEC>::load(u + (t0 + j) * C + c, xu[j]);
        Vec<Tg, VEC>::load(g + (t0 + j) * C + c, xg[j]);
      }
#pragma unroll
    for (int j = 0; j < U; ++j)
      if (t0 + j < eos) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] = __fadd_rn(__fmul_rn(acc[i], xg[j][i]), xu[j][i]);
        Vec<Tu, VEC>::store(h + (t0 + j) * C + c, acc);
      }
  }
}

template <typename Tu, typename Tg, int VEC>
__global__ void __launch_bounds__(256) scan_bwd_kernel(const Tu* __restrict__ dout,
                                                       const Tg* __restrict__ g,
                                                       const Tu* __restrict__ h,
                                                       Tu* __restrict__ du, Tg* __restrict__ dg,
                                                       const int64_t* __restrict__ cu,
                                                       int64_t n_seqs, int64_t C) {
  const int64_t CV = C / VEC;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_seqs * CV) return;
  const int64_t seq = idx / CV;
  const int64_t c = (idx - seq * CV) * VEC;
  const int64_t bos = cu[seq], eos = cu[seq + 1];
  float dh[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) dh[i] = 0.f;
  // tokens in batches of U from the end, loads of a batch issued together (as the forward)
  constexpr int U = 4;
  for (int64_t t1 = eos - 1; t1 >= bos; t1 -= U) {
    float xdo[U][VEC], xg[U][VEC], xh[U][VEC];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int64_t t = t1 - j;
      if (t >= bos) {
        Vec<Tu, VEC>::load(dout + t * C + c, xdo[j]);
        Vec<Tg, VEC>::load(g + t * C + c, xg[j]);
        if (t > bos) {
          Vec<Tu, VEC>::load(h + (t - 1) * C + c, xh[j]);
        } else {
#pragma unroll
          for (int i = 0; i < VEC; ++i) xh[j][i] = 0.f;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int64_t t = t1 - j;
      if (t >= bos) {
        float xdg[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          dh[i] = __fadd_rn(dh[i], xdo[j][i]);
          xdg[i] = __fmul_rn(dh[i], xh[j][i]);
        }
        Vec<Tg, VEC>::store(dg + t * C + c, xdg);
        Vec<Tu, VEC>::store(du + t * C + c, dh);
#pragma unroll
        for (int i = 0; i < VEC; ++i) dh[i] = __fmul_rn(dh[i], xg[j][i]);
      }
    }
  }
}

// Scalar-state GLA: S_t = exp(g_t) S_{t-1} + k_t v_t ; o_t = (scale q_t) S_t.
template <typename T, typename Tg>
__global__ void __launch_bounds__(256) gla_scalar_fwd_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const Tg* __restrict__ g, const int64_t* __restrict__ cu, int64_t n_seqs, int64_t H,
    float scale, const float* __restrict__ h0, T* __restrict__ o, float* __restrict__ ht) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_seqs * H) return;
  const int64_t seq = idx / H, hh = idx - seq * H;
  const int64_t bos = cu[seq], eos = cu[seq + 1];
  float S = h0 ? h0[idx] : 0.f;
  for (int64_t t = bos; t < eos; ++t) {
    const int64_t off = t * H + hh;
    const float d = expf(ldf(g + off));
    S = __fadd_rn(__fmul_rn(d, S), __fmul_rn(ldf(k + off), ldf(v + off)));
    stf(o + off, __fmul_rn(__fmul_rn(ldf(q + off), scale), S));
  }
  if (ht) ht[idx] = S;
}

// Backward of the scalar recurrence.  dS_t = scale q_t do_t + exp(g_{t+1}) dS_{t+1};
// dq_t = scale do_t S_t; dk_t = dS_t v_t; dv_t = dS_t k_t; dg_t = dS_t exp(g_t) S_{t-1}.
// The forward states S_{t-1} are parked in dg (fp32) by a first forward walk.
template <typename T, typename Tg>
__global__ void __launch_bounds__(256) gla_scalar_bwd_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const Tg* __restrict__ g, const int64_t* __restrict__ cu, int64_t n_seqs, int64_t H,
    float scale, const float* __restrict__ h0, const T* __restrict__ dout,
    const float* __restrict__ dht, T* __restrict__ dq, T* __restrict__ dk, T* __restrict__ dv,
    float* __restrict__ dg, float* __restrict__ dh0) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_seqs * H) return;
  const int64_t seq = idx / H, hh = idx - seq * H;
  const int64_t bos = cu[seq], eos = cu[seq + 1];
  float S = h0 ? h0[idx] : 0.f;
  for (int64_t t = bos; t < eos; ++t) {
    const int64_t off = t * H + hh;
    dg[off] = S;  // S_{t-1}
    const float d = expf(ldf(g + off));
    S = __fadd_rn(__fmul_rn(d, S), __fmul_rn(ldf(k + off), ldf(v + off)));
  }
  float dS = dht ? dht[idx] : 0.f;
  for (int64_t t = eos - 1; t >= bos; --t) {
    const int64_t off = t * H + hh;
    const float xq = ldf(q + off), xk = ldf(k + off), xv = ldf(v + off), xdo = ldf(dout + off);
    const float d = expf(ldf(g + off));
    const float Sprev = dg[off];
    const float St = d * Sprev + xk * xv;
    dS = dS + scale * xq * xdo;
    stf(dq + off, scale * xdo * St);
    stf(dk + off, dS * xv);
    stf(dv + off, dS * xk);
    dg[off] = dS * d * Sprev;
    dS = dS * d;
  }
  if (dh0) dh0[idx] = dS;
}

template <typename Tu, typename Tg>
int launch_scan_fwd(const void* u, const void* g, void* h, const int64_t* cu, int64_t N,
                    int64_t C, cudaStream_t s) {
  const bool v4 = (C % 4 == 0) && aligned_to(u, 4 * sizeof(Tu)) && aligned_to(h, 4 * sizeof(Tu)) &&
                  aligned_to(g, 4 * sizeof(Tg));
  const int64_t threads = N * (v4 ? C / 4 : C);
  if (threads == 0) return SSLA_OK;
  const int grid = ceil_div(threads, 256);
  if (v4)
    scan_fwd_kernel<Tu, Tg, 4><<<grid, 256, 0, s>>>((const Tu*)u, (const Tg*)g, (Tu*)h, cu, N, C);
  else
    scan_fwd_kernel<Tu, Tg, 1><<<grid, 256, 0, s>>>((const Tu*)u, (const Tg*)g, (Tu*)h, cu, N, C);
  SSLA_CHECK_LAUNCH("ssla_scan_fwd");
  return SSLA_OK;
}

template <typename Tu, typename Tg>
int launch_scan_bwd(const void* dout, const void* g, const void* h, void* du, void* dg,
                    const int64_t* cu, int64_t N, int64_t C, cudaStream_t s) {
  const bool v4 = (C % 4 == 0) && aligned_to(dout, 4 * sizeof(Tu)) &&
                  aligned_to(h, 4 * sizeof(Tu)) && aligned_to(du, 4 * sizeof(Tu)) &&
                  aligned_to(g, 4 * sizeof(Tg)) && aligned_to(dg, 4 * sizeof(Tg));
  const int64_t threads = N * (v4 ? C / 4 : C);
  if (threads == 0) return SSLA_OK;
  const int grid = ceil_div(threads, 256);
  if (v4)
    scan_bwd_kernel<Tu, Tg, 4><<<grid, 256, 0, s>>>((const Tu*)dout, (const Tg*)g, (const Tu*)h,
                                                    (Tu*)du, (Tg*)dg, cu, N, C);
  else
    scan_bwd_kernel<Tu, Tg, 1><<<grid, 256, 0, s>>>((const Tu*)dout, (const Tg*)g, (const Tu*)h,
                                                    (Tu*)du, (Tg*)dg, cu, N, C);
  SSLA_CHECK_LAUNCH("ssla_scan_bwd");
  return SSLA_OK;
}

}  // namespace
}  // namespace ssla

using namespace ssla;

extern "C" int ssla_scan_fwd(const void* u, int dtype_u, const void* g, int dtype_g, void* h,
                             int dtype_h, const int64_t* cu_seqlens, int64_t n_seqs, int64_t T,
                             int64_t C, ssla_stream_t stream) {
  SSLA_CHECK_ARG(dtype_ok(dtype_u) && dtype_ok(dtype_g), "ssla_scan_fwd: bad dtype");
  SSLA_CHECK_ARG(dtype_h == dtype_u, "ssla_scan_fwd: h must have u's dtype");
  SSLA_CHECK_ARG(n_seqs >= 0 && T >= 0 && C >= 0, "ssla_scan_fwd: negative size");
  if (n_seqs == 0 || C == 0 || T == 0) return SSLA_OK;
  SSLA_CHECK_ARG(u && g && h && cu_seqlens, "ssla_scan_fwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  return SSLA_DISPATCH_DTYPE(dtype_u, Tu, [&] {
    return SSLA_DISPATCH_DTYPE(dtype_g, Tg,
                               [&] { return launch_scan_fwd<Tu, Tg>(u, g, h, cu_seqlens, n_seqs, C, s); });
  });
}

extern "C" int ssla_scan_bwd(const void* dout, int dtype_do, const void* g, int dtype_g,
                             const void* h, int dtype_h, void* du, int dtype_du, void* dg,
                             int dtype_dg, const int64_t* cu_seqlens, int64_t n_seqs, int64_t T,
                             int64_t C, ssla_stream_t stream) {
  SSLA_CHECK_ARG(dtype_ok(dtype_do) && dtype_ok(dtype_g), "ssla_scan_bwd: bad dtype");
  SSLA_CHECK_ARG(dtype_h == dtype_do && dtype_du == dtype_do,
                 "ssla_scan_bwd: do, h and du must share one dtype");
  SSLA_CHECK_ARG(dtype_dg == dtype_g, "ssla_scan_bwd: dg must have g's dtype");
  SSLA_CHECK_ARG(n_seqs >= 0 && T >= 0 && C >= 0, "ssla_scan_bwd: negative size");
  if (n_seqs == 0 || C == 0 || T == 0) return SSLA_OK;
  SSLA_CHECK_ARG(dout && g && h && du && dg && cu_seqlens, "ssla_scan_bwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  return SSLA_DISPATCH_DTYPE(dtype_do, Tu, [&] {
    return SSLA_DISPATCH_DTYPE(dtype_g, Tg, [&] {
      return launch_scan_bwd<Tu, Tg>(dout, g, h, du, dg, cu_seqlens, n_seqs, C, s);
    });
  });
}

extern "C" int ssla_gla_scalar_fwd(const void* q, const void* k, const void* v, const void* g,
                                   int dtype, int dtype_g, const int64_t* cu_seqlens,
                                   int64_t n_seqs, int64_t T, int64_t H, float scale,
                                   const float* h0, void* o, float* ht, ssla_stream_t stream) {
  SSLA_CHECK_ARG(dtype_ok(dtype) && dtype_ok(dtype_g), "ssla_gla_scalar_fwd: bad dtype");
  SSLA_CHECK_ARG(n_seqs >= 0 && T >= 0 && H >= 0, "ssla_gla_scalar_fwd: negative size");
  if (n_seqs == 0 || H == 0) return SSLA_OK;
  SSLA_CHECK_ARG(cu_seqlens && (T == 0 || (q && k && v && g && o)), "ssla_gla_scalar_fwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const int grid = ceil_div(n_seqs * H, 256);
  return SSLA_DISPATCH_DTYPE(dtype, T_, [&] {
    return SSLA_DISPATCH_DTYPE(dtype_g, Tg, [&] {
      gla_scalar_fwd_kernel<T_, Tg><<<grid, 256, 0, s>>>(
          (const T_*)q, (const T_*)k, (const T_*)v, (const Tg*)g, cu_seqlens, n_seqs, H, scale, h0,
          (T_*)o, ht);
      SSLA_CHECK_LAUNCH("ssla_gla_scalar_fwd");
      return SSLA_OK;
    });
  });
}

extern "C" int ssla_gla_scalar_bwd(const void* q, const void* k, const void* v, const void* g,
                                   int dtype, int dtype_g, const int64_t* cu_seqlens,
                                   int64_t n_seqs, int64_t T, int64_t H, float scale,
                                   const float* h0, const void* dout, const float* dht, void* dq,
                                   void* dk, void* dv, float* dg, float* dh0,
                                   ssla_stream_t stream) {
  SSLA_CHECK_ARG(dtype_ok(dtype) && dtype_ok(dtype_g), "ssla_gla_scalar_bwd: bad dtype");
  SSLA_CHECK_ARG(n_seqs >= 0 && T >= 0 && H >= 0, "ssla_gla_scalar_bwd: negative size");
  if (n_seqs == 0 || H == 0) return SSLA_OK;
  SSLA_CHECK_ARG(cu_seqlens && (T == 0 || (q && k && v && g && dout && dq && dk && dv && dg)),
                 "ssla_gla_scalar_bwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const int grid = ceil_div(n_seqs * H, 256);
  return SSLA_DISPATCH_DTYPE(dtype, T_, [&] {
    return SSLA_DISPATCH_DTYPE(dtype_g, Tg, [&] {
      gla_scalar_bwd_kernel<T_, Tg><<<grid, 256, 0, s>>>(
          (const T_*)q, (const T_*)k, (const T_*)v, (const Tg*)g, cu_seqlens, n_seqs, H, scale, h0,
          (const T_*)dout, dht, (T_*)dq, (T_*)dk, (T_*)dv, dg, dh0);
      SSLA_CHECK_LAUNCH("ssla_gla_scalar_bwd");
      return SSLA_OK;
    });
  });
}
