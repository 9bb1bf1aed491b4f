// Fused inference kernels of the MoS attention layer (layers/mos_attention.py:75-146) and the
// residual + LayerNorm that closes it.
//
// mos_patch_scan: the per-patch work of the layer in one pass.  Every patch event t (rows of
// the patch sequences, packed by cu_seqlens, each sequence in time order) reads its projected
// row y[key[t]] = [q | v | g_pre] (3C floats, produced by one GEMM over the pixel events with
// the q/v/g projections folded into the per-position scatter weights), and runs
//   h = sigmoid(g_pre) * h + v         (the gated scan, ops/common/scan.py:35-43, same order)
//   z[dst[t]] = q * h
// so the q/v/g tensors, the scan output and q*h never go through HBM.  One thread owns 4
// adjacent channels of one sequence.
//
// layernorm_residual: out = LayerNorm(x + r) * w + b over rows of C channels (two-pass mean /
// variance in fp32).  Rows of up to 32 channels take one thread each, wider rows one warp.
#include "common.cuh"
#include "vec.cuh"

namespace ssla {
namespace {

__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }

__global__ void __launch_bounds__(256) mos_patch_scan_kernel(const float* __restrict__ y,
                                                             const int64_t* __restrict__ key,
                                                             const int64_t* __restrict__ dst,
                                                             const int64_t* __restrict__ cu, int64_t n_seqs,
                                                             int64_t C, float* __restrict__ z) {
  const int64_t CV = C / 4;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_seqs * CV) return;
  const int64_t seq = idx / CV;
  const int64_t c = (idx - seq * CV) * 4;
  const int64_t bos = cu[seq], eos = cu[seq + 1];
  float h[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t t = bos; t < eos; ++t) {
    const float* row = y + key[t] * 3 * C + c;
    const float4 q = *reinterpret_cast<const float4*>(row);
    const float4 v = *reinterpret_cast<const float4*>(row + C);
    const float4 gp = *reinterpret_cast<const float4*>(row + 2 * C);
    const float qa[4] = {q.x, q.y, q.z, q.w}, va[4] = {v.x, v.y, v.z, v.w}, ga[4] = {gp.x, gp.y, gp.z, gp.w};
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      h[i] = __fadd_rn(__fmul_rn(h[i], sigmoid_f(ga[i])), va[i]);
      o[i] = __fmul_rn(qa[i], h[i]);
    }
    *reinterpret_cast<float4*>(z + dst[t] * C + c) = make_float4(o[0], o[1], o[2], o[3]);
  }
}

// One thread per row (C <= 32).
__global__ void __launch_bounds__(256) ln_row_thread_kernel(const float* __restrict__ x, const float* __restrict__ r,
                                                            const float* __restrict__ w, const float* __restrict__ b,
                                                            int64_t rows, int C, float eps, float* __restrict__ out) {
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  float v[32];
  float s = 0.f;
  for (int i = 0; i < C; ++i) {
    v[i] = x[row * C + i] + (r ? r[row * C + i] : 0.f);
    s += v[i];
  }
  const float mean = s / C;
  float q = 0.f;
  for (int i = 0; i < C; ++i) {
    const float d = v[i] - mean;
    q = fmaf(d, d, q);
  }
  const float rstd = rsqrtf(q / C + eps);
  for (int i = 0; i < C; ++i) out[row * C + i] = (v[i] - mean) * rstd * w[i] + b[i];
}

// One warp per row (32 < C <= 1024): lane l holds channels l, l+32, ... below C.
__global__ void __launch_bounds__(256) ln_row_warp_kernel(const float* __restrict__ x, const float* __restrict__ r,
                                                          const float* __restrict__ w, const float* __restrict__ b,
                                                          int64_t rows, int C, float eps, float* __restrict__ out) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int n = (C + 31) >> 5;
  float v[32];
  float s = 0.f;
  for (int j = 0; j < n; ++j) {
    const int c = lane + 32 * j;
    const int64_t o = row * C + c;
    v[j] = c < C ? x[o] + (r ? r[o] : 0.f) : 0.f;
    s += v[j];
  }
#pragma unroll
  for (int k = 16; k > 0; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
  const float mean = s / C;
  float q = 0.f;
  for (int j = 0; j < n; ++j) {
    const float d = lane + 32 * j < C ? v[j] - mean : 0.f;
    q = fmaf(d, d, q);
  }
#pragma unroll
  for (int k = 16; k > 0; k >>= 1) q += __shfl_xor_sync(0xffffffffu, q, k);
  const float rstd = rsqrtf(q / C + eps);
  for (int j = 0; j < n; ++j) {
    const int c = lane + 32 * j;
    if (c < C) out[row * C + c] = (v[j] - mean) * rstd * w[c] + b[c];
  }
}

}  // namespace
}  // namespace ssla

using namespace ssla;

extern "C" int ssla_mos_patch_scan_fwd(const float* y, const int64_t* key, const int64_t* dst, const int64_t* cu,
                                       int64_t n_seqs, int64_t C, float* z, ssla_stream_t stream) {
  SSLA_CHECK_ARG(n_seqs >= 0 && C > 0 && C % 4 == 0, "ssla_mos_patch_scan_fwd: C=%lld must be a positive multiple of 4",
                 (long long)C);
  if (n_seqs == 0) return SSLA_OK;
  SSLA_CHECK_ARG(y && key && dst && cu && z, "ssla_mos_patch_scan_fwd: null pointer");
  SSLA_CHECK_ARG(aligned_to(y, 16) && aligned_to(z, 16), "ssla_mos_patch_scan_fwd: y and z must be 16-byte aligned");
  const int64_t threads = n_seqs * (C / 4);
  mos_patch_scan_kernel<<<(unsigned)ceil_div(threads, 256), 256, 0, (cudaStream_t)stream>>>(y, key, dst, cu, n_seqs, C,
                                                                                           z);
  SSLA_CHECK_LAUNCH("ssla_mos_patch_scan_fwd");
  return SSLA_OK;
}

extern "C" int ssla_layernorm_residual_fwd(const float* x, const float* r, const float* w, const float* b,
                                           int64_t rows, int64_t C, float eps, float* out, ssla_stream_t stream) {
  SSLA_CHECK_ARG(rows >= 0 && C >= 1 && C <= 1024, "ssla_layernorm_residual_fwd: C=%lld unsupported (1 .. 1024)",
                 (long long)C);
  if (rows == 0) return SSLA_OK;
  SSLA_CHECK_ARG(x && w && b && out, "ssla_layernorm_residual_fwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  if (C <= 32) {
    ln_row_thread_kernel<<<(unsigned)ceil_div(rows, 256), 256, 0, s>>>(x, r, w, b, rows, (int)C, eps, out);
  } else {
    ln_row_warp_kernel<<<(unsigned)ceil_div(rows * 32, 256), 256, 0, s>>>(x, r, w, b, rows, (int)C, eps, out);
  }
  SSLA_CHECK_LAUNCH("ssla_layernorm_residual_fwd");
  return SSLA_OK;
}
