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
// mos_patch_scan_proj: the same, with the projection computed in the kernel instead of read
// from y: [q | v | g_pre] = W[pos[t]] x[src[t]] with W [P, 3C, I] staged in shared memory as
// [P, 3, I, C] (float4 reads of 4 consecutive channels) and x the layer's input rows (I
// floats, read by all threads of a sequence at once).  One thread owns 4 channels of one
// sequence (each x element feeds 12 FMAs); events are taken U at a time so their loads and
// projections overlap, only the scan itself is serial.  Used when W fits in shared memory (the narrow, high-volume layers).
//
// rows_matmul: out[M, N] = A[M, K] @ B[K, N] (fp32) for the skinny shapes of the MoS layer
// (K or N of a few dozen: the folded scatter projection [events, I] x [I, P*3C] and the gather
// projection [events, P*C] x [P*C, C]), where a tiled library GEMM wastes most of its tile.
// Persistent blocks stage B once in shared memory; one thread owns one row, streams it in
// float4 pieces and accumulates 32 output columns at a time from broadcast float4 reads of B.
//
// layernorm_residual: out = LayerNorm(x + r) * w + b over rows of C channels (two-pass mean /
// variance in fp32).  Rows of up to 32 channels take one thread each, wider rows one warp.
#include "common.cuh"
#include "vec.cuh"

namespace ssla {
namespace {

__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }

// Patch event t of a sequence reads y row key(t) and writes z row dst(t).  INDEXED: both come
// from the key / dst arrays; otherwise they are formed from the routing's (src, pos) pair as
// key = src * P + pos (src when P == 1) and dst = src * Pg + pos (dst = t when Pg == 0), which
// saves the elementwise passes that would build the two index arrays.
template <bool INDEXED>
__global__ void __launch_bounds__(256) mos_patch_scan_kernel(const float* __restrict__ y,
                                                             const int64_t* __restrict__ key,
                                                             const int64_t* __restrict__ dst,
                                                             int64_t P, int64_t Pg,
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
    int64_t kt, dt;
    if (INDEXED) {
      kt = key[t];
      dt = dst[t];
    } else {  // key = src, dst = pos (possibly null)
      const int64_t sv = key[t], pv = dst ? dst[t] : 0;
      kt = P > 1 ? sv * P + pv : sv;
      dt = Pg > 0 ? sv * Pg + pv : t;
    }
    const float* row = y + kt * 3 * C + c;
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
    *reinterpret_cast<float4*>(z + dt * C + c) = make_float4(o[0], o[1], o[2], o[3]);
  }
}

constexpr int PS_U = 4;

// Shared-memory stride between positions: 3*I*C floats rounded up to 4 (mod 32), so the
// float4 reads of threads on different positions start in different 16-byte bank groups.
__host__ __device__ __forceinline__ int pstride(int I, int C) {
  const int n = 3 * I * C;
  return n + ((4 - n % 32) + 32) % 32;
}

__global__ void __launch_bounds__(256) mos_patch_scan_proj_kernel(
    const float* __restrict__ x, int I, const float* __restrict__ w, int P, const int64_t* __restrict__ src,
    const int64_t* __restrict__ pos, const int64_t* __restrict__ dst, const int64_t* __restrict__ cu, int64_t n_seqs,
    int C, float* __restrict__ z) {
  extern __shared__ float ws[];  // [P][3][I][C], position stride pstride(I, C) floats
  const int n_w = P * 3 * I * C;
  const int ps = pstride(I, C);
  for (int e = threadIdx.x; e < n_w; e += blockDim.x) {
    // e enumerates the global layout [P][3C][I]: p, row (= part * C + c), i
    const int i = e % I, pr = e / I, row = pr % (3 * C), p = pr / (3 * C);
    const int part = row / C, c = row % C;
    ws[p * ps + (part * I + i) * C + c] = w[e];
  }
  __syncthreads();
  // persistent: the grid covers the GPU once and strides over (sequence, 4-channel group)
  // pairs, so the weights are staged once per block
  const int CV = C >> 2;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n_seqs * CV;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t seq = idx / CV;
    const int c = (int)(idx - seq * CV) << 2;
    const int64_t bos = cu[seq], eos = cu[seq + 1];
    float h[4] = {0.f, 0.f, 0.f, 0.f};
    for (int64_t t0 = bos; t0 < eos; t0 += PS_U) {
      const int n = (int)((eos - t0) < PS_U ? (eos - t0) : PS_U);
      float4 q[PS_U], v[PS_U], g[PS_U];
      int64_t d[PS_U];
#pragma unroll
      for (int u = 0; u < PS_U; ++u) {
        q[u] = v[u] = g[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        d[u] = 0;
        if (u < n) {
          const float* xr = x + src[t0 + u] * I;
          const float* wp = ws + (int)pos[t0 + u] * ps + c;
          d[u] = dst[t0 + u];
          for (int i = 0; i < I; ++i) {
            const float xi = xr[i];
            const float4 wq = *reinterpret_cast<const float4*>(wp + i * C);
            const float4 wv = *reinterpret_cast<const float4*>(wp + (I + i) * C);
            const float4 wg = *reinterpret_cast<const float4*>(wp + (2 * I + i) * C);
            q[u].x = fmaf(wq.x, xi, q[u].x); q[u].y = fmaf(wq.y, xi, q[u].y);
            q[u].z = fmaf(wq.z, xi, q[u].z); q[u].w = fmaf(wq.w, xi, q[u].w);
            v[u].x = fmaf(wv.x, xi, v[u].x); v[u].y = fmaf(wv.y, xi, v[u].y);
            v[u].z = fmaf(wv.z, xi, v[u].z); v[u].w = fmaf(wv.w, xi, v[u].w);
            g[u].x = fmaf(wg.x, xi, g[u].x); g[u].y = fmaf(wg.y, xi, g[u].y);
            g[u].z = fmaf(wg.z, xi, g[u].z); g[u].w = fmaf(wg.w, xi, g[u].w);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < PS_U; ++u) {
        if (u < n) {
          const float qa[4] = {q[u].x, q[u].y, q[u].z, q[u].w}, va[4] = {v[u].x, v[u].y, v[u].z, v[u].w},
                      ga[4] = {g[u].x, g[u].y, g[u].z, g[u].w};
          float o[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            h[k] = __fadd_rn(__fmul_rn(h[k], sigmoid_f(ga[k])), va[k]);
            o[k] = __fmul_rn(qa[k], h[k]);
          }
          *reinterpret_cast<float4*>(z + d[u] * C + c) = make_float4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
}

constexpr int RM_THREADS = 128, RM_NC = 32;

template <bool VEC_A>
__global__ void __launch_bounds__(RM_THREADS) rows_matmul_kernel(const float* __restrict__ A, int64_t M, int K, int64_t lda,
                                                                 const float* __restrict__ B, int N,
                                                                 float* __restrict__ out, int64_t ldo) {
  extern __shared__ float bs[];  // [K][Np], Np = N rounded up to RM_NC (zero padded)
  const int Np = (N + RM_NC - 1) / RM_NC * RM_NC;
  for (int e = threadIdx.x; e < K * Np; e += RM_THREADS) {
    const int k = e / Np, n = e - k * Np;
    bs[e] = n < N ? B[(int64_t)k * N + n] : 0.f;
  }
  __syncthreads();
  for (int64_t row = (int64_t)blockIdx.x * RM_THREADS + threadIdx.x; row < M; row += (int64_t)gridDim.x * RM_THREADS) {
    const float* a = A + row * lda;
    float* o = out + row * ldo;
    for (int n0 = 0; n0 < N; n0 += RM_NC) {
      float acc[RM_NC];
#pragma unroll
      for (int j = 0; j < RM_NC; ++j) acc[j] = 0.f;
      int k = 0;
      if (VEC_A) {
        for (; k + 4 <= K; k += 4) {
          const float4 av = *reinterpret_cast<const float4*>(a + k);
          const float ak[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const float* br = bs + (k + kk) * Np + n0;
#pragma unroll
            for (int j = 0; j < RM_NC; j += 4) {
              const float4 b = *reinterpret_cast<const float4*>(br + j);
              acc[j] = fmaf(ak[kk], b.x, acc[j]);
              acc[j + 1] = fmaf(ak[kk], b.y, acc[j + 1]);
              acc[j + 2] = fmaf(ak[kk], b.z, acc[j + 2]);
              acc[j + 3] = fmaf(ak[kk], b.w, acc[j + 3]);
            }
          }
        }
      }
      for (; k < K; ++k) {
        const float ak = a[k];
        const float* br = bs + k * Np + n0;
#pragma unroll
        for (int j = 0; j < RM_NC; j += 4) {
          const float4 b = *reinterpret_cast<const float4*>(br + j);
          acc[j] = fmaf(ak, b.x, acc[j]);
          acc[j + 1] = fmaf(ak, b.y, acc[j + 1]);
          acc[j + 2] = fmaf(ak, b.z, acc[j + 2]);
          acc[j + 3] = fmaf(ak, b.w, acc[j + 3]);
        }
      }
      const int nn = N - n0 < RM_NC ? N - n0 : RM_NC;
      if (nn == RM_NC && ((reinterpret_cast<uintptr_t>(o + n0) & 15) == 0)) {
#pragma unroll
        for (int j = 0; j < RM_NC; j += 4)
          *reinterpret_cast<float4*>(o + n0 + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < RM_NC; ++j)
          if (j < nn) o[n0 + j] = acc[j];
      }
    }
  }
}

// One thread per row (C <= 32).
// Rows of C = 4 * L floats (L <= 32 lanes of one float4 each), GP lanes per row (GP the power
// of two >= L): coalesced 16-byte loads of x and r, mean and variance (two passes over the
// registers) reduced by xor shuffles inside the lane group.
template <int GP>
__global__ void __launch_bounds__(256) ln_row_vec4_kernel(const float* __restrict__ x, const float* __restrict__ r,
                                                          const float* __restrict__ w, const float* __restrict__ b,
                                                          int64_t rows, int C, float eps, float* __restrict__ out) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = t / GP;
  const int gl = (int)(t % GP);
  const int L = C >> 2;
  const bool on = row < rows && gl < L;
  const int64_t o = row * C + 4 * gl;
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (on) {
    v = *reinterpret_cast<const float4*>(x + o);
    if (r) {
      const float4 u = *reinterpret_cast<const float4*>(r + o);
      v.x += u.x;
      v.y += u.y;
      v.z += u.z;
      v.w += u.w;
    }
  }
  float s = (v.x + v.y) + (v.z + v.w);
#pragma unroll
  for (int k = GP / 2; k > 0; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k, GP);
  const float mean = s / C;
  const float dx = v.x - mean, dy = v.y - mean, dz = v.z - mean, dw = v.w - mean;
  float q = on ? fmaf(dx, dx, fmaf(dy, dy, fmaf(dz, dz, dw * dw))) : 0.f;
#pragma unroll
  for (int k = GP / 2; k > 0; k >>= 1) q += __shfl_xor_sync(0xffffffffu, q, k, GP);
  const float rstd = rsqrtf(q / C + eps);
  if (!on) return;
  const float4 ww = *reinterpret_cast<const float4*>(w + 4 * gl), bb = *reinterpret_cast<const float4*>(b + 4 * gl);
  *reinterpret_cast<float4*>(out + o) =
      make_float4(dx * rstd * ww.x + bb.x, dy * rstd * ww.y + bb.y, dz * rstd * ww.z + bb.z, dw * rstd * ww.w + bb.w);
}

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
  mos_patch_scan_kernel<true><<<(unsigned)ceil_div(threads, 256), 256, 0, (cudaStream_t)stream>>>(
      y, key, dst, 0, 0, cu, n_seqs, C, z);
  SSLA_CHECK_LAUNCH("ssla_mos_patch_scan_fwd");
  return SSLA_OK;
}

extern "C" int ssla_mos_patch_scan_routed_fwd(const float* y, const int64_t* src, const int64_t* pos, int64_t P,
                                              int64_t Pg, const int64_t* cu, int64_t n_seqs, int64_t C, float* z,
                                              ssla_stream_t stream) {
  SSLA_CHECK_ARG(n_seqs >= 0 && C > 0 && C % 4 == 0 && P >= 1 && Pg >= 0,
                 "ssla_mos_patch_scan_routed_fwd: bad sizes (C=%lld must be a positive multiple of 4)", (long long)C);
  if (n_seqs == 0) return SSLA_OK;
  SSLA_CHECK_ARG(y && src && cu && z && (pos || (P == 1 && Pg <= 1)), "ssla_mos_patch_scan_routed_fwd: null pointer");
  SSLA_CHECK_ARG(aligned_to(y, 16) && aligned_to(z, 16),
                 "ssla_mos_patch_scan_routed_fwd: y and z must be 16-byte aligned");
  const int64_t threads = n_seqs * (C / 4);
  mos_patch_scan_kernel<false><<<(unsigned)ceil_div(threads, 256), 256, 0, (cudaStream_t)stream>>>(
      y, src, pos, P, Pg, cu, n_seqs, C, z);
  SSLA_CHECK_LAUNCH("ssla_mos_patch_scan_routed_fwd");
  return SSLA_OK;
}

extern "C" size_t ssla_mos_patch_scan_proj_smem_bytes(int64_t P, int64_t C, int64_t I) {
  return (size_t)(P * pstride((int)I, (int)C)) * sizeof(float);
}

extern "C" int ssla_mos_patch_scan_proj_fwd(const float* x, int64_t I, const float* w, int64_t P, const int64_t* src,
                                            const int64_t* pos, const int64_t* dst, const int64_t* cu, int64_t n_seqs,
                                            int64_t C, float* z, ssla_stream_t stream) {
  SSLA_CHECK_ARG(n_seqs >= 0 && C > 0 && C % 4 == 0 && I > 0 && P > 0,
                 "ssla_mos_patch_scan_proj_fwd: bad sizes (C must be a multiple of 4)");
  const size_t smem = ssla_mos_patch_scan_proj_smem_bytes(P, C, I);
  SSLA_CHECK_ARG(smem <= 200 * 1024, "ssla_mos_patch_scan_proj_fwd: weights of %zu bytes exceed shared memory", smem);
  if (n_seqs == 0) return SSLA_OK;
  SSLA_CHECK_ARG(x && w && src && pos && dst && cu && z, "ssla_mos_patch_scan_proj_fwd: null pointer");
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(mos_patch_scan_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess) {
    set_error("ssla_mos_patch_scan_proj_fwd: cannot reserve %zu bytes of shared memory", smem);
    return SSLA_ERR_CUDA;
  }
  int dev = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mos_patch_scan_proj_kernel, 256, smem) != cudaSuccess ||
      per_sm < 1) {
    set_error("ssla_mos_patch_scan_proj_fwd: occupancy query failed");
    return SSLA_ERR_CUDA;
  }
  const int64_t blocks = ceil_div(n_seqs * (C / 4), 256);
  const int64_t cap = (int64_t)per_sm * sms;
  mos_patch_scan_proj_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, smem, (cudaStream_t)stream>>>(
      x, (int)I, w, (int)P, src, pos, dst, cu, n_seqs, (int)C, z);
  SSLA_CHECK_LAUNCH("ssla_mos_patch_scan_proj_fwd");
  return SSLA_OK;
}

extern "C" size_t ssla_rows_matmul_smem_bytes(int64_t K, int64_t N) {
  return (size_t)K * (size_t)((N + RM_NC - 1) / RM_NC * RM_NC) * sizeof(float);
}

extern "C" int ssla_rows_matmul_f32(const float* A, int64_t M, int64_t K, int64_t lda, const float* B, int64_t N,
                                    float* out, int64_t ldo, ssla_stream_t stream) {
  SSLA_CHECK_ARG(M >= 0 && K > 0 && N > 0 && lda >= K && ldo >= N, "ssla_rows_matmul_f32: bad sizes");
  const size_t smem = ssla_rows_matmul_smem_bytes(K, N);
  SSLA_CHECK_ARG(smem <= 96 * 1024, "ssla_rows_matmul_f32: B of %zu bytes exceeds shared memory", smem);
  if (M == 0) return SSLA_OK;
  SSLA_CHECK_ARG(A && B && out, "ssla_rows_matmul_f32: null pointer");
  const bool vec = lda % 4 == 0 && aligned_to(A, 16);
  auto launch = [&](auto kern) -> int {
    if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
      set_error("ssla_rows_matmul_f32: cannot reserve %zu bytes of shared memory", smem);
      return SSLA_ERR_CUDA;
    }
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, RM_THREADS, smem) != cudaSuccess || per_sm < 1)
      per_sm = 1;
    const int64_t blocks = ceil_div(M, RM_THREADS);
    const int64_t cap = (int64_t)per_sm * sms;
    kern<<<(unsigned)(blocks < cap ? blocks : cap), RM_THREADS, smem, (cudaStream_t)stream>>>(A, M, (int)K, lda, B,
                                                                                            (int)N, out, ldo);
    SSLA_CHECK_LAUNCH("ssla_rows_matmul_f32");
    return SSLA_OK;
  };
  return vec ? launch(rows_matmul_kernel<true>) : launch(rows_matmul_kernel<false>);
}

extern "C" int ssla_layernorm_residual_fwd(const float* x, const float* r, const float* w, const float* b,
                                           int64_t rows, int64_t C, float eps, float* out, ssla_stream_t stream) {
  SSLA_CHECK_ARG(rows >= 0 && C >= 1 && C <= 1024, "ssla_layernorm_residual_fwd: C=%lld unsupported (1 .. 1024)",
                 (long long)C);
  if (rows == 0) return SSLA_OK;
  SSLA_CHECK_ARG(x && w && b && out, "ssla_layernorm_residual_fwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const bool vec4 = C % 4 == 0 && C <= 128 && ((uintptr_t)x | (uintptr_t)r | (uintptr_t)w | (uintptr_t)b |
                                                (uintptr_t)out) % 16 == 0;
  if (vec4) {
    const int L = (int)(C / 4);
    const int GP = L <= 1 ? 1 : L <= 2 ? 2 : L <= 4 ? 4 : L <= 8 ? 8 : L <= 16 ? 16 : 32;
    const unsigned grid = (unsigned)ceil_div(rows * GP, 256);
    switch (GP) {
      case 1: ln_row_vec4_kernel<1><<<grid, 256, 0, s>>>(x, r, w, b, rows, (int)C, eps, out); break;
      case 2: ln_row_vec4_kernel<2><<<grid, 256, 0, s>>>(x, r, w, b, rows, (int)C, eps, out); break;
      case 4: ln_row_vec4_kernel<4><<<grid, 256, 0, s>>>(x, r, w, b, rows, (int)C, eps, out); break;
      case 8: ln_row_vec4_kernel<8><<<grid, 256, 0, s>>>(x, r, w, b, rows, (int)C, eps, out); break;
      case 16: ln_row_vec4_kernel<16><<<grid, 256, 0, s>>>(x, r, w, b, rows, (int)C, eps, out); break;
      default: ln_row_vec4_kernel<32><<<grid, 256, 0, s>>>(x, r, w, b, rows, (int)C, eps, out); break;
    }
  } else if (C <= 32) {
    ln_row_thread_kernel<<<(unsigned)ceil_div(rows, 256), 256, 0, s>>>(x, r, w, b, rows, (int)C, eps, out);
  } else {
    ln_row_warp_kernel<<<(unsigned)ceil_div(rows * 32, 256), 256, 0, s>>>(x, r, w, b, rows, (int)C, eps, out);
  }
  SSLA_CHECK_LAUNCH("ssla_layernorm_residual_fwd");
  return SSLA_OK;
}
