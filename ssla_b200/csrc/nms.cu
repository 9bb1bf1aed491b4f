// Batched greedy non-maximum suppression for the detection post-processing
// (MosModel.postprocess_with_nms, model_mos.py:232-299, which calls torchvision's nms on
// class-offset boxes, model_mos.py:20-29).
//
// One block per image:
//   1. candidates (score >= conf when filtering) are keyed (score bits, index) and sorted by
//      a shared-memory bitonic sort: descending score, ascending index among equal scores;
//   2. the upper triangle of the pairwise suppression matrix (IoU > threshold, IoU =
//      inter / (area_a + area_b - inter) in fp32 with IEEE division, the formula of
//      torchvision's nms) is written as 64-bit row masks to a global scratch;
//   3. one warp walks the sorted candidates keeping every box not yet suppressed and OR-ing
//      its mask row into the suppressed set, until max_det boxes are kept.
// Output: kept anchor indices in score order and their count per image.
#include "common.cuh"
#include "vec.cuh"

namespace ssla {
namespace {

constexpr int NMS_THREADS = 1024, NMS_MAXN = 4096, NMS_WORDS = NMS_MAXN / 64;

// Orderable unsigned image of a float (larger float -> larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float iou(const float4& a, const float4& b) {
  const float w = fmaxf(0.f, __fsub_rn(fminf(a.z, b.z), fmaxf(a.x, b.x)));
  const float h = fmaxf(0.f, __fsub_rn(fminf(a.w, b.w), fmaxf(a.y, b.y)));
  const float inter = __fmul_rn(w, h);
  const float sa = __fmul_rn(__fsub_rn(a.z, a.x), __fsub_rn(a.w, a.y));
  const float sb = __fmul_rn(__fsub_rn(b.z, b.x), __fsub_rn(b.w, b.y));
  return __fdiv_rn(inter, __fsub_rn(__fadd_rn(sa, sb), inter));
}

__global__ void __launch_bounds__(NMS_THREADS) nms_kernel(const float* __restrict__ boxes, const float* __restrict__ scores,
                                                          int N, int filtering, float conf, float iou_thr, int max_det,
                                                          unsigned long long* __restrict__ masks,
                                                          int64_t* __restrict__ keep, int64_t* __restrict__ count) {
  __shared__ unsigned long long key[NMS_MAXN];
  __shared__ unsigned long long removed[NMS_WORDS];
  __shared__ int s_n;
  const int b = blockIdx.x, tid = threadIdx.x;
  const float* sc = scores + (int64_t)b * N;
  const float4* bx = reinterpret_cast<const float4*>(boxes) + (int64_t)b * N;
  int P = 1;
  while (P < N) P <<= 1;
  // 1. keys: valid -> (score key << 32) | ~index (descending sort gives ascending index on ties)
  for (int i = tid; i < P; i += NMS_THREADS) {
    unsigned long long k = 0ull;
    if (i < N && (!filtering || sc[i] >= conf))
      k = ((unsigned long long)float_key(sc[i]) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)i);
    key[i] = k;
  }
  if (tid == 0) s_n = 0;
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < P; i += NMS_THREADS) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;  // descending runs first: the final order is descending
          const unsigned long long a = key[i], c = key[j];
          if (desc ? (a < c) : (a > c)) {
            key[i] = c;
            key[j] = a;
          }
        }
      }
      __syncthreads();
    }
  for (int i = tid; i < P; i += NMS_THREADS)
    if (key[i] != 0ull && (i + 1 == P || key[i + 1] == 0ull)) s_n = i + 1;  // number of valid keys
  __syncthreads();
  const int n = s_n;
  const int words = (n + 63) / 64;
  unsigned long long* M = masks + (int64_t)b * NMS_MAXN * NMS_WORDS;
  // 2. suppression masks of the sorted candidates (row r: bits of later candidates it suppresses)
  for (int e = tid; e < n * words; e += NMS_THREADS) {
    const int r = e / words, w = e - r * words;
    const float4 a = bx[0xffffffffu - (uint32_t)(key[r] & 0xffffffffu)];
    unsigned long long m = 0ull;
    for (int t = 0; t < 64; ++t) {
      const int c = w * 64 + t;
      if (c > r && c < n && iou(a, bx[0xffffffffu - (uint32_t)(key[c] & 0xffffffffu)]) > iou_thr) m |= 1ull << t;
    }
    M[(int64_t)r * NMS_WORDS + w] = m;
  }
  for (int w = tid; w < NMS_WORDS; w += NMS_THREADS) removed[w] = 0ull;
  __syncthreads();
  // 3. greedy pass (warp 0)
  if (tid < 32) {
    int kept = 0;
    for (int r = 0; r < n && kept < max_det; ++r) {
      const bool alive = ((removed[r >> 6] >> (r & 63)) & 1ull) == 0ull;
      if (alive) {
        if (tid == 0) keep[(int64_t)b * max_det + kept] = 0xffffffffu - (uint32_t)(key[r] & 0xffffffffu);
        ++kept;
        for (int w = tid; w < words; w += 32) removed[w] |= M[(int64_t)r * NMS_WORDS + w];
      }
      __syncwarp();
    }
    if (tid == 0) count[b] = kept;
  }
}

}  // namespace
}  // namespace ssla

using namespace ssla;

extern "C" size_t ssla_batched_nms_workspace_bytes(int64_t B) {
  return (size_t)B * NMS_MAXN * NMS_WORDS * sizeof(unsigned long long);
}

extern "C" int ssla_batched_nms(const float* boxes, const float* scores, int64_t B, int64_t N, int filtering, float conf,
                                float iou_thr, int64_t max_det, int64_t* keep, int64_t* count, void* workspace,
                                size_t workspace_bytes, ssla_stream_t stream) {
  SSLA_CHECK_ARG(B >= 0 && N >= 0 && N <= NMS_MAXN && max_det > 0,
                 "ssla_batched_nms: N=%lld must be at most %d, max_det positive", (long long)N, NMS_MAXN);
  if (B == 0) return SSLA_OK;
  SSLA_CHECK_ARG(boxes && scores && keep && count && workspace, "ssla_batched_nms: null pointer");
  SSLA_CHECK_ARG(aligned_to(boxes, 16), "ssla_batched_nms: boxes must be 16-byte aligned [B, N, 4] fp32");
  if (workspace_bytes < ssla_batched_nms_workspace_bytes(B)) {
    set_error("ssla_batched_nms: workspace of %zu bytes < %zu needed", workspace_bytes, ssla_batched_nms_workspace_bytes(B));
    return SSLA_ERR_WORKSPACE;
  }
  nms_kernel<<<(unsigned)B, NMS_THREADS, 0, (cudaStream_t)stream>>>(boxes, scores, (int)N, filtering, conf, iou_thr,
                                                                    (int)max_det, (unsigned long long*)workspace, keep,
                                                                    count);
  SSLA_CHECK_LAUNCH("ssla_batched_nms");
  return SSLA_OK;
}
