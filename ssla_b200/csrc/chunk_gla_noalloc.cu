// chunk_gla forward for callers that must not allocate device memory.
//
// Some hosts embed this library where cudaMalloc is off limits: a serving process whose
// memory is fully carved up by its own pool before the model loads, or a plugin that is
// handed only input/output buffers by a runtime that owns all allocations.  The regular
// ssla_chunk_gla_fwd needs a caller-provided workspace and `states` buffer; this variant
// takes only inputs and outputs and uses a fixed scratch array that is part of the library
// image instead.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes (64 MiB), so every GPU
// that loads the library holds those 64 MiB until the process exits.  Calls whose scratch
// need (the forward's states buffer plus its workspace) exceeds it are rejected with
// SSLA_ERR_WORKSPACE.  All calls on one device share the
// array: two calls that overlap on the GPU (different streams, or host threads racing) would
// corrupt each other's intermediates, so serialise them (one stream, or events).  The forward
// writes every scratch byte it later reads, so nothing has to be cleared between calls.
#include <mutex>

#include "chunk_gla.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device.  The host-side symbol
// g_noalloc_scratch is only a stand-in and must never be passed to a kernel; the real
// address comes from cudaGetSymbolAddress with the device current.  Done once per device,
// on that device's first call (which therefore should not happen during stream capture).
// The address is kept for the life of the process: after cudaDeviceReset on a device the
// cached address is stale, so this entry point must not be used on that device again.
int scratch_on_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    ssla::set_error("ssla_chunk_gla_fwd_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(e));
    return SSLA_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    ssla::set_error("ssla_chunk_gla_fwd_noalloc: device %d out of range", dev);
    return SSLA_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      ssla::set_error("ssla_chunk_gla_fwd_noalloc: cudaGetSymbolAddress failed: %s",
                      cudaGetErrorString(e));
      return SSLA_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return SSLA_OK;
}

}  // namespace

extern "C" int ssla_chunk_gla_fwd_noalloc(const void* q, const void* k, const void* v,
                                          const void* g, int dtype, int dtype_g,
                                          const int64_t* cu_seqlens, int64_t n_seqs, int64_t T,
                                          int64_t H, int64_t K, int64_t V, float scale,
                                          const float* h0, void* o, float* ht,
                                          ssla_stream_t stream) {
  using namespace ssla::chunk;
  // the regular entry point's argument checks first, so the size arithmetic below only sees
  // valid dtypes and 1 <= K, V <= 64
  if (!ssla::dtype_ok(dtype) || (dtype_g != dtype && dtype_g != SSLA_F32)) {
    ssla::set_error("ssla_chunk_gla_fwd_noalloc: bad dtype");
    return SSLA_ERR_INVALID_ARG;
  }
  if (n_seqs < 0 || T < 0 || H < 0 || K < 1 || V < 1 || K > 64 || V > 64) {
    ssla::set_error("ssla_chunk_gla_fwd_noalloc: bad size (N, T, H >= 0 and 1 <= K, V <= 64)");
    return SSLA_ERR_INVALID_ARG;
  }
  // Bound the chunk count by division before multiplying: every (chunk, head) needs at least
  // K*V*4 bytes of scratch, so more than kNoAllocScratchBytes / (4*K*V) of them cannot fit.
  // n_seqs and T are bounded first so that max_chunks() cannot overflow.
  const int64_t lim = (int64_t)kNoAllocScratchBytes;
  const int64_t MC = (n_seqs > lim || T > lim) ? lim : max_chunks(n_seqs, T);
  const bool fits = H == 0 || MC == 0 || MC <= lim / (4 * K * V) / H;
  const bool tc = tc_shape(dtype, dtype_g, K, V);
  const size_t st = fits ? saved_bytes(n_seqs, T, H, K, V, tc) : 0;
  const size_t ws = fits ? fwd_workspace_bytes(n_seqs, T, H, K, V) : 0;
  if (!fits || st + ws > kNoAllocScratchBytes) {
    ssla::set_error(
        "ssla_chunk_gla_fwd_noalloc: this shape needs more scratch than the %zu-byte built-in "
        "limit; use ssla_chunk_gla_fwd with caller-allocated buffers",
        kNoAllocScratchBytes);
    return SSLA_ERR_WORKSPACE;
  }
  void* base = nullptr;
  int rc = scratch_on_current_device(&base);
  if (rc) return rc;
  void* states = base;
  void* workspace = (char*)base + st;
  return ssla_chunk_gla_fwd(q, k, v, g, dtype, dtype_g, cu_seqlens, n_seqs, T, H, K, V, scale, h0,
                            o, ht, states, st, workspace, ws, stream);
}
