// Shared definitions of the chunked GLA path (forward + backward).
//
// Tokens of each sequence are cut into chunks of BT = 64 (the last chunk of a sequence may
// be shorter).  A global chunk id enumerates the chunks of all sequences in order;
// chunk_off[n] is the first global chunk of sequence n (exclusive scan of ceil(len/64)),
// computed on the device so that no host synchronisation is needed.  Kernels are launched
// over the upper bound max_chunks = (T + 63 N) / 64 and idle CTAs exit.
#pragma once
#include "common.cuh"

namespace ssla {
namespace chunk {

constexpr int BT = 64;   // tokens per chunk
constexpr int BC = 16;   // sub-chunk rows (gate reference granularity)
constexpr int NC = BT / BC;
// A sub-chunk whose in-chunk log-decay span exceeds this uses exact per-element exponents
// instead of the factorised exp(gc_i - ref) * exp(ref - gc_j) form (guards fp overflow).
constexpr float kSpanLimit = 60.f;

inline int64_t max_chunks(int64_t N, int64_t T) { return (T + 63 * N) / BT; }

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Workspace {
  int64_t* chunk_off;  // [N+1]
  float* dS;           // [MC,H,K,V]  per-chunk state increment (fwd) / its adjoint (bwd)
  float* decay;        // [MC,H,K]    exp(g summed over the chunk)
  float* dstates;      // [MC,H,K,V]  adjoint of the state at the end of each chunk (bwd)
};

inline size_t workspace_bytes(int64_t N, int64_t T, int64_t H, int64_t K, int64_t V) {
  const int64_t MC = max_chunks(N, T);
  return align256(8 * (N + 1)) + 2 * align256(4 * (size_t)MC * H * K * V) +
         align256(4 * (size_t)MC * H * K);
}

inline Workspace carve(void* base, int64_t N, int64_t T, int64_t H, int64_t K, int64_t V) {
  const int64_t MC = max_chunks(N, T);
  char* p = (char*)base;
  Workspace w;
  w.chunk_off = (int64_t*)p;
  p += align256(8 * (N + 1));
  w.dS = (float*)p;
  p += align256(4 * (size_t)MC * H * K * V);
  w.dstates = (float*)p;
  p += align256(4 * (size_t)MC * H * K * V);
  w.decay = (float*)p;
  return w;
}

// Resolve global chunk id -> (sequence, first token, valid rows).  Returns false for ids
// beyond the last chunk.
__device__ __forceinline__ bool locate_chunk(int64_t cid, const int64_t* __restrict__ chunk_off,
                                             const int64_t* __restrict__ cu, int64_t N,
                                             int64_t& seq, int64_t& t0, int& len) {
  if (cid >= chunk_off[N]) return false;
  int64_t lo = 0, hi = N - 1;  // last n with chunk_off[n] <= cid
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (chunk_off[mid] <= cid) lo = mid; else hi = mid - 1;
  }
  seq = lo;
  t0 = cu[lo] + (cid - chunk_off[lo]) * BT;
  const int64_t rem = cu[lo + 1] - t0;
  len = (int)(rem < BT ? rem : BT);
  return true;
}

// Host launchers shared by the CUDA-core and tensor-core implementations (chunk_gla.cu).
int launch_chunk_offsets(const int64_t* cu, int64_t N, int64_t* chunk_off, cudaStream_t s);
int launch_state_scan(const float* dS, const float* decay, const int64_t* chunk_off, int64_t N,
                      int64_t H, int64_t K, int64_t V, const float* init, float* per_chunk,
                      float* final_state, bool reverse, cudaStream_t s);

// Tensor-core (tcgen05) implementation for 16-bit inputs (chunk_gla_tc.cu).
int tc_supported(int dtype, int dtype_g, int64_t K, int64_t V);
int tc_local_state(int dtype, int dtype_g, int mode, const void* a_src, const void* b_src,
                   const void* g, const int64_t* cu, const int64_t* chunk_off, int64_t N,
                   int64_t MC, int64_t H, float scale, float* dS, float* decay, cudaStream_t s);
int tc_fwd_o(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
             const int64_t* cu, const int64_t* chunk_off, int64_t N, int64_t MC, int64_t H,
             float scale, const float* states, void* o, cudaStream_t s);
int tc_bwd(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
           const int64_t* cu, const int64_t* chunk_off, int64_t N, int64_t MC, int64_t H,
           float scale, const float* states, const float* dstates, const void* dout, void* dq,
           void* dk, void* dv, float* dg, cudaStream_t s);

}  // namespace chunk
}  // namespace ssla
