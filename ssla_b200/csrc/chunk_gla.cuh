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
  longlong2* chunk_tab;  // [MC]  per global chunk: {first token, valid rows | seq << 32}; seq -1 = none
  float* dS;           // [MC,H,K,V]  per-chunk state increment (fwd) / its adjoint (bwd)
  float* decay;        // [MC,H,K]    exp(g summed over the chunk)
  float* dstates;      // [MC,H,K,V]  adjoint of the state at the end of each chunk (bwd)
  int* flags;          // [1+MC*H]    [0] = number of (chunk, head) items left to the exact
                       //             CUDA-core kernels, then their ids chunk*H + head
};

inline size_t workspace_bytes(int64_t N, int64_t T, int64_t H, int64_t K, int64_t V) {
  const int64_t MC = max_chunks(N, T);
  return align256(8 * (N + 1)) + align256(16 * (size_t)(MC > 0 ? MC : 1)) +
         2 * align256(4 * (size_t)MC * H * K * V) +
         align256(4 * (size_t)MC * H * K) + align256(4 * ((size_t)MC * H + 1));
}

inline Workspace carve(void* base, int64_t N, int64_t T, int64_t H, int64_t K, int64_t V) {
  const int64_t MC = max_chunks(N, T);
  char* p = (char*)base;
  Workspace w;
  w.chunk_off = (int64_t*)p;
  p += align256(8 * (N + 1));
  w.chunk_tab = (longlong2*)p;
  p += align256(16 * (size_t)(MC > 0 ? MC : 1));
  w.dS = (float*)p;
  p += align256(4 * (size_t)MC * H * K * V);
  w.dstates = (float*)p;
  p += align256(4 * (size_t)MC * H * K * V);
  w.decay = (float*)p;
  p += align256(4 * (size_t)MC * H * K);
  w.flags = (int*)p;
  return w;
}

// Resolve global chunk id -> (sequence, first token, valid rows) through the chunk table
// written by launch_chunk_offsets (one load).  Returns false for ids beyond the last chunk.
__device__ __forceinline__ bool locate_chunk(int64_t cid, const longlong2* __restrict__ tab,
                                             int64_t& seq, int64_t& t0, int& len) {
  const longlong2 e = tab[cid];
  seq = e.y >> 32;
  if (seq < 0) return false;
  t0 = e.x;
  len = (int)(e.y & 0xffffffff);
  return true;
}

// Host launchers shared by the CUDA-core and tensor-core implementations (chunk_gla.cu).
// Also resets the exact-item count flags[0] of the call.
int launch_chunk_offsets(const int64_t* cu, int64_t N, int64_t MC, int64_t* chunk_off,
                         longlong2* chunk_tab, int* flags, cudaStream_t s);
int launch_state_scan(const float* dS, const float* decay, const int64_t* chunk_off, int64_t N,
                      int64_t H, int64_t K, int64_t V, const float* init, float* per_chunk,
                      float* final_state, bool reverse, cudaStream_t s);

// CUDA-core per-chunk kernels (chunk_gla.cu).  With `flags` non-null only the items listed
// there are processed (fallback of the tensor-core kernels).
int simt_fwd_o(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
               const int64_t* cu, const longlong2* chunk_tab, int64_t N, int64_t MC, int64_t H,
               int64_t K, int64_t V, float scale, const float* states, void* o, const int* flags,
               cudaStream_t s);
int simt_bwd(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
             const int64_t* cu, const longlong2* chunk_tab, int64_t N, int64_t MC, int64_t H,
             int64_t K, int64_t V, float scale, const float* states, const float* dstates,
             const void* dout, void* dq, void* dk, void* dv, float* dg, const int* flags,
             cudaStream_t s);

// Tensor-core (tcgen05) implementation for 16-bit inputs with K = V = 64 (chunk_gla_tc.cu).
// tc_fwd_o / tc_bwd append the items they leave to the exact kernels to `flags`.
int tc_supported(int dtype, int dtype_g, int64_t K, int64_t V);
// 1 when every pointer is 16-byte aligned (TMA base addresses).
int tc_aligned(const void* const* ptrs, int n);
int tc_local_state(int dtype, int dtype_g, int mode, const void* a_src, const void* b_src, const void* g,
                   const longlong2* chunk_tab, int64_t T, int64_t MC, int64_t H, float scale, float* dS,
                   float* decay, cudaStream_t s);
int tc_fwd_o(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
             const longlong2* chunk_tab, int64_t T, int64_t MC, int64_t H, float scale, const float* states,
             void* o, int* flags, cudaStream_t s);
int tc_bwd(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
           const longlong2* chunk_tab, int64_t T, int64_t MC, int64_t H, float scale, const float* states,
           const float* dstates, const void* dout, void* dq, void* dk, void* dv, float* dg, int* flags,
           cudaStream_t s);

}  // namespace chunk
}  // namespace ssla
