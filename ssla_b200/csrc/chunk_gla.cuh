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

// Tensor-core path: 16-bit inputs (bf16 / f16), gates of that dtype or fp32, K = V = 64.
inline bool tc_shape(int dtype, int dtype_g, int64_t K, int64_t V) {
  return (dtype == SSLA_BF16 || dtype == SSLA_F16) && (dtype_g == dtype || dtype_g == SSLA_F32) && K == 64 &&
         V == 64;
}

// What the forward leaves for the backward (the caller's `states` buffer).
//  * the chunk table of the call (so the backward needs no table pass);
//  * xflag [MC*H]: 1 for a (chunk, head) whose in-chunk decay range is too wide for the
//    tensor-core kernels' single-reference exponent factorisation (recomputed by the exact
//    CUDA-core kernels), written by the forward's local-state pass, which also lists those
//    items in xlist ([0] = count, zeroed by the chunk-table pass, then the item ids);
//  * h32 [MC,H,K,V] fp32: state at every chunk start.  On the tensor-core path only the
//    entries of flagged items are written (the exact kernels' input);
//  * h16 [MC,H,K,V] 16-bit (tensor-core path): H' = exp(ref) h, the state already scaled by
//    the chunk's reference decay (ref = in-chunk cumulative gate of row 31) in the operand
//    dtype, i.e. the B operand of the output / backward MMAs.
struct Saved {
  int64_t* chunk_off;    // [N+1]
  longlong2* chunk_tab;  // [MC]  per global chunk: {first token, valid rows | seq << 32}; seq -1 = none
  unsigned char* xflag;  // [MC*H]
  int* xlist;            // [1 + MC*H]
  float* h32;            // [MC,H,K,V]
  void* h16;             // [MC,H,K,V] (tensor-core path only)
};

inline size_t saved_bytes(int64_t N, int64_t T, int64_t H, int64_t K, int64_t V, bool tc) {
  const int64_t MC = max_chunks(N, T);
  const size_t st = (size_t)MC * H * K * V;
  return align256(8 * (N + 1)) + align256(16 * (size_t)(MC > 0 ? MC : 1)) + align256((size_t)MC * H + 1) +
         align256(4 * ((size_t)MC * H + 1)) + align256(4 * st) + (tc ? align256(2 * st) : 0);
}

inline Saved carve_saved(void* base, int64_t N, int64_t T, int64_t H, int64_t K, int64_t V, bool tc) {
  const int64_t MC = max_chunks(N, T);
  const size_t st = (size_t)MC * H * K * V;
  char* p = (char*)base;
  Saved s;
  s.chunk_off = (int64_t*)p;
  p += align256(8 * (N + 1));
  s.chunk_tab = (longlong2*)p;
  p += align256(16 * (size_t)(MC > 0 ? MC : 1));
  s.xflag = (unsigned char*)p;
  p += align256((size_t)MC * H + 1);
  s.xlist = (int*)p;
  p += align256(4 * ((size_t)MC * H + 1));
  s.h32 = (float*)p;
  p += align256(4 * st);
  s.h16 = tc ? (void*)p : nullptr;
  return s;
}

// Per-call scratch.  The forward uses the prefix dS | decay | escale; the backward also the
// adjoint states.
struct Workspace {
  float* dS;      // [MC,H,K,V]  per-chunk state increment (fwd) / its adjoint (bwd)
  float* decay;   // [MC,H,K]    exp(g summed over the chunk)
  float* escale;  // [MC,H,K]    fwd: exp(ref); bwd: exp(gL - ref) (16-bit state scaling)
  float* dh32;    // [MC,H,K,V]  adjoint of the state at the end of each chunk (bwd, fp32)
  void* dh16;     // [MC,H,K,V]  dH' = exp(gL - ref) dh in the operand dtype (bwd, tensor cores)
};

inline size_t fwd_workspace_bytes(int64_t N, int64_t T, int64_t H, int64_t K, int64_t V) {
  const int64_t MC = max_chunks(N, T);
  return align256(4 * (size_t)MC * H * K * V) + 2 * align256(4 * (size_t)MC * H * K);
}

inline size_t workspace_bytes(int64_t N, int64_t T, int64_t H, int64_t K, int64_t V, bool tc) {
  const int64_t MC = max_chunks(N, T);
  const size_t st = (size_t)MC * H * K * V;
  return fwd_workspace_bytes(N, T, H, K, V) + align256(4 * st) + (tc ? align256(2 * st) : 0);
}

inline Workspace carve(void* base, int64_t N, int64_t T, int64_t H, int64_t K, int64_t V, bool tc) {
  const int64_t MC = max_chunks(N, T);
  const size_t st = (size_t)MC * H * K * V;
  char* p = (char*)base;
  Workspace w;
  w.dS = (float*)p;
  p += align256(4 * st);
  w.decay = (float*)p;
  p += align256(4 * (size_t)MC * H * K);
  w.escale = (float*)p;
  p += align256(4 * (size_t)MC * H * K);
  w.dh32 = (float*)p;
  p += align256(4 * st);
  w.dh16 = tc ? (void*)p : nullptr;
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
// Also zeroes the exact-item count *xcount (nullable).
int launch_chunk_offsets(const int64_t* cu, int64_t N, int64_t MC, int64_t* chunk_off,
                         longlong2* chunk_tab, int* xcount, cudaStream_t s);
// h_{c+1} = decay_c h_c + dS_c along each sequence's chunks (reverse: the adjoint).  Writes the
// value at every chunk into h32 (all chunks when xflag is null, else only flagged items) and,
// when h16 is non-null, escale[c][k] * value into h16 in 16-bit dtype `dtype16`.
int launch_state_scan(const float* dS, const float* decay, const int64_t* chunk_off, int64_t N,
                      int64_t H, int64_t K, int64_t V, const float* init, float* h32,
                      const unsigned char* xflag, void* h16, int dtype16, const float* escale,
                      float* final_state, bool reverse, cudaStream_t s);

// CUDA-core per-chunk kernels (chunk_gla.cu).  With `xlist` non-null only the listed
// (chunk, head) items are processed (fallback of the tensor-core kernels; none: it exits).
int simt_local(int dtype, int dtype_g, int mode, const void* a_src, const void* b_src, const void* g,
               const int64_t* cu, const longlong2* chunk_tab, int64_t N, int64_t MC, int64_t H,
               int64_t K, int64_t V, float scale, float* dS, float* decay, cudaStream_t s);
int simt_fwd_o(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
               const int64_t* cu, const longlong2* chunk_tab, int64_t N, int64_t MC, int64_t H,
               int64_t K, int64_t V, float scale, const float* states, void* o,
               const int* xlist, cudaStream_t s);
int simt_bwd(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
             const int64_t* cu, const longlong2* chunk_tab, int64_t N, int64_t MC, int64_t H,
             int64_t K, int64_t V, float scale, const float* states, const float* dstates,
             const void* dout, void* dq, void* dk, void* dv, float* dg, const int* xlist,
             cudaStream_t s);

// Tensor-core (tcgen05) implementation for 16-bit inputs with K = V = 64 (chunk_gla_tc.cu).
// 1 when every pointer is 16-byte aligned (TMA base addresses).
int tc_aligned(const void* const* ptrs, int n);
// mode 0: forward increments, decay, escale = exp(ref), xflag and xlist; mode 1: adjoint
// increments, decay, escale = exp(gL - ref) (xflag, xlist null).
int tc_local_state(int dtype, int dtype_g, int mode, const void* a_src, const void* b_src, const void* g,
                   const longlong2* chunk_tab, int64_t T, int64_t MC, int64_t H, float scale, float* dS,
                   float* decay, float* escale, unsigned char* xflag, int* xlist, cudaStream_t s);
int tc_fwd_o(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
             const longlong2* chunk_tab, int64_t T, int64_t MC, int64_t H, float scale, const void* h16,
             const unsigned char* xflag, void* o, cudaStream_t s);
int tc_bwd(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
           const longlong2* chunk_tab, int64_t T, int64_t MC, int64_t H, float scale, const void* h16,
           const void* dh16, const unsigned char* xflag, const void* dout, void* dq, void* dk, void* dv,
           float* dg, cudaStream_t s);

}  // namespace chunk
}  // namespace ssla
