// Chunked gated linear attention, forward and backward (chunk_gla, ops/gla/chunk.py:906-1116).
//
// Algorithm (per sequence, per head, chunks of 64 tokens, gc = in-chunk cumulative log-decay,
// gL = gc of the chunk's last token, h = state at the chunk start):
//   o_i     = scale (q_i * exp(gc_i)) h + sum_{j<=i} A_ij v_j
//   A_ij    = scale sum_k q_ik k_jk exp(gc_ik - gc_jk)                        (j <= i)
//   h_next  = exp(gL) * h + sum_j (k_j * exp(gL - gc_j))^T v_j
// The reference runs the state recurrence as one serial program per (sequence, head-block)
// (ops/common/chunk_h.py:13-128), i.e. 8-32 programs for its benchmark.  Here it is split in
// two levels so all 148 SMs stay busy:
//   1. local_state: every chunk computes its increment dS = sum_j (k_j exp(gL-gc_j))^T v_j
//      and decay exp(gL) independently;
//   2. state_scan: h_{c+1} = exp(gL_c) * h_c + dS_c is element-wise in (k, v), so one thread
//      per state element walks the chunks of its sequence (N*H*K*V threads);
//   3. output: every chunk computes o from h_c (chunk-parallel).
// The backward mirrors this with the adjoint state (chunk_bwd_dh, ops/common/chunk_h.py:131-239)
// and one fused per-chunk kernel for dq, dk, dv, dg (ops/gla/chunk.py:253-641).
//
// Numerics: exp(gc_i - gc_j) is factorised per 16-row sub-chunk around a reference row
// (the sub-chunk scheme of ops/gla/chunk.py:23-176), so every factor stays bounded; a
// sub-chunk whose decay span could overflow the factorisation falls back to exact
// per-element exponents.  This file is the CUDA-core (fp32 FMA) implementation: it is used
// for fp32 inputs, where results must match an fp32 reference to ~1e-6, and for shapes the
// tensor-core kernels (chunk_gla_tc.cu) do not cover.
#include <type_traits>

#include "chunk_gla.cuh"

namespace ssla {
namespace chunk {
namespace {

constexpr int NTHR = 256;

// --------------------------------------------------------------------------- prep + scans
// Chunk offsets (exclusive scan of ceil(len / 64) over the sequences) and the chunk table.
// With up to kOffSmem sequences the offsets are also kept in shared memory and every chunk id
// finds its sequence by binary search there; with more sequences (typically short ones) each
// thread fills the table entries of its own sequences.
constexpr int kOffSmem = 4096;

__global__ void __launch_bounds__(1024) chunk_offsets_kernel(const int64_t* __restrict__ cu,
                                                             int64_t N, int64_t MC,
                                                             int64_t* __restrict__ off,
                                                             longlong2* __restrict__ tab,
                                                             int* __restrict__ xcount) {
  __shared__ int64_t warp_sums[32];
  __shared__ int64_t carry;
  __shared__ int64_t soff[kOffSmem + 1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool small = N <= kOffSmem;
  griddep_launch_dependents();
  griddep_wait();  // the previous call's kernels may still read the table
  if (tid == 0) {
    carry = 0;
    if (xcount) *xcount = 0;
  }
  __syncthreads();
  for (int64_t base = 0; base < N; base += 1024) {
    const int64_t n = base + tid;
    int64_t x = 0;
    if (n < N) {
      const int64_t len = cu[n + 1] - cu[n];
      x = (len + BT - 1) / BT;
    }
    int64_t incl = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int64_t w = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_sums[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int64_t before = carry + (warp > 0 ? warp_sums[warp - 1] : 0);
    if (n < N) {
      off[n] = before + incl - x;
      if (small) soff[n] = before + incl - x;
    }
    __syncthreads();
    if (tid == 1023) carry = before + incl;
    __syncthreads();
  }
  const int64_t total = carry;
  if (tid == 0) {
    off[N] = total;
    if (small) soff[N] = total;
  }
  __syncthreads();
  // chunk table: {first token, valid rows | sequence << 32}, -1 sequence for unused ids
  if (small) {
    for (int64_t c = tid; c < total; c += 1024) {
      int64_t lo = 0, hi = N - 1;  // last n with soff[n] <= c
      while (lo < hi) {
        const int64_t mid = (lo + hi + 1) >> 1;
        if (soff[mid] <= c) lo = mid; else hi = mid - 1;
      }
      const int64_t t = cu[lo] + (c - soff[lo]) * BT;
      const int64_t e = cu[lo + 1];
      const int64_t len = (e - t) < BT ? (e - t) : BT;
      tab[c] = make_longlong2(t, len | (lo << 32));
    }
  } else {
    for (int64_t n = tid; n < N; n += 1024) {
      const int64_t s0 = cu[n], e = cu[n + 1];
      int64_t c = off[n];
      for (int64_t t = s0; t < e; t += BT, ++c) tab[c] = make_longlong2(t, ((e - t) < BT ? (e - t) : BT) | (n << 32));
    }
  }
  for (int64_t c = total + tid; c < MC; c += 1024) tab[c] = make_longlong2(0, (int64_t)-1 << 32);
}

// h_{c+1} = decay_c * h_c + dS_c along the chunks of each sequence, element-wise in (k, v).
// One thread per (state element, segment): the chunk axis is cut into `nseg` segments (chosen
// on the host so the grid is about one resident wave); each segment first composes its affine
// map (prod decay, local sum), segment start values are chained in shared memory, then every
// segment re-walks its chunks from its start value writing the per-chunk states.  Loads are
// issued SCAN_U chunks at a time (they do not depend on the running state).  Per chunk the
// value is written to h32 (fp32; every chunk when xflag is null, else only flagged items) and,
// for the tensor-core kernels, escale[chunk][k] * value to h16 in the 16-bit operand dtype T16
// (T16 = float: no 16-bit output).
constexpr int SCAN_EL = 32, SCAN_MAXSEG = 8;

// VEC consecutive state elements (one key row, consecutive value columns) per thread.
template <int VEC> struct SVec;
template <> struct SVec<1> {
  using type = float;
  static __device__ __forceinline__ float ld(const float* p) { return *p; }
  static __device__ __forceinline__ void st(float* p, float x) { *p = x; }
  static __device__ __forceinline__ float fma(float d, float x, float a) { return fmaf(d, x, a); }
  static __device__ __forceinline__ float zero() { return 0.f; }
  template <typename T16> static __device__ __forceinline__ void st16(T16* p, float s, float x) { stf(p, s * x); }
};
template <> struct SVec<4> {
  using type = float4;
  static __device__ __forceinline__ float4 ld(const float* p) { return *reinterpret_cast<const float4*>(p); }
  static __device__ __forceinline__ void st(float* p, float4 x) { *reinterpret_cast<float4*>(p) = x; }
  static __device__ __forceinline__ float4 fma(float d, float4 x, float4 a) {
    return make_float4(fmaf(d, x.x, a.x), fmaf(d, x.y, a.y), fmaf(d, x.z, a.z), fmaf(d, x.w, a.w));
  }
  static __device__ __forceinline__ float4 zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
  template <typename T16> static __device__ __forceinline__ void st16(T16* p, float s, float4 x) {
    T16 y[4];
    stf(y + 0, s * x.x);
    stf(y + 1, s * x.y);
    stf(y + 2, s * x.z);
    stf(y + 3, s * x.w);
    *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(y);
  }
};

template <> struct SVec<8> {
  struct type {
    float4 a, b;
  };
  static __device__ __forceinline__ type ld(const float* p) {
    return {reinterpret_cast<const float4*>(p)[0], reinterpret_cast<const float4*>(p)[1]};
  }
  static __device__ __forceinline__ void st(float* p, type x) {
    reinterpret_cast<float4*>(p)[0] = x.a;
    reinterpret_cast<float4*>(p)[1] = x.b;
  }
  static __device__ __forceinline__ type fma(float d, type x, type y) {
    return {SVec<4>::fma(d, x.a, y.a), SVec<4>::fma(d, x.b, y.b)};
  }
  static __device__ __forceinline__ type zero() { return {SVec<4>::zero(), SVec<4>::zero()}; }
  template <typename T16> static __device__ __forceinline__ void st16(T16* p, float s, type x) {
    SVec<4>::template st16<T16>(p, s, x.a);
    SVec<4>::template st16<T16>(p + 4, s, x.b);
  }
};

template <int VEC, typename T16>
__global__ void __launch_bounds__(SCAN_EL * SCAN_MAXSEG, VEC == 8 ? 2 : 4) state_scan_kernel(
    const float* __restrict__ dS, const float* __restrict__ decay,
    const int64_t* __restrict__ chunk_off, int64_t N, int H, int K, int V,
    const float* __restrict__ init, float* __restrict__ h32, const unsigned char* __restrict__ xflag,
    T16* __restrict__ h16, const float* __restrict__ escale, float* __restrict__ fin,
    bool reverse, int nseg) {
  using S = SVec<VEC>;
  using vec = typename S::type;
  constexpr bool kOut16 = !std::is_same<T16, float>::value;
  // chunks whose loads are in flight together; a segment of at most SCAN_U chunks keeps them in
  // registers for the second pass (one round trip to memory in all)
  constexpr int SCAN_U = VEC == 8 ? 8 : 4;
  constexpr int LOOP_U = 4;  // batch of the general (longer segment) loops
  __shared__ float sA[SCAN_MAXSEG][SCAN_EL];
  __shared__ vec sB[SCAN_MAXSEG][SCAN_EL], sX[SCAN_MAXSEG][SCAN_EL];
  const int el = threadIdx.x % SCAN_EL, sg = threadIdx.x / SCAN_EL;
  griddep_launch_dependents();
  griddep_wait();
  const int64_t KV = (int64_t)K * V, HKV = (int64_t)H * KV, HK = (int64_t)H * K;
  const int64_t idx = ((int64_t)blockIdx.x * SCAN_EL + el) * VEC;  // first element of this thread
  const bool valid = idx < N * HKV;
  int64_t len = 0;
  // this thread's elements in its segment's first chunk; steps between chunks
  int64_t ce = 0, cd = 0, cf = 0;  // element offset, decay / escale offset, flag offset
  int64_t sa = 0, sd = 0, sf = 0;
  if (valid) {
    const int64_t seq = idx / HKV;
    const int64_t rem = idx - seq * HKV;
    const int64_t head = rem / KV;
    const int64_t kv = rem - head * KV;
    const int64_t c0 = chunk_off[seq];
    const int64_t n = chunk_off[seq + 1] - c0;
    const int64_t Ls = (n + nseg - 1) / nseg;
    const int64_t i0 = sg * Ls, i1 = (i0 + Ls < n) ? i0 + Ls : n;
    len = i1 > i0 ? i1 - i0 : 0;
    const int64_t dir = reverse ? -1 : 1;
    const int64_t cfirst = (reverse ? c0 + n - 1 : c0) + dir * i0;
    if (len > 0) {
      ce = cfirst * HKV + head * KV + kv;
      cd = cfirst * HK + head * K + kv / V;
      cf = cfirst * H + head;
    }
    sa = dir * HKV;
    sd = dir * HK;
    sf = dir * H;
  }
  // 1. compose this segment's affine map x -> A x + B.  Loads are issued SCAN_U chunks at a time
  // (predicated, so a short segment still costs one round trip): they do not depend on B.
  float A = 1.f;
  vec B = S::zero();
  float d0[SCAN_U], e0[SCAN_U];  // the first batch, kept for pass 3 when it is the whole segment
  vec a0[SCAN_U];
#pragma unroll
  for (int u = 0; u < SCAN_U; ++u) {
    const bool in = u < len;
    d0[u] = in ? decay[cd + u * sd] : 1.f;
    e0[u] = (kOut16 && in) ? escale[cd + u * sd] : 0.f;
    a0[u] = in ? S::ld(dS + ce + u * sa) : S::zero();
  }
#pragma unroll
  for (int u = 0; u < SCAN_U; ++u) { B = S::fma(d0[u], B, a0[u]); A *= d0[u]; }
  for (int64_t i = SCAN_U; i < len; i += LOOP_U) {
    float d[LOOP_U];
    vec a[LOOP_U];
#pragma unroll
    for (int u = 0; u < LOOP_U; ++u) {
      const bool in = i + u < len;
      d[u] = in ? decay[cd + (i + u) * sd] : 1.f;
      a[u] = in ? S::ld(dS + ce + (i + u) * sa) : S::zero();
    }
#pragma unroll
    for (int u = 0; u < LOOP_U; ++u) { B = S::fma(d[u], B, a[u]); A *= d[u]; }
  }
  // 2. chain the segment start values
  vec x;
  if (nseg > 1) {
    sA[sg][el] = A;
    sB[sg][el] = B;
    __syncthreads();
    if (sg == 0) {
      vec y = (valid && init) ? S::ld(init + idx) : S::zero();
      for (int s2 = 0; s2 < nseg; ++s2) {
        sX[s2][el] = y;
        y = S::fma(sA[s2][el], y, sB[s2][el]);
      }
      if (valid && fin) S::st(fin + idx, y);
    }
    __syncthreads();
    x = sX[sg][el];
  } else {
    x = (valid && init) ? S::ld(init + idx) : S::zero();
    if (valid && fin) S::st(fin + idx, S::fma(A, x, B));
  }
  // 3. re-walk from the start value, writing the state at every chunk
  auto put = [&](int64_t e, int64_t dd, int64_t f, vec val) {
    if (!xflag || xflag[f]) S::st(h32 + e, val);
    if constexpr (kOut16) S::template st16<T16>(h16 + e, escale[dd], val);
  };
  if (len <= SCAN_U) {
#pragma unroll
    for (int u = 0; u < SCAN_U; ++u) {
      if (u < len) {
        if (!xflag || xflag[cf + u * sf]) S::st(h32 + ce + u * sa, x);
        if constexpr (kOut16) S::template st16<T16>(h16 + ce + u * sa, e0[u], x);
      }
      x = S::fma(d0[u], x, a0[u]);
    }
    return;
  }
  for (int64_t i = 0; i < len; i += LOOP_U) {
    float d[LOOP_U];
    vec a[LOOP_U];
#pragma unroll
    for (int u = 0; u < LOOP_U; ++u) {
      const bool in = i + u < len;
      d[u] = in ? decay[cd + (i + u) * sd] : 1.f;
      a[u] = in ? S::ld(dS + ce + (i + u) * sa) : S::zero();
    }
#pragma unroll
    for (int u = 0; u < LOOP_U; ++u) {
      if (i + u < len) put(ce + (i + u) * sa, cd + (i + u) * sd, cf + (i + u) * sf, x);
      x = S::fma(d[u], x, a[u]);
    }
  }
}

// --------------------------------------------------------------------------- tile helpers
template <int P> struct L { static constexpr int LD = P + 1; };
constexpr int LDA = BT + 1;

// [BT, P] fp32 tile of rows t0.. (row stride H*D), zero-padded beyond `len` rows / D cols.
template <typename T, int P>
__device__ __forceinline__ void load_tile(float* s, const T* __restrict__ src, int64_t t0, int len,
                                          int H, int head, int D) {
  constexpr int LD = L<P>::LD;
  for (int e = threadIdx.x; e < BT * P; e += blockDim.x) {
    const int r = e / P, c = e - r * P;
    float x = 0.f;
    if (r < len && c < D) x = ldf(src + ((t0 + r) * H + head) * (int64_t)D + c);
    s[r * LD + c] = x;
  }
}

// [P, P] fp32 state tile from [.., K, V] global (zero pad).
template <int P>
__device__ __forceinline__ void load_state(float* s, const float* __restrict__ src, int K, int V) {
  constexpr int LD = L<P>::LD;
  for (int e = threadIdx.x; e < P * P; e += blockDim.x) {
    const int r = e / P, c = e - r * P;
    s[r * LD + c] = (r < K && c < V) ? src[(int64_t)r * V + c] : 0.f;
  }
}

// In-place inclusive cumulative sum over the BT rows of each column (one warp per column).
template <int P>
__device__ __forceinline__ void col_cumsum(float* s) {
  constexpr int LD = L<P>::LD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int c = warp; c < P; c += nw) {
    const float a = s[(2 * lane) * LD + c], b = s[(2 * lane + 1) * LD + c];
    float x = a + b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    float excl = __shfl_up_sync(0xffffffffu, x, 1);
    if (lane == 0) excl = 0.f;
    s[(2 * lane) * LD + c] = excl + a;
    s[(2 * lane + 1) * LD + c] = excl + a + b;
  }
}

// C[m][n] = sum_l a(l,m) * b(l,n), M x N outputs in 4x4 register tiles over the block.
template <int M, int N, class FA, class FB, class FE>
__device__ __forceinline__ void mm4(int Lr, FA a, FB b, FE epi) {
  constexpr int TN = N / 4, TILES = (M / 4) * TN;
  for (int tile = threadIdx.x; tile < TILES; tile += blockDim.x) {
    const int m0 = (tile / TN) * 4, n0 = (tile - (tile / TN) * TN) * 4;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    for (int l = 0; l < Lr; ++l) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) { av[i] = a(l, m0 + i); bv[i] = b(l, n0 + i); }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) epi(m0 + i, n0 + j, acc[i][j]);
  }
}

// Per sub-chunk r: reference row value ref[r][c] = gc[16r+7][c], and whether the factorised
// exponent form is safe for (a) rows of r against columns <= end(r) (A, dq) and (b) columns
// of r against rows >= start(r) (dk).
template <int P>
__device__ __forceinline__ void sub_chunk_refs(const float* sg, float* ref, int* exact_q,
                                               int* exact_k) {
  constexpr int LD = L<P>::LD;
  __shared__ float lo[NC][P], hi[NC][P];
  if (threadIdx.x < NC) { exact_q[threadIdx.x] = 0; exact_k[threadIdx.x] = 0; }
  for (int e = threadIdx.x; e < NC * P; e += blockDim.x) {
    const int r = e / P, c = e - r * P;
    float mn = sg[(r * BC) * LD + c], mx = mn;
    for (int i = 1; i < BC; ++i) {
      const float x = sg[(r * BC + i) * LD + c];
      mn = fminf(mn, x);
      mx = fmaxf(mx, x);
    }
    lo[r][c] = mn;
    hi[r][c] = mx;
    ref[r * P + c] = sg[(r * BC + BC / 2 - 1) * LD + c];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < NC * P; e += blockDim.x) {
    const int r = e / P, c = e - r * P;
    const float rf = ref[r * P + c];
    float mn = lo[r][c], mxl = hi[r][c];
    for (int s = 0; s < r; ++s) mn = fminf(mn, lo[s][c]);
    for (int s = r + 1; s < NC; ++s) mxl = fmaxf(mxl, hi[s][c]);
    if (hi[r][c] - rf > kSpanLimit || rf - mn > kSpanLimit) atomicOr(&exact_q[r], 1);
    if (mxl - rf > kSpanLimit || rf - lo[r][c] > kSpanLimit) atomicOr(&exact_k[r], 1);
  }
  __syncthreads();
}

// --------------------------------------------------------------------------- local state
// mode 0: dS = sum_t (k_t exp(gL - gc_t))^T v_t       (forward state increment)
// mode 1: dS = sum_t (scale q_t exp(gc_t))^T do_t      (backward adjoint increment)
template <typename T, typename Tg, int P>
__global__ void __launch_bounds__(NTHR) local_state_kernel(
    int mode, const T* __restrict__ a_src, const T* __restrict__ b_src, const Tg* __restrict__ g,
    const int64_t* __restrict__ cu, const longlong2* __restrict__ chunk_tab, int64_t N, int H,
    int K, int V, float scale, float* __restrict__ dS, float* __restrict__ decay) {
  constexpr int LD = L<P>::LD;
  extern __shared__ float sm[];
  float* sg = sm;
  float* sa = sg + BT * LD;
  float* sb = sa + BT * LD;
  __shared__ float sL[P];
  const int64_t cid = blockIdx.x;
  const int head = blockIdx.y;
  int64_t seq, t0;
  int len;
  if (!locate_chunk(cid, chunk_tab, seq, t0, len)) return;
  load_tile<Tg, P>(sg, g, t0, len, H, head, K);
  load_tile<T, P>(sa, a_src, t0, len, H, head, K);
  load_tile<T, P>(sb, b_src, t0, len, H, head, V);
  __syncthreads();
  col_cumsum<P>(sg);
  __syncthreads();
  if (threadIdx.x < P) sL[threadIdx.x] = sg[(BT - 1) * LD + threadIdx.x];
  __syncthreads();
  for (int e = threadIdx.x; e < BT * P; e += blockDim.x) {
    const int r = e / P, c = e - r * P;
    const float gc = sg[r * LD + c];
    sa[r * LD + c] *= (mode == 0) ? expf(sL[c] - gc) : scale * expf(gc);
  }
  __syncthreads();
  float* out = dS + (cid * H + head) * (int64_t)K * V;
  mm4<P, P>(
      BT, [&](int l, int m) { return sa[l * LD + m]; }, [&](int l, int n) { return sb[l * LD + n]; },
      [&](int m, int n, float x) {
        if (m < K && n < V) out[(int64_t)m * V + n] = x;
      });
  if (threadIdx.x < K) decay[(cid * H + head) * K + threadIdx.x] = expf(sL[threadIdx.x]);
}

// --------------------------------------------------------------------------- forward output
template <typename T, typename Tg, int P>
__device__ __forceinline__ void fwd_o_body(int64_t cid, int head, 
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const Tg* __restrict__ g, const int64_t* __restrict__ cu, const longlong2* __restrict__ chunk_tab,
    int64_t N, int H, int K, int V, float scale, const float* __restrict__ states,
    T* __restrict__ o) {
  constexpr int LD = L<P>::LD;
  extern __shared__ float sm[];
  float* sq = sm;
  float* sk = sq + BT * LD;
  float* sg = sk + BT * LD;
  float* sv = sg + BT * LD;
  float* sh = sv + BT * LD;
  float* sW = sh + P * LD;
  float* sQh = sW + BT * LD;
  float* sO = sQh + BT * LD;
  float* sA = sO + BT * LD;
  __shared__ float ref[NC * P];
  __shared__ int exact_q[NC], exact_k[NC];
  int64_t seq, t0;
  int len;
  if (!locate_chunk(cid, chunk_tab, seq, t0, len)) return;
  load_tile<T, P>(sq, q, t0, len, H, head, K);
  load_tile<T, P>(sk, k, t0, len, H, head, K);
  load_tile<Tg, P>(sg, g, t0, len, H, head, K);
  load_tile<T, P>(sv, v, t0, len, H, head, V);
  load_state<P>(sh, states + (cid * H + head) * (int64_t)K * V, K, V);
  for (int e = threadIdx.x; e < BT * LDA; e += blockDim.x) sA[e] = 0.f;
  __syncthreads();
  col_cumsum<P>(sg);
  __syncthreads();
  sub_chunk_refs<P>(sg, ref, exact_q, exact_k);
  for (int e = threadIdx.x; e < BT * P; e += blockDim.x) {
    const int r = e / P, c = e - r * P;
    const float gc = sg[r * LD + c], xq = sq[r * LD + c] * scale;
    sW[r * LD + c] = xq * expf(gc);
    sQh[r * LD + c] = xq * expf(gc - ref[(r / BC) * P + c]);
  }
  __syncthreads();
  // inter-chunk part: sO = (scale q exp(gc)) h
  mm4<BT, P>(
      P, [&](int l, int m) { return sW[m * LD + l]; }, [&](int l, int n) { return sh[l * LD + n]; },
      [&](int m, int n, float x) { sO[m * LD + n] = x; });
  // intra-chunk scores, one 16-row sub-chunk at a time
  for (int r = 0; r < NC; ++r) {
    __syncthreads();
    const int jend = (r + 1) * BC;  // columns 0..jend-1
    for (int e = threadIdx.x; e < jend * P; e += blockDim.x) {
      const int j = e / P, c = e - j * P;
      sW[j * LD + c] = sk[j * LD + c] * expf(ref[r * P + c] - sg[j * LD + c]);
    }
    __syncthreads();
    const bool ex = exact_q[r] != 0;
    for (int e = threadIdx.x; e < BC * jend; e += blockDim.x) {
      const int ii = e / jend, j = e - ii * jend, i = r * BC + ii;
      if (j > i) continue;
      float acc = 0.f;
      if (!ex) {
        for (int c = 0; c < P; ++c) acc = fmaf(sQh[i * LD + c], sW[j * LD + c], acc);
      } else {
        for (int c = 0; c < P; ++c)
          acc = fmaf(sq[i * LD + c] * scale, sk[j * LD + c] * expf(sg[i * LD + c] - sg[j * LD + c]), acc);
      }
      sA[i * LDA + j] = acc;
    }
  }
  __syncthreads();
  T* out = o + (t0 * H + head) * (int64_t)V;
  const int64_t ostride = (int64_t)H * V;
  mm4<BT, P>(
      BT, [&](int l, int m) { return sA[m * LDA + l]; }, [&](int l, int n) { return sv[l * LD + n]; },
      [&](int m, int n, float x) {
        if (m < len && n < V) stf(out + m * ostride + n, sO[m * LD + n] + x);
      });
}

// Plain launch: grid (chunks, heads).  Gated launch (xlist != null, fallback of the tensor-core
// kernels): a small grid strides over the listed (chunk, head) items only (none: it exits).
template <typename T, typename Tg, int P>
__global__ void __launch_bounds__(NTHR) fwd_o_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const Tg* __restrict__ g, const int64_t* __restrict__ cu, const longlong2* __restrict__ chunk_tab,
    int64_t N, int H, int K, int V, float scale, const float* __restrict__ states,
    T* __restrict__ o, const int* __restrict__ xlist, int64_t MC) {
  griddep_launch_dependents();
  griddep_wait();
  if (!xlist) {
    fwd_o_body<T, Tg, P>(blockIdx.x, blockIdx.y, q, k, v, g, cu, chunk_tab, N, H, K, V, scale, states, o);
    return;
  }
  const int n = xlist[0];
  for (int i = blockIdx.x; i < n; i += gridDim.x) {
    const int w = xlist[1 + i];
    fwd_o_body<T, Tg, P>(w / H, w % H, q, k, v, g, cu, chunk_tab, N, H, K, V, scale, states, o);
    __syncthreads();
  }
}

// --------------------------------------------------------------------------- backward
template <typename T, typename Tg, int P>
__device__ __forceinline__ void bwd_body(int64_t cid, int head, 
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const Tg* __restrict__ g, const int64_t* __restrict__ cu, const longlong2* __restrict__ chunk_tab,
    int64_t N, int H, int K, int V, float scale, const float* __restrict__ states,
    const float* __restrict__ dstates, const T* __restrict__ dout, T* __restrict__ dq,
    T* __restrict__ dk, T* __restrict__ dv, float* __restrict__ dg) {
  constexpr int LD = L<P>::LD;
  extern __shared__ float sm[];
  float* sq = sm;
  float* sk = sq + BT * LD;
  float* sg = sk + BT * LD;
  float* sv = sg + BT * LD;
  float* sdo = sv + BT * LD;
  float* sh = sdo + BT * LD;
  float* sdh = sh + P * LD;
  float* sW = sdh + P * LD;
  float* sDQ = sW + BT * LD;  // holds q-hat while the scores are rebuilt
  float* sDK = sDQ + BT * LD;
  float* sA = sDK + BT * LD;
  float* sdA = sA + BT * LDA;
  __shared__ float ref[NC * P];
  __shared__ float sL[P], sLg[P];
  __shared__ int exact_q[NC], exact_k[NC];
  int64_t seq, t0;
  int len;
  if (!locate_chunk(cid, chunk_tab, seq, t0, len)) return;
  load_tile<T, P>(sq, q, t0, len, H, head, K);
  load_tile<T, P>(sk, k, t0, len, H, head, K);
  load_tile<Tg, P>(sg, g, t0, len, H, head, K);
  load_tile<T, P>(sv, v, t0, len, H, head, V);
  load_tile<T, P>(sdo, dout, t0, len, H, head, V);
  const int64_t soff = (cid * H + head) * (int64_t)K * V;
  load_state<P>(sh, states + soff, K, V);
  load_state<P>(sdh, dstates + soff, K, V);
  for (int e = threadIdx.x; e < BT * LDA; e += blockDim.x) { sA[e] = 0.f; sdA[e] = 0.f; }
  __syncthreads();
  col_cumsum<P>(sg);
  __syncthreads();
  if (threadIdx.x < P) sL[threadIdx.x] = sg[(BT - 1) * LD + threadIdx.x];
  sub_chunk_refs<P>(sg, ref, exact_q, exact_k);  // ends with __syncthreads
  const float* sQh = sDQ;
  for (int e = threadIdx.x; e < BT * P; e += blockDim.x) {
    const int r = e / P, c = e - r * P;
    sDQ[r * LD + c] = sq[r * LD + c] * scale * expf(sg[r * LD + c] - ref[(r / BC) * P + c]);
  }
  // ---- scores A (recomputed) and dA = do v^T (lower triangle)
  for (int r = 0; r < NC; ++r) {
    __syncthreads();
    const int jend = (r + 1) * BC;
    for (int e = threadIdx.x; e < jend * P; e += blockDim.x) {
      const int j = e / P, c = e - j * P;
      sW[j * LD + c] = sk[j * LD + c] * expf(ref[r * P + c] - sg[j * LD + c]);
    }
    __syncthreads();
    const bool ex = exact_q[r] != 0;
    for (int e = threadIdx.x; e < BC * jend; e += blockDim.x) {
      const int ii = e / jend, j = e - ii * jend, i = r * BC + ii;
      if (j > i) continue;
      float acc = 0.f, dacc = 0.f;
      if (!ex) {
        for (int c = 0; c < P; ++c) acc = fmaf(sQh[i * LD + c], sW[j * LD + c], acc);
      } else {
        for (int c = 0; c < P; ++c)
          acc = fmaf(sq[i * LD + c] * scale, sk[j * LD + c] * expf(sg[i * LD + c] - sg[j * LD + c]), acc);
      }
      for (int c = 0; c < P; ++c) dacc = fmaf(sdo[i * LD + c], sv[j * LD + c], dacc);
      sA[i * LDA + j] = acc;
      sdA[i * LDA + j] = dacc;
    }
  }
  __syncthreads();
  // ---- dv = A^T do + (k exp(gL - gc)) dh_next
  for (int e = threadIdx.x; e < BT * P; e += blockDim.x) {
    const int r = e / P, c = e - r * P;
    sW[r * LD + c] = sk[r * LD + c] * expf(sL[c] - sg[r * LD + c]);
  }
  __syncthreads();
  {
    T* out = dv + (t0 * H + head) * (int64_t)V;
    const int64_t st = (int64_t)H * V;
    mm4<BT, P>(
        BT + P,
        [&](int l, int m) { return l < BT ? sA[l * LDA + m] : sW[m * LD + (l - BT)]; },
        [&](int l, int n) { return l < BT ? sdo[l * LD + n] : sdh[(l - BT) * LD + n]; },
        [&](int m, int n, float x) {
          if (m < len && n < V) stf(out + m * st + n, x);
        });
  }
  __syncthreads();
  // ---- dq inter: scale exp(gc) * (do h^T);  dk inter: exp(gL - gc) * (v dh^T)
  mm4<BT, P>(
      P, [&](int l, int m) { return sdo[m * LD + l]; }, [&](int l, int n) { return sh[n * LD + l]; },
      [&](int m, int n, float x) { sDQ[m * LD + n] = x * scale * expf(sg[m * LD + n]); });
  mm4<BT, P>(
      P, [&](int l, int m) { return sv[m * LD + l]; }, [&](int l, int n) { return sdh[n * LD + l]; },
      [&](int m, int n, float x) { sDK[m * LD + n] = x * expf(sL[n] - sg[m * LD + n]); });
  __syncthreads();
  // gate gradient of the chunk's total decay: exp(gL) sum_v h dh + sum_j k_j dk_inter_j
  if (threadIdx.x < P) {
    const int c = threadIdx.x;
    float a = 0.f, b = 0.f;
    for (int vv = 0; vv < P; ++vv) a = fmaf(sh[c * LD + vv], sdh[c * LD + vv], a);
    for (int j = 0; j < BT; ++j) b = fmaf(sk[j * LD + c], sDK[j * LD + c], b);
    sLg[c] = expf(sL[c]) * a + b;
  }
  // ---- dq intra (rows of sub-chunk r against columns <= end(r))
  for (int r = 0; r < NC; ++r) {
    __syncthreads();
    const int jend = (r + 1) * BC;
    for (int e = threadIdx.x; e < jend * P; e += blockDim.x) {
      const int j = e / P, c = e - j * P;
      sW[j * LD + c] = sk[j * LD + c] * expf(ref[r * P + c] - sg[j * LD + c]);
    }
    __syncthreads();
    if (!exact_q[r]) {
      mm4<BC, P>(
          jend, [&](int l, int m) { return sdA[(r * BC + m) * LDA + l]; },
          [&](int l, int n) { return sW[l * LD + n]; },
          [&](int m, int n, float x) {
            const int i = r * BC + m;
            sDQ[i * LD + n] += scale * x * expf(sg[i * LD + n] - ref[r * P + n]);
          });
    } else {
      for (int e = threadIdx.x; e < BC * P; e += blockDim.x) {
        const int ii = e / P, c = e - ii * P, i = r * BC + ii;
        float acc = 0.f;
        for (int j = 0; j <= i; ++j)
          acc = fmaf(sdA[i * LDA + j], sk[j * LD + c] * expf(sg[i * LD + c] - sg[j * LD + c]), acc);
        sDQ[i * LD + c] += scale * acc;
      }
    }
  }
  // ---- dk intra (columns of sub-chunk s against rows >= start(s))
  for (int s = 0; s < NC; ++s) {
    __syncthreads();
    const int i0 = s * BC;
    for (int e = threadIdx.x; e < (BT - i0) * P; e += blockDim.x) {
      const int i = i0 + e / P, c = e - (e / P) * P;
      sW[i * LD + c] = sq[i * LD + c] * scale * expf(sg[i * LD + c] - ref[s * P + c]);
    }
    __syncthreads();
    if (!exact_k[s]) {
      mm4<BC, P>(
          BT - i0, [&](int l, int m) { return sdA[(i0 + l) * LDA + (i0 + m)]; },
          [&](int l, int n) { return sW[(i0 + l) * LD + n]; },
          [&](int m, int n, float x) {
            const int j = i0 + m;
            sDK[j * LD + n] += x * expf(ref[s * P + n] - sg[j * LD + n]);
          });
    } else {
      for (int e = threadIdx.x; e < BC * P; e += blockDim.x) {
        const int jj = e / P, c = e - jj * P, j = i0 + jj;
        float acc = 0.f;
        for (int i = j; i < BT; ++i)
          acc = fmaf(sdA[i * LDA + j], sq[i * LD + c] * expf(sg[i * LD + c] - sg[j * LD + c]), acc);
        sDK[j * LD + c] += scale * acc;
      }
    }
  }
  __syncthreads();
  // ---- write dq, dk; dg = reverse in-chunk cumsum of (q dq - k dk) (+ decay term at the end)
  {
    const int64_t st = (int64_t)H * K;
    T* oq = dq + (t0 * H + head) * (int64_t)K;
    T* ok = dk + (t0 * H + head) * (int64_t)K;
    for (int e = threadIdx.x; e < len * P; e += blockDim.x) {
      const int r = e / P, c = e - r * P;
      if (c < K) {
        stf(oq + r * st + c, sDQ[r * LD + c]);
        stf(ok + r * st + c, sDK[r * LD + c]);
      }
    }
    float* og = dg + (t0 * H + head) * (int64_t)K;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int c = warp; c < K; c += nw) {
      // rows 2*lane, 2*lane+1; reverse inclusive scan over rows
      float x0 = sq[(2 * lane) * LD + c] * sDQ[(2 * lane) * LD + c] -
                 sk[(2 * lane) * LD + c] * sDK[(2 * lane) * LD + c];
      float x1 = sq[(2 * lane + 1) * LD + c] * sDQ[(2 * lane + 1) * LD + c] -
                 sk[(2 * lane + 1) * LD + c] * sDK[(2 * lane + 1) * LD + c];
      if (lane == 31) x1 += sLg[c];
      float x = x0 + x1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_down_sync(0xffffffffu, x, o);
        if (lane + o < 32) x += y;
      }
      float after = __shfl_down_sync(0xffffffffu, x, 1);  // sum over rows > 2*lane+1
      if (lane == 31) after = 0.f;
      const float r1 = after + x1, r0 = r1 + x0;
      if (2 * lane < len) og[(2 * lane) * st + c] = r0;
      if (2 * lane + 1 < len) og[(2 * lane + 1) * st + c] = r1;
    }
  }
}

// Plain launch: grid (chunks, heads).  Gated launch (xlist != null, fallback of the tensor-core
// kernels): a small grid strides over the listed (chunk, head) items only (none: it exits).
template <typename T, typename Tg, int P>
__global__ void __launch_bounds__(NTHR) bwd_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const Tg* __restrict__ g, const int64_t* __restrict__ cu, const longlong2* __restrict__ chunk_tab,
    int64_t N, int H, int K, int V, float scale, const float* __restrict__ states,
    const float* __restrict__ dstates, const T* __restrict__ dout, T* __restrict__ dq,
    T* __restrict__ dk, T* __restrict__ dv, float* __restrict__ dg, const int* __restrict__ xlist,
    int64_t MC) {
  griddep_launch_dependents();
  griddep_wait();
  if (!xlist) {
    bwd_body<T, Tg, P>(blockIdx.x, blockIdx.y, q, k, v, g, cu, chunk_tab, N, H, K, V, scale, states, dstates, dout, dq, dk, dv, dg);
    return;
  }
  const int n = xlist[0];
  for (int i = blockIdx.x; i < n; i += gridDim.x) {
    const int w = xlist[1 + i];
    bwd_body<T, Tg, P>(w / H, w % H, q, k, v, g, cu, chunk_tab, N, H, K, V, scale, states, dstates, dout, dq, dk, dv, dg);
    __syncthreads();
  }
}

// --------------------------------------------------------------------------- launchers
template <int P> constexpr size_t smem_local() { return 3 * BT * L<P>::LD * 4; }
template <int P> constexpr size_t smem_fwd_o() {
  return (7 * BT * L<P>::LD + P * L<P>::LD + BT * LDA) * 4;
}
template <int P> constexpr size_t smem_bwd() {
  return (8 * BT * L<P>::LD + 2 * P * L<P>::LD + 2 * BT * LDA) * 4;
}

template <typename T, typename Tg, int P>
int run_local(int mode, const void* a_src, const void* b_src, const void* g, const int64_t* cu,
              const longlong2* off, int64_t N, int64_t MC, int H, int K, int V, float scale,
              float* dS, float* decay, cudaStream_t s) {
  auto kern = local_state_kernel<T, Tg, P>;
  const size_t smem = smem_local<P>();
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<dim3((unsigned)MC, H), NTHR, smem, s>>>(mode, (const T*)a_src, (const T*)b_src,
                                                 (const Tg*)g, cu, off, N, H, K, V, scale, dS, decay);
  SSLA_CHECK_LAUNCH("chunk_gla local_state");
  return SSLA_OK;
}

template <typename T, typename Tg, int P>
int run_fwd_o(const void* q, const void* k, const void* v, const void* g, const int64_t* cu,
              const longlong2* off, int64_t N, int64_t MC, int H, int K, int V, float scale,
              const float* states, void* o, const int* xlist, cudaStream_t s) {
  auto kern = fwd_o_kernel<T, Tg, P>;
  const size_t smem = smem_fwd_o<P>();
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const dim3 grid = xlist ? dim3((unsigned)(MC * H < kNumSMs ? MC * H : kNumSMs), 1)
                          : dim3((unsigned)MC, H);
  launch_pdl(kern, grid, dim3(NTHR), smem, s, (const T*)q, (const T*)k, (const T*)v, (const Tg*)g, cu, off, N, H, K,
             V, scale, states, (T*)o, xlist, MC);
  SSLA_CHECK_LAUNCH("chunk_gla fwd_o");
  return SSLA_OK;
}

template <typename T, typename Tg, int P>
int run_bwd(const void* q, const void* k, const void* v, const void* g, const int64_t* cu,
            const longlong2* off, int64_t N, int64_t MC, int H, int K, int V, float scale,
            const float* states, const float* dstates, const void* dout, void* dq, void* dk,
            void* dv, float* dg, const int* xlist, cudaStream_t s) {
  auto kern = bwd_kernel<T, Tg, P>;
  const size_t smem = smem_bwd<P>();
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const dim3 grid = xlist ? dim3((unsigned)(MC * H < kNumSMs ? MC * H : kNumSMs), 1)
                          : dim3((unsigned)MC, H);
  launch_pdl(kern, grid, dim3(NTHR), smem, s, (const T*)q, (const T*)k, (const T*)v, (const Tg*)g, cu, off, N, H, K,
             V, scale, states, dstates, (const T*)dout, (T*)dq, (T*)dk, (T*)dv, dg, xlist, MC);
  SSLA_CHECK_LAUNCH("chunk_gla bwd");
  return SSLA_OK;
}

inline int pad_of(int64_t K, int64_t V) {
  const int64_t m = K > V ? K : V;
  return m <= 16 ? 16 : (m <= 32 ? 32 : (m <= 64 ? 64 : 0));
}

#define SSLA_DISPATCH_PAD(P_, ...)                       \
  [&]() -> int {                                         \
    switch (P_) {                                        \
      case 16: { constexpr int P = 16; return __VA_ARGS__(); } \
      case 32: { constexpr int P = 32; return __VA_ARGS__(); } \
      default: { constexpr int P = 64; return __VA_ARGS__(); } \
    }                                                    \
  }()

// dtype_g is either the input dtype or fp32.
#define SSLA_DISPATCH_QG(dtype, dtype_g, T, Tg, ...)                                   \
  SSLA_DISPATCH_DTYPE(dtype, T, [&] {                                                  \
    if (dtype_g == SSLA_F32) { using Tg = float; return __VA_ARGS__(); }               \
    using Tg = T;                                                                      \
    return __VA_ARGS__();                                                              \
  })

}  // namespace

int simt_fwd_o(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
               const int64_t* cu, const longlong2* off, int64_t N, int64_t MC, int64_t H, int64_t K,
               int64_t V, float scale, const float* states, void* o, const int* xlist,
               cudaStream_t s) {
  return SSLA_DISPATCH_QG(dtype, dtype_g, T_, Tg, [&] {
    return SSLA_DISPATCH_PAD(pad_of(K, V), [&] {
      return run_fwd_o<T_, Tg, P>(q, k, v, g, cu, off, N, MC, (int)H, (int)K, (int)V, scale,
                                  states, o, xlist, s);
    });
  });
}

int simt_bwd(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
             const int64_t* cu, const longlong2* off, int64_t N, int64_t MC, int64_t H, int64_t K,
             int64_t V, float scale, const float* states, const float* dstates, const void* dout,
             void* dq, void* dk, void* dv, float* dg, const int* xlist, cudaStream_t s) {
  return SSLA_DISPATCH_QG(dtype, dtype_g, T_, Tg, [&] {
    return SSLA_DISPATCH_PAD(pad_of(K, V), [&] {
      return run_bwd<T_, Tg, P>(q, k, v, g, cu, off, N, MC, (int)H, (int)K, (int)V, scale, states,
                                dstates, dout, dq, dk, dv, dg, xlist, s);
    });
  });
}

int launch_chunk_offsets(const int64_t* cu, int64_t N, int64_t MC, int64_t* chunk_off,
                         longlong2* chunk_tab, int* xcount, cudaStream_t s) {
  launch_pdl(chunk_offsets_kernel, dim3(1), dim3(1024), 0, s, cu, N, MC, chunk_off, chunk_tab, xcount);
  SSLA_CHECK_LAUNCH("chunk_gla chunk_offsets");
  return SSLA_OK;
}

int simt_local(int dtype, int dtype_g, int mode, const void* a_src, const void* b_src, const void* g,
               const int64_t* cu, const longlong2* chunk_tab, int64_t N, int64_t MC, int64_t H,
               int64_t K, int64_t V, float scale, float* dS, float* decay, cudaStream_t s) {
  return SSLA_DISPATCH_QG(dtype, dtype_g, T_, Tg, [&] {
    return SSLA_DISPATCH_PAD(pad_of(K, V), [&] {
      return run_local<T_, Tg, P>(mode, a_src, b_src, g, cu, chunk_tab, N, MC, (int)H, (int)K, (int)V, scale, dS,
                                  decay, s);
    });
  });
}

int launch_state_scan(const float* dS, const float* decay, const int64_t* chunk_off, int64_t N,
                      int64_t H, int64_t K, int64_t V, const float* init, float* h32,
                      const unsigned char* xflag, void* h16, int dtype16, const float* escale,
                      float* final_state, bool reverse, cudaStream_t s) {
  // 4 consecutive value columns per thread when rows split evenly and the state arrays align
  const bool v4 = V % 4 == 0 &&
                  ((uintptr_t)dS | (uintptr_t)h32 | (uintptr_t)init | (uintptr_t)final_state | (uintptr_t)h16) % 16 == 0;
  const bool v8 = v4 && V % 8 == 0;
  const int vec = v8 ? 8 : (v4 ? 4 : 1);
  const int64_t threads = N * H * K * V / vec;
  if (threads == 0) return SSLA_OK;
  // segments per element: as many as keep the grid within one resident wave (about 1024
  // threads per SM at 64 registers, 512 at the 8-wide variant's 128): a second wave would cost
  // more than the extra segments save
  int64_t nseg = (int64_t)kNumSMs * (vec == 8 ? 512 : 1024) / threads;
  nseg = nseg < 1 ? 1 : (nseg > SCAN_MAXSEG ? SCAN_MAXSEG : nseg);
  const dim3 grid(ceil_div(threads, SCAN_EL)), block(SCAN_EL * (int)nseg);
  auto go = [&](auto kern, auto* out16) {
    launch_pdl(kern, grid, block, 0, s, dS, decay, chunk_off, N, (int)H, (int)K, (int)V, init, h32, xflag, out16,
               escale, final_state, reverse, (int)nseg);
  };
  if (!h16) {
    if (v8) go(state_scan_kernel<8, float>, (float*)nullptr);
    else if (v4) go(state_scan_kernel<4, float>, (float*)nullptr);
    else go(state_scan_kernel<1, float>, (float*)nullptr);
  } else if (dtype16 == SSLA_BF16) {
    if (v8) go(state_scan_kernel<8, __nv_bfloat16>, (__nv_bfloat16*)h16);
    else if (v4) go(state_scan_kernel<4, __nv_bfloat16>, (__nv_bfloat16*)h16);
    else go(state_scan_kernel<1, __nv_bfloat16>, (__nv_bfloat16*)h16);
  } else {
    if (v8) go(state_scan_kernel<8, __half>, (__half*)h16);
    else if (v4) go(state_scan_kernel<4, __half>, (__half*)h16);
    else go(state_scan_kernel<1, __half>, (__half*)h16);
  }
  SSLA_CHECK_LAUNCH("chunk_gla state_scan");
  return SSLA_OK;
}

}  // namespace chunk
}  // namespace ssla

using namespace ssla;
using namespace ssla::chunk;

static int check_common(const char* name, int dtype, int dtype_g, int64_t N, int64_t T, int64_t H,
                        int64_t K, int64_t V) {
  SSLA_CHECK_ARG(dtype_ok(dtype), "%s: bad dtype", name);
  SSLA_CHECK_ARG(dtype_g == dtype || dtype_g == SSLA_F32, "%s: g must have q's dtype or fp32", name);
  SSLA_CHECK_ARG(N >= 0 && T >= 0 && H >= 0, "%s: negative size", name);
  SSLA_CHECK_ARG(K >= 1 && V >= 1 && K <= 64 && V <= 64,
                 "%s: K=%lld V=%lld not supported (1 <= K, V <= 64 in this build)", name,
                 (long long)K, (long long)V);
  return SSLA_OK;
}

extern "C" int64_t ssla_chunk_gla_max_chunks(int64_t n_seqs, int64_t T) {
  return max_chunks(n_seqs, T);
}

extern "C" size_t ssla_chunk_gla_states_bytes(int64_t n_seqs, int64_t T, int64_t H, int64_t K, int64_t V,
                                              int dtype, int dtype_g) {
  return saved_bytes(n_seqs, T, H, K, V, tc_shape(dtype, dtype_g, K, V));
}

extern "C" size_t ssla_chunk_gla_workspace_bytes(int64_t n_seqs, int64_t T, int64_t H, int64_t K,
                                                 int64_t V, int dtype, int dtype_g) {
  return workspace_bytes(n_seqs, T, H, K, V, tc_shape(dtype, dtype_g, K, V));
}

extern "C" int ssla_chunk_gla_fwd(const void* q, const void* k, const void* v, const void* g,
                                  int dtype, int dtype_g, const int64_t* cu_seqlens,
                                  int64_t n_seqs, int64_t T, int64_t H, int64_t K, int64_t V,
                                  float scale, const float* h0, void* o, float* ht,
                                  void* states, size_t states_bytes, void* workspace,
                                  size_t workspace_bytes_, ssla_stream_t stream) {
  int rc = check_common("ssla_chunk_gla_fwd", dtype, dtype_g, n_seqs, T, H, K, V);
  if (rc) return rc;
  if (n_seqs == 0 || H == 0) return SSLA_OK;
  SSLA_CHECK_ARG(cu_seqlens && states && workspace, "ssla_chunk_gla_fwd: null pointer");
  SSLA_CHECK_ARG(T == 0 || (q && k && v && g && o), "ssla_chunk_gla_fwd: null pointer");
  const bool tc_layout = tc_shape(dtype, dtype_g, K, V);
  if (states_bytes < saved_bytes(n_seqs, T, H, K, V, tc_layout)) {
    set_error("ssla_chunk_gla_fwd: states buffer of %zu bytes < %zu needed", states_bytes,
              saved_bytes(n_seqs, T, H, K, V, tc_layout));
    return SSLA_ERR_WORKSPACE;
  }
  if (workspace_bytes_ < fwd_workspace_bytes(n_seqs, T, H, K, V)) {
    set_error("ssla_chunk_gla_fwd: workspace of %zu bytes < %zu needed", workspace_bytes_,
              fwd_workspace_bytes(n_seqs, T, H, K, V));
    return SSLA_ERR_WORKSPACE;
  }
  cudaStream_t s = (cudaStream_t)stream;
  const Saved sv = carve_saved(states, n_seqs, T, H, K, V, tc_layout);
  const Workspace w = carve(workspace, n_seqs, T, H, K, V, tc_layout);
  const int64_t MC = max_chunks(n_seqs, T);
  if ((rc = launch_chunk_offsets(cu_seqlens, n_seqs, MC, sv.chunk_off, sv.chunk_tab, sv.xlist, s))) return rc;
  const void* in[4] = {q, k, v, g};
  const bool tc = tc_layout && tc_aligned(in, 4);
  if (MC > 0) {
    rc = tc ? tc_local_state(dtype, dtype_g, 0, k, v, g, sv.chunk_tab, T, MC, H, scale, w.dS, w.decay, w.escale,
                             sv.xflag, sv.xlist, s)
            : simt_local(dtype, dtype_g, 0, k, v, g, cu_seqlens, sv.chunk_tab, n_seqs, MC, H, K, V, scale, w.dS,
                         w.decay, s);
    if (rc) return rc;
  }
  if ((rc = launch_state_scan(w.dS, w.decay, sv.chunk_off, n_seqs, H, K, V, h0, sv.h32, tc ? sv.xflag : nullptr,
                              tc ? sv.h16 : nullptr, dtype, w.escale, ht, false, s)))
    return rc;
  if (MC == 0) return SSLA_OK;
  if (tc) {
    if ((rc = tc_fwd_o(dtype, dtype_g, q, k, v, g, sv.chunk_tab, T, MC, H, scale, sv.h16, sv.xflag, o, s))) return rc;
    return simt_fwd_o(dtype, dtype_g, q, k, v, g, cu_seqlens, sv.chunk_tab, n_seqs, MC, H, K, V, scale, sv.h32, o,
                      sv.xlist, s);
  }
  return simt_fwd_o(dtype, dtype_g, q, k, v, g, cu_seqlens, sv.chunk_tab, n_seqs, MC, H, K, V, scale, sv.h32, o,
                    nullptr, s);
}

extern "C" int ssla_chunk_gla_bwd(const void* q, const void* k, const void* v, const void* g,
                                  int dtype, int dtype_g, const int64_t* cu_seqlens,
                                  int64_t n_seqs, int64_t T, int64_t H, int64_t K, int64_t V,
                                  float scale, const void* states, size_t states_bytes,
                                  const void* dout, const float* dht, void* dq, void* dk, void* dv,
                                  float* dg, float* dh0, void* workspace, size_t workspace_bytes_,
                                  ssla_stream_t stream) {
  int rc = check_common("ssla_chunk_gla_bwd", dtype, dtype_g, n_seqs, T, H, K, V);
  if (rc) return rc;
  if (n_seqs == 0 || H == 0) return SSLA_OK;
  SSLA_CHECK_ARG(cu_seqlens && states && workspace, "ssla_chunk_gla_bwd: null pointer");
  SSLA_CHECK_ARG(T == 0 || (q && k && v && g && dout && dq && dk && dv && dg),
                 "ssla_chunk_gla_bwd: null pointer");
  const bool tc_layout = tc_shape(dtype, dtype_g, K, V);
  if (states_bytes < saved_bytes(n_seqs, T, H, K, V, tc_layout)) {
    set_error("ssla_chunk_gla_bwd: states buffer of %zu bytes < %zu needed", states_bytes,
              saved_bytes(n_seqs, T, H, K, V, tc_layout));
    return SSLA_ERR_WORKSPACE;
  }
  if (workspace_bytes_ < workspace_bytes(n_seqs, T, H, K, V, tc_layout)) {
    set_error("ssla_chunk_gla_bwd: workspace of %zu bytes < %zu needed", workspace_bytes_,
              workspace_bytes(n_seqs, T, H, K, V, tc_layout));
    return SSLA_ERR_WORKSPACE;
  }
  cudaStream_t s = (cudaStream_t)stream;
  // the forward's chunk table, exact-item flags and states (read only)
  const Saved sv = carve_saved(const_cast<void*>(states), n_seqs, T, H, K, V, tc_layout);
  const Workspace w = carve(workspace, n_seqs, T, H, K, V, tc_layout);
  const int64_t MC = max_chunks(n_seqs, T);
  const void* in[5] = {q, k, v, g, dout};
  const bool tc = tc_layout && tc_aligned(in, 5);
  if (MC > 0) {
    rc = tc ? tc_local_state(dtype, dtype_g, 1, q, dout, g, sv.chunk_tab, T, MC, H, scale, w.dS, w.decay, w.escale,
                             nullptr, nullptr, s)
            : simt_local(dtype, dtype_g, 1, q, dout, g, cu_seqlens, sv.chunk_tab, n_seqs, MC, H, K, V, scale, w.dS,
                         w.decay, s);
    if (rc) return rc;
  }
  if ((rc = launch_state_scan(w.dS, w.decay, sv.chunk_off, n_seqs, H, K, V, dht, w.dh32, tc ? sv.xflag : nullptr,
                              tc ? w.dh16 : nullptr, dtype, w.escale, dh0, true, s)))
    return rc;
  if (MC == 0) return SSLA_OK;
  if (tc) {
    if ((rc = tc_bwd(dtype, dtype_g, q, k, v, g, sv.chunk_tab, T, MC, H, scale, sv.h16, w.dh16, sv.xflag, dout, dq,
                     dk, dv, dg, s)))
      return rc;
    return simt_bwd(dtype, dtype_g, q, k, v, g, cu_seqlens, sv.chunk_tab, n_seqs, MC, H, K, V, scale, sv.h32, w.dh32,
                    dout, dq, dk, dv, dg, sv.xlist, s);
  }
  return simt_bwd(dtype, dtype_g, q, k, v, g, cu_seqlens, sv.chunk_tab, n_seqs, MC, H, K, V, scale, sv.h32, w.dh32,
                  dout, dq, dk, dv, dg, nullptr, s);
}
