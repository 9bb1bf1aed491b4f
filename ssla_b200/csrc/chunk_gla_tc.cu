// Tensor-core (tcgen05 / TMEM) kernels of the chunked GLA path for 16-bit inputs, K = V = 64.
//
// One CTA of 256 threads (8 warps) owns one (64-token chunk, head).  TMEM is allocated first
// (allocating after outstanding loads was measured to serialise the CTAs of an SM); input
// tiles are then copied with cp.async straight into 16-bit operand tiles in shared memory
// ("8x8 blocked", see tc_util.cuh) and gated in place; one thread issues 64x64x16
// tcgen05.mma instructions into fp32 TMEM accumulators; the epilogue reads TMEM with
// tcgen05.ld.  An M=64 accumulator occupies lanes 0-15 of each of the four TMEM
// subpartitions; warps w and w+4 share subpartition w and split the accumulator's columns.
//
// Gating: with gc the in-chunk cumulative log decay, ref = gc of the chunk's 32nd row and
// E = exp(gc - ref) (the only exponentials evaluated by the output / backward kernels),
//   Q^ = scale q E,  K^ = k / E,  H' = exp(ref) h,  dh' = exp(gL - ref) dh,
// so that (the algebra of ops/gla/chunk.py:23-249 and :253-641)
//   A   = tril(Q^ K^^T)                       o  = Q^ H' + A v
//   dv  = A^T do + K^ dh'                      dq = scale E * (do H'^T + dA K^)
//   dk  = (v dh'^T + dA^T Q^) / E              dA = tril(do v^T)
//   dg  = reverse-cumsum_rows(q dq - k dk) + exp(gL) h.dh + dh'.(K^^T v)
// and for the per-chunk state increments (local_state): mode 0 dS = (k exp(gL - gc))^T v,
// mode 1 dS = (scale q exp(gc))^T do, with per-element exponents.  Every factor of the output
// and backward kernels is bounded by exp(span/2), span = the chunk's decay range; a chunk with
// span > kTcSpan is flagged and recomputed by the exact CUDA-core kernels (chunk_gla.cu).
#include "chunk_gla.cuh"
#include "tc_util.cuh"

namespace ssla {
namespace chunk {
namespace {

using namespace ssla::tc;

constexpr int NT = 256;
constexpr int NWARP = NT / 32;
constexpr int D = 64;         // K = V = 64
constexpr int LDG = D + 1;    // fp32 gate tile stride
constexpr float kTcSpan = 40.f;
constexpr int TILE = BT * D * 2;  // bytes of one 64x64 16-bit tile
constexpr int GRAW = BT * D * 4;  // staging bytes of the raw gate tile (fp32 worst case)

template <typename T> struct Fmt;
template <> struct Fmt<__nv_bfloat16> { static constexpr int v = 1; };
template <> struct Fmt<__half> { static constexpr int v = 0; };

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 x = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&x);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 x = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&x);
}

template <typename T> __device__ __forceinline__ void load8(const T* p, float* x) {
  const uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
  const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = ldf(e + i);
}
template <> __device__ __forceinline__ void load8<float>(const float* p, float* x) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

template <typename T> __device__ __forceinline__ uint4 pack8(const float* x) {
  uint4 u;
  u.x = pack2<T>(x[0], x[1]);
  u.y = pack2<T>(x[2], x[3]);
  u.z = pack2<T>(x[4], x[5]);
  u.w = pack2<T>(x[6], x[7]);
  return u;
}
template <typename T> __device__ __forceinline__ void store8_tile(unsigned char* tile, int r, int c, const float* x) {
  *reinterpret_cast<uint4*>(tile + blk_off(r, c, D)) = pack8<T>(x);
}
template <typename T> __device__ __forceinline__ void store8_global(T* p, const float* x) {
  *reinterpret_cast<uint4*>(p) = pack8<T>(x);
}
// 16 values of row r, columns c..c+15, of an 8x8-blocked 16-bit tile.
template <typename T>
__device__ __forceinline__ void tile_row16(const unsigned char* tile, int r, int c, float* x) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint4 u = *reinterpret_cast<const uint4*>(tile + blk_off(r, c + 8 * h, D));
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[8 * h + i] = ldf(e + i);
  }
}

struct GateSmem {
  float E[BT * LDG];  // exp(gc - ref) (or gc itself for local_state); dg scratch at the end
  float ref[D];       // gc of row 31
  float eref[D];      // exp(ref)
  float egl[D];       // exp(gL - ref), gL = gc of row 63
  float gl[D];        // gL
  float part[4][D];   // per-quarter partial sums (dg reverse cumsum, dgL)
  unsigned int span_bits;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Copy a [64 tokens, 64] 16-bit tile of one head into an 8x8-blocked operand tile (rows >= len
// are zero-filled).
template <typename T>
__device__ __forceinline__ void stage_tile(unsigned char* tile, const T* __restrict__ src, int64_t t0,
                                           int len, int H, int head) {
  for (int e = threadIdx.x; e < BT * (D / 8); e += NT) {
    const int r = e >> 3, c = (e & 7) * 8;
    const T* p = src + ((t0 + (r < len ? r : 0)) * H + head) * (int64_t)D + c;
    cp_async16(tile + blk_off(r, c, D), p, r < len);
  }
}
// The gate tile, row-major in `raw` (element type Tg).
template <typename Tg>
__device__ __forceinline__ void stage_gate(unsigned char* raw, const Tg* __restrict__ g, int64_t t0,
                                           int len, int H, int head) {
  constexpr int PER_ROW = D * (int)sizeof(Tg) / 16;
  for (int e = threadIdx.x; e < BT * PER_ROW; e += NT) {
    const int r = e / PER_ROW, c = (e % PER_ROW) * (16 / (int)sizeof(Tg));
    const Tg* p = g + ((t0 + (r < len ? r : 0)) * H + head) * (int64_t)D + c;
    cp_async16(raw + (r * D + c) * sizeof(Tg), p, r < len);
  }
}

// From the staged raw gate tile: in-chunk cumulative sums gc, ref (gc of row 31), gL (row 63),
// exp(ref), exp(gL - ref), the largest |gc - ref| of the chunk, and E = exp(gc - ref)
// (STORE_GC: gc itself).  Thread (column c = tid % 64, quarter q = tid / 64) scans rows
// 16q .. 16q+15 of its column serially in registers; the quarter totals are combined
// through shared memory (two barriers, no shuffle chains).
template <typename Tg, bool STORE_GC>
__device__ __forceinline__ void gate_prep(GateSmem& G, const unsigned char* raw) {
  static_assert(NT == 256, "gate_prep maps 4 threads to each of the 64 columns");
  const int tid = threadIdx.x, c = tid & 63, qt = tid >> 6;
  const Tg* gr = reinterpret_cast<const Tg*>(raw);
  if (tid == 0) G.span_bits = 0u;
  float x[16];
  float run = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    run += ldf(gr + (16 * qt + i) * D + c);
    x[i] = run;
  }
  G.part[qt][c] = run;
  __syncthreads();
  float off = 0.f;
  for (int j = 0; j < qt; ++j) off += G.part[j][c];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] += off;
  if (qt == 1) G.ref[c] = x[15];  // row 31
  if (qt == 3) G.gl[c] = x[15];   // row 63
  __syncthreads();
  const float ref = G.ref[c];
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    m = fmaxf(m, fabsf(x[i] - ref));
    G.E[(16 * qt + i) * LDG + c] = STORE_GC ? x[i] : __expf(x[i] - ref);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((tid & 31) == 0) atomicMax(&G.span_bits, __float_as_uint(m));
  if (qt == 0) {
    G.eref[c] = __expf(ref);
    G.egl[c] = __expf(G.gl[c] - ref);
  }
  __syncthreads();
}

// In-place gating of an 8x8-blocked 16-bit tile: x[r][c] *= f(r, c); optionally keeps the raw
// tile in `raw_copy`.
template <typename T, class F>
__device__ __forceinline__ void gate_tile(unsigned char* tile, F f, unsigned char* raw_copy = nullptr) {
  for (int e = threadIdx.x; e < BT * (D / 8); e += NT) {
    const int r = e >> 3, c = (e & 7) * 8;
    uint4* p = reinterpret_cast<uint4*>(tile + blk_off(r, c, D));
    const uint4 u = *p;
    if (raw_copy) *reinterpret_cast<uint4*>(raw_copy + blk_off(r, c, D)) = u;
    const T* x = reinterpret_cast<const T*>(&u);
    float y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = ldf(x + i) * f(r, c + i);
    *p = pack8<T>(y);
  }
}

__device__ __forceinline__ void mbar_setup(uint64_t* mbar) {
  if (threadIdx.x == 0) {
    mbar_init(mbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
}

// All threads: publish smem operand writes to the tensor core and order them before the MMA.
__device__ __forceinline__ void operands_ready() {
  fence_proxy_async();
  fence_before();
  __syncthreads();
  fence_after();
}

__device__ __forceinline__ void wait_mma(uint64_t* mbar, uint32_t parity) {
  mbar_wait(mbar, parity);
  fence_after();
}

// Four k-steps (K = 64) of D (+)= A * B^T.
__device__ __forceinline__ void mma64(uint32_t d, const void* a, int a_mn, const void* b, int b_mn,
                                      uint32_t idesc, bool accumulate) {
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint64_t da = a_mn ? desc_mnmajor(a, D, s) : desc_kmajor(a, D, s);
    const uint64_t db = b_mn ? desc_mnmajor(b, D, s) : desc_kmajor(b, D, s);
    mma_f16(d, da, db, idesc, (accumulate || s > 0) ? 1u : 0u);
  }
}

// Gate the staged q and k tiles in one pass: Q^ = scale q E, K^ = k / E (optionally keeping
// the raw tiles).
template <typename T>
__device__ __forceinline__ void gate_qk(unsigned char* sQ, unsigned char* sK, const GateSmem& G, float scale,
                                        unsigned char* rawQ, unsigned char* rawK) {
  for (int e = threadIdx.x; e < BT * (D / 8); e += NT) {
    const int r = e >> 3, c = (e & 7) * 8;
    uint4* pq = reinterpret_cast<uint4*>(sQ + blk_off(r, c, D));
    uint4* pk = reinterpret_cast<uint4*>(sK + blk_off(r, c, D));
    const uint4 uq = *pq, uk = *pk;
    if (rawQ) {
      *reinterpret_cast<uint4*>(rawQ + blk_off(r, c, D)) = uq;
      *reinterpret_cast<uint4*>(rawK + blk_off(r, c, D)) = uk;
    }
    const T* xq = reinterpret_cast<const T*>(&uq);
    const T* xk = reinterpret_cast<const T*>(&uk);
    float yq[8], yk[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float e = G.E[r * LDG + c + i];
      yq[i] = ldf(xq + i) * (scale * e);
      yk[i] = __fdividef(ldf(xk + i), e);
    }
    *pq = pack8<T>(yq);
    *pk = pack8<T>(yk);
  }
}

// Epilogue mapping: TMEM subpartition (row block) and column half of this warp.
struct Epi {
  int sp, c0, row;
  __device__ __forceinline__ Epi() {
    const int warp = threadIdx.x >> 5;
    sp = warp & 3;
    c0 = (warp >> 2) * 32;
    row = 16 * sp + (threadIdx.x & 31);
  }
  __device__ __forceinline__ bool owns() const { return (threadIdx.x & 31) < 16; }
};

// --------------------------------------------------------------------------- local state
template <typename T, typename Tg>
__global__ void __launch_bounds__(NT) tc_local_state_kernel(
    int mode, const T* __restrict__ a_src, const T* __restrict__ b_src, const Tg* __restrict__ g,
    const int64_t* __restrict__ cu, const longlong2* __restrict__ chunk_tab, int64_t N, int H,
    float scale, float* __restrict__ dS, float* __restrict__ decay) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sA = smem;
  unsigned char* sB = sA + TILE;
  unsigned char* graw = sB + TILE;
  GateSmem& G = *reinterpret_cast<GateSmem*>(graw + GRAW);
  __shared__ uint64_t mbar;
  __shared__ uint32_t tbase_s;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t cid = blockIdx.x;
  const int head = blockIdx.y;
  int64_t seq, t0;
  int len;
  if (!locate_chunk(cid, chunk_tab, seq, t0, len)) return;
  if (warp == 0) tmem_alloc(&tbase_s, 64);
  mbar_setup(&mbar);
  stage_gate<Tg>(graw, g, t0, len, H, head);
  stage_tile<T>(sA, a_src, t0, len, H, head);
  stage_tile<T>(sB, b_src, t0, len, H, head);
  cp_async_wait_all();
  __syncthreads();
  gate_prep<Tg, true>(G, graw);
  if (mode == 0)
    gate_tile<T>(sA, [&](int r, int c) { return __expf(G.gl[c] - G.E[r * LDG + c]); });
  else
    gate_tile<T>(sA, [&](int r, int c) { return scale * __expf(G.E[r * LDG + c]); });
  operands_ready();
  const uint32_t tb = tbase_s;
  if (tid == 0) {
    mma64(tb, sA, 1, sB, 1, idesc_f16(64, 64, Fmt<T>::v, 1, 1), false);
    commit(&mbar);
  }
  wait_mma(&mbar, 0);
  const Epi ep;
  float* out = dS + (cid * H + head) * (int64_t)D * D;
  for (int cb = ep.c0; cb < ep.c0 + 32; cb += 16) {
    float v[16];
    tmem_ld16(tmem_addr(tb, ep.sp, cb), v);
    if (ep.owns()) {
      float4* o4 = reinterpret_cast<float4*>(out + ep.row * D + cb);
#pragma unroll
      for (int i = 0; i < 4; ++i) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
  }
  if (tid < D) decay[(cid * H + head) * D + tid] = __expf(G.gl[tid]);
  fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, 64);
}

// --------------------------------------------------------------------------- forward output
template <typename T, typename Tg>
__global__ void __launch_bounds__(NT) tc_fwd_o_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const Tg* __restrict__ g, const int64_t* __restrict__ cu, const longlong2* __restrict__ chunk_tab,
    int64_t N, int H, float scale, const float* __restrict__ states, T* __restrict__ o,
    int* __restrict__ flags) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sQ = smem;
  unsigned char* sK = sQ + TILE;
  unsigned char* sV = sK + TILE;
  unsigned char* sH = sV + TILE;
  unsigned char* sA = sH + TILE;
  unsigned char* graw = sA + TILE;
  GateSmem& G = *reinterpret_cast<GateSmem*>(graw + GRAW);
  __shared__ uint64_t mbar;
  __shared__ uint32_t tbase_s;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t cid = blockIdx.x;
  const int head = blockIdx.y;
  int64_t seq, t0;
  int len;
  if (!locate_chunk(cid, chunk_tab, seq, t0, len)) return;
  if (warp == 0) tmem_alloc(&tbase_s, 128);
  mbar_setup(&mbar);
  stage_gate<Tg>(graw, g, t0, len, H, head);
  stage_tile<T>(sQ, q, t0, len, H, head);
  stage_tile<T>(sK, k, t0, len, H, head);
  stage_tile<T>(sV, v, t0, len, H, head);
  // chunk-start state: fetched into registers while the tiles land
  constexpr int SV = D * (D / 8) / NT;  // 8-float vectors per thread
  float hreg[SV][8];
  {
    const float* hs = states + (cid * H + head) * (int64_t)D * D;
#pragma unroll
    for (int j = 0; j < SV; ++j) {
      const int e = tid + j * NT;
      load8(hs + (e >> 3) * D + (e & 7) * 8, hreg[j]);
    }
  }
  cp_async_wait_all();
  __syncthreads();
  gate_prep<Tg, false>(G, graw);
  const bool exact = __uint_as_float(G.span_bits) > kTcSpan;
  if (tid == 0) flags[cid * H + head] = exact ? 1 : 0;
  const uint32_t tb = tbase_s;
  if (exact) {
    if (warp == 0) tmem_dealloc(tb, 128);
    return;
  }
  gate_qk<T>(sQ, sK, G, scale, nullptr, nullptr);
#pragma unroll
  for (int j = 0; j < SV; ++j) {
    const int e = tid + j * NT, r = e >> 3;
#pragma unroll
    for (int i = 0; i < 8; ++i) hreg[j][i] *= G.eref[r];
    store8_tile<T>(sH, r, (e & 7) * 8, hreg[j]);
  }
  operands_ready();
  constexpr uint32_t F = Fmt<T>::v;
  if (tid == 0) {
    mma64(tb, sQ, 0, sK, 0, idesc_f16(64, 64, F, 0, 0), false);        // A = Q^ K^^T
    mma64(tb + 64, sQ, 0, sH, 1, idesc_f16(64, 64, F, 0, 1), false);   // O = Q^ H'
    commit(&mbar);
  }
  wait_mma(&mbar, 0);
  const Epi ep;
  for (int cb = ep.c0; cb < ep.c0 + 32; cb += 16) {
    float x[16];
    tmem_ld16(tmem_addr(tb, ep.sp, cb), x);
    if (ep.owns()) {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (cb + i > ep.row) x[i] = 0.f;
      store8_tile<T>(sA, ep.row, cb, x);
      store8_tile<T>(sA, ep.row, cb + 8, x + 8);
    }
  }
  operands_ready();
  if (tid == 0) {
    mma64(tb + 64, sA, 0, sV, 1, idesc_f16(64, 64, F, 0, 1), true);    // O += A V
    commit(&mbar);
  }
  wait_mma(&mbar, 1);
  for (int cb = ep.c0; cb < ep.c0 + 32; cb += 16) {
    float x[16];
    tmem_ld16(tmem_addr(tb + 64, ep.sp, cb), x);
    if (ep.owns() && ep.row < len) {
      T* dst = o + ((t0 + ep.row) * H + head) * (int64_t)D + cb;
      store8_global<T>(dst, x);
      store8_global<T>(dst + 8, x + 8);
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, 128);
}

// --------------------------------------------------------------------------- backward
template <typename T, typename Tg>
__global__ void __launch_bounds__(NT) tc_bwd_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const Tg* __restrict__ g, const int64_t* __restrict__ cu, const longlong2* __restrict__ chunk_tab,
    int64_t N, int H, float scale, const float* __restrict__ states,
    const float* __restrict__ dstates, const T* __restrict__ dout, T* __restrict__ dq,
    T* __restrict__ dk, T* __restrict__ dv, float* __restrict__ dg, int* __restrict__ flags) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sQ = smem;
  unsigned char* sK = sQ + TILE;
  unsigned char* sV = sK + TILE;
  unsigned char* sDO = sV + TILE;
  unsigned char* sH = sDO + TILE;
  unsigned char* sDH = sH + TILE;
  unsigned char* sA = sDH + TILE;
  unsigned char* sdA = sA + TILE;
  unsigned char* graw = sdA + TILE;
  GateSmem& G = *reinterpret_cast<GateSmem*>(graw + GRAW);
  __shared__ uint64_t mbar;
  __shared__ uint32_t tbase_s;
  __shared__ float s_hdh[D], s_dgl[D];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t cid = blockIdx.x;
  const int head = blockIdx.y;
  int64_t seq, t0;
  int len;
  if (!locate_chunk(cid, chunk_tab, seq, t0, len)) return;
  if (warp == 0) tmem_alloc(&tbase_s, 256);
  mbar_setup(&mbar);
  if (tid < D) s_hdh[tid] = 0.f;
  stage_gate<Tg>(graw, g, t0, len, H, head);
  stage_tile<T>(sQ, q, t0, len, H, head);
  stage_tile<T>(sK, k, t0, len, H, head);
  stage_tile<T>(sV, v, t0, len, H, head);
  stage_tile<T>(sDO, dout, t0, len, H, head);
  // chunk-start state and its adjoint: fetched into registers while the tiles land
  constexpr int SV = D * (D / 8) / NT;  // 8-float vectors per thread
  const int64_t soff = (cid * H + head) * (int64_t)D * D;
  float hreg[SV][8], dhreg[SV][8];
#pragma unroll
  for (int j = 0; j < SV; ++j) {
    const int e = tid + j * NT;
    load8(states + soff + (e >> 3) * D + (e & 7) * 8, hreg[j]);
    load8(dstates + soff + (e >> 3) * D + (e & 7) * 8, dhreg[j]);
  }
  cp_async_wait_all();
  __syncthreads();
  gate_prep<Tg, false>(G, graw);
  const bool exact = __uint_as_float(G.span_bits) > kTcSpan;
  if (tid == 0) flags[cid * H + head] = exact ? 1 : 0;
  const uint32_t tb = tbase_s;
  if (exact) {
    if (warp == 0) tmem_dealloc(tb, 256);
    return;
  }
  // raw q and k stay (blocked layout) in the gate staging area for dg = q dq - k dk
  unsigned char* rawQ = graw;
  unsigned char* rawK = graw + TILE;
  gate_qk<T>(sQ, sK, G, scale, rawQ, rawK);
#pragma unroll
  for (int j = 0; j < SV; ++j) {
    const int e = tid + j * NT, r = e >> 3, c = (e & 7) * 8;
    float hd = 0.f;
    const float er = G.eref[r], egl = G.egl[r];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      hd = fmaf(hreg[j][i], dhreg[j][i], hd);
      hreg[j][i] *= er;
      dhreg[j][i] *= egl;
    }
    atomicAdd(&s_hdh[r], hd);
    store8_tile<T>(sH, r, c, hreg[j]);
    store8_tile<T>(sDH, r, c, dhreg[j]);
  }
  operands_ready();
  constexpr uint32_t F = Fmt<T>::v;
  if (tid == 0) {
    mma64(tb, sQ, 0, sK, 0, idesc_f16(64, 64, F, 0, 0), false);         // A  = Q^ K^^T
    mma64(tb + 64, sDO, 0, sV, 0, idesc_f16(64, 64, F, 0, 0), false);   // dA = do v^T
    mma64(tb + 128, sK, 1, sV, 1, idesc_f16(64, 64, F, 1, 1), false);   // S  = K^^T v
    commit(&mbar);
  }
  wait_mma(&mbar, 0);
  const Epi ep;
  float dgl_part = 0.f;
  for (int cb = ep.c0; cb < ep.c0 + 32; cb += 16) {
    float x[16], y[16], z[16];
    tmem_ld16(tmem_addr(tb, ep.sp, cb), x);
    tmem_ld16(tmem_addr(tb + 64, ep.sp, cb), y);
    tmem_ld16(tmem_addr(tb + 128, ep.sp, cb), z);
    if (ep.owns()) {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (cb + i > ep.row) { x[i] = 0.f; y[i] = 0.f; }
      store8_tile<T>(sA, ep.row, cb, x);
      store8_tile<T>(sA, ep.row, cb + 8, x + 8);
      store8_tile<T>(sdA, ep.row, cb, y);
      store8_tile<T>(sdA, ep.row, cb + 8, y + 8);
      // row `row` of S is key index `row`: dh'[row, :] . S[row, :]
      float dh16[16];
      tile_row16<T>(sDH, ep.row, cb, dh16);
#pragma unroll
      for (int i = 0; i < 16; ++i) dgl_part = fmaf(dh16[i], z[i], dgl_part);
    }
  }
  if (ep.owns()) G.part[warp >> 2][ep.row] = dgl_part;
  operands_ready();
  if (tid == 0) {
    mma64(tb + 192, sA, 1, sDO, 1, idesc_f16(64, 64, F, 1, 1), false);  // dv  = A^T do
    mma64(tb + 192, sK, 0, sDH, 1, idesc_f16(64, 64, F, 0, 1), true);   //     + K^ dh'
    mma64(tb, sDO, 0, sH, 0, idesc_f16(64, 64, F, 0, 0), false);        // dq~ = do H'^T
    mma64(tb, sdA, 0, sK, 1, idesc_f16(64, 64, F, 0, 1), true);         //     + dA K^
    mma64(tb + 64, sV, 0, sDH, 0, idesc_f16(64, 64, F, 0, 0), false);   // dk~ = v dh'^T
    mma64(tb + 64, sdA, 1, sQ, 1, idesc_f16(64, 64, F, 1, 1), true);    //     + dA^T Q^
    commit(&mbar);
  }
  // dgL per key index: exp(gL) h.dh + dh'.(K^^T v)
  if (tid < D) s_dgl[tid] = G.eref[tid] * G.egl[tid] * s_hdh[tid] + G.part[0][tid] + G.part[1][tid];
  wait_mma(&mbar, 1);
  const int64_t roff = ((t0 + ep.row) * H + head) * (int64_t)D;
  const bool live = ep.owns() && ep.row < len;
  for (int cb = ep.c0; cb < ep.c0 + 32; cb += 16) {
    float x[16], y[16], z[16];
    tmem_ld16(tmem_addr(tb + 192, ep.sp, cb), z);
    tmem_ld16(tmem_addr(tb, ep.sp, cb), x);
    tmem_ld16(tmem_addr(tb + 64, ep.sp, cb), y);
    if (ep.owns()) {
      float qr[16], kr[16];
      tile_row16<T>(rawQ, ep.row, cb, qr);
      tile_row16<T>(rawK, ep.row, cb, kr);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float e = G.E[ep.row * LDG + cb + i];
        x[i] *= scale * e;
        y[i] = __fdividef(y[i], e);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) G.E[ep.row * LDG + cb + i] = qr[i] * x[i] - kr[i] * y[i];  // dgc
      if (live) {
        store8_global<T>(dv + roff + cb, z);
        store8_global<T>(dv + roff + cb + 8, z + 8);
        store8_global<T>(dq + roff + cb, x);
        store8_global<T>(dq + roff + cb + 8, x + 8);
        store8_global<T>(dk + roff + cb, y);
        store8_global<T>(dk + roff + cb + 8, y + 8);
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, 256);
  // dg = reverse cumulative sum over rows of dgc (+ dgL at every row): 4 quarters of 16 rows
  {
    const int c = tid & 63, qt = tid >> 6;
    float s = 0.f;
    for (int r = 16 * qt + 15; r >= 16 * qt; --r) { s += G.E[r * LDG + c]; G.E[r * LDG + c] = s; }
    G.part[qt][c] = s;
    __syncthreads();
    float after = s_dgl[c];
    for (int j = qt + 1; j < 4; ++j) after += G.part[j][c];
    for (int r = 16 * qt; r < 16 * qt + 16; ++r) G.E[r * LDG + c] += after;
    __syncthreads();
    for (int e = tid; e < len * D; e += NT) {
      const int r = e >> 6, cc = e & 63;
      dg[((t0 + r) * H + head) * (int64_t)D + cc] = G.E[r * LDG + cc];
    }
  }
}

template <typename K_>
int prepare(K_ kern, size_t smem) {
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
    set_error("chunk_gla tensor-core kernel: cannot reserve %zu bytes of shared memory", smem);
    return SSLA_ERR_CUDA;
  }
  return SSLA_OK;
}

#define SSLA_DISPATCH_TC(dtype, dtype_g, T, Tg, ...)                                    \
  [&]() -> int {                                                                        \
    if (dtype == SSLA_BF16) {                                                           \
      using T = __nv_bfloat16;                                                          \
      if (dtype_g == SSLA_F32) { using Tg = float; return __VA_ARGS__(); }              \
      using Tg = T;                                                                     \
      return __VA_ARGS__();                                                             \
    }                                                                                   \
    using T = __half;                                                                   \
    if (dtype_g == SSLA_F32) { using Tg = float; return __VA_ARGS__(); }                \
    using Tg = T;                                                                       \
    return __VA_ARGS__();                                                               \
  }()

constexpr size_t kGateBytes = sizeof(GateSmem);

}  // namespace

int tc_supported(int dtype, int dtype_g, int64_t K, int64_t V) {
  return (dtype == SSLA_BF16 || dtype == SSLA_F16) && (dtype_g == dtype || dtype_g == SSLA_F32) &&
         K == D && V == D;
}

int tc_local_state(int dtype, int dtype_g, int mode, const void* a_src, const void* b_src,
                   const void* g, const int64_t* cu, const longlong2* chunk_tab, int64_t N,
                   int64_t MC, int64_t H, float scale, float* dS, float* decay, cudaStream_t s) {
  return SSLA_DISPATCH_TC(dtype, dtype_g, T, Tg, [&] {
    auto kern = tc_local_state_kernel<T, Tg>;
    const size_t smem = 2 * TILE + GRAW + kGateBytes;
    int rc = prepare(kern, smem);
    if (rc) return rc;
    kern<<<dim3((unsigned)MC, (unsigned)H), NT, smem, s>>>(mode, (const T*)a_src, (const T*)b_src,
                                                         (const Tg*)g, cu, chunk_tab, N, (int)H,
                                                         scale, dS, decay);
    SSLA_CHECK_LAUNCH("chunk_gla tc_local_state");
    return SSLA_OK;
  });
}

int tc_fwd_o(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
             const int64_t* cu, const longlong2* chunk_tab, int64_t N, int64_t MC, int64_t H,
             float scale, const float* states, void* o, int* flags, cudaStream_t s) {
  return SSLA_DISPATCH_TC(dtype, dtype_g, T, Tg, [&] {
    auto kern = tc_fwd_o_kernel<T, Tg>;
    const size_t smem = 5 * TILE + GRAW + kGateBytes;
    int rc = prepare(kern, smem);
    if (rc) return rc;
    kern<<<dim3((unsigned)MC, (unsigned)H), NT, smem, s>>>((const T*)q, (const T*)k, (const T*)v,
                                                         (const Tg*)g, cu, chunk_tab, N, (int)H,
                                                         scale, states, (T*)o, flags);
    SSLA_CHECK_LAUNCH("chunk_gla tc_fwd_o");
    return SSLA_OK;
  });
}

int tc_bwd(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
           const int64_t* cu, const longlong2* chunk_tab, int64_t N, int64_t MC, int64_t H,
           float scale, const float* states, const float* dstates, const void* dout, void* dq,
           void* dk, void* dv, float* dg, int* flags, cudaStream_t s) {
  return SSLA_DISPATCH_TC(dtype, dtype_g, T, Tg, [&] {
    auto kern = tc_bwd_kernel<T, Tg>;
    const size_t smem = 8 * TILE + GRAW + kGateBytes;
    int rc = prepare(kern, smem);
    if (rc) return rc;
    kern<<<dim3((unsigned)MC, (unsigned)H), NT, smem, s>>>(
        (const T*)q, (const T*)k, (const T*)v, (const Tg*)g, cu, chunk_tab, N, (int)H, scale, states,
        dstates, (const T*)dout, (T*)dq, (T*)dk, (T*)dv, dg, flags);
    SSLA_CHECK_LAUNCH("chunk_gla tc_bwd");
    return SSLA_OK;
  });
}

}  // namespace chunk
}  // namespace ssla
