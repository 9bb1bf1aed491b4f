// Tensor-core (tcgen05 / TMEM) kernels of the chunked GLA path for 16-bit inputs, K = V = 64.
//
// Work item = (64-token chunk, head).  Every kernel is persistent: a CTA of 512 threads
// (16 warps) walks items blockIdx.x, blockIdx.x + gridDim.x, ... and, while it computes one
// item, the next item's tiles are already in flight into the other of two shared-memory
// stages.  Loads are TMA: warp 0 issues one tensor copy per 64x64 tile (q/k/v/do, the gate)
// and two per fp32 chunk state, completing on the stage's mbarrier, so no thread waits on a
// copy it issued.  Tiles use the 128-byte swizzle: row r occupies bytes r*128 .. r*128+127
// with its 16-byte piece j stored at piece position j ^ (r % 8).  A 16-bit tile then serves
// as a K-major operand (rows = M/N) or an MN-major operand (rows = K) of tcgen05.mma through
// SWIZZLE_128B descriptors, and threads that touch piece j of 8 consecutive rows hit 8
// different bank groups.  One thread issues 64x64x16 tcgen05.mma instructions into fp32 TMEM
// accumulators; the epilogues read TMEM with the 16x256b shape, so all 32 lanes of a warp
// carry data (an M=64 accumulator fills lanes 0-15 of each TMEM subpartition).  Warps w, w+4,
// w+8, w+12 share subpartition w % 4 and take 16 accumulator columns each.
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
// span > kTcSpan is listed in `flags` and recomputed by the exact CUDA-core kernels
// (chunk_gla.cu).
#include <cuda.h>

#include "chunk_gla.cuh"
#include "tc_util.cuh"
#include "tma_map.cuh"

namespace ssla {
namespace chunk {
namespace {

using namespace ssla::tc;

constexpr int NT = 512;
constexpr int D = 64;                      // K = V = 64
constexpr int NWARP = NT / 32;
constexpr int NG = NT / 64;                // gate-scan groups: thread (column, group) owns RG rows
constexpr int RG = BT / NG;
constexpr int EPI_COLS = D / (NWARP / 4);  // accumulator columns per warp in the epilogues
constexpr int LDG = D + 1;                 // fp32 gate tile stride
constexpr float kTcSpan = 40.f;
constexpr int TILE = BT * D * 2;           // bytes of one 64x64 16-bit tile
constexpr int STATE = D * D * 4;           // bytes of one staged fp32 state (two 32-column halves)
static_assert(EPI_COLS == 16, "epilogues read 16 columns per warp (16x256b.x2)");
static_assert(NT == BT * D / 8, "staging assumes one 16-byte chunk of a 16-bit tile per thread");

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
template <typename T> __device__ __forceinline__ void unpack2(uint32_t u, float& a, float& b) {
  const T* e = reinterpret_cast<const T*>(&u);
  a = ldf(e);
  b = ldf(e + 1);
}
template <typename T> __device__ __forceinline__ uint4 pack8(const float* x) {
  uint4 u;
  u.x = pack2<T>(x[0], x[1]);
  u.y = pack2<T>(x[2], x[3]);
  u.z = pack2<T>(x[4], x[5]);
  u.w = pack2<T>(x[6], x[7]);
  return u;
}

// Byte offset of element (r, c) of a 128-byte-swizzled 64x64 16-bit tile.
__device__ __forceinline__ int toff(int r, int c) { return (r << 7) + ((((c >> 3) ^ r) & 7) << 4) + ((c & 7) << 1); }

// SWIZZLE_128B descriptors of such a tile (1024-byte aligned).  Within one 64x64x16 MMA the
// only stride the tensor core needs is between groups of 8 rows along the tile (1024 bytes;
// given as both LBO and SBO).  A k-step of 16 elements advances the start address by 32 bytes
// (K-major: within the swizzled row) or 2048 bytes (MN-major: 16 rows).
__device__ __forceinline__ uint64_t desc_sw128(const void* tile) {
  return smem_desc(smem_u32(tile), 1024u, 1024u) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ uint64_t desc_k(const void* tile) { return desc_sw128(tile); }
__device__ __forceinline__ uint64_t desc_mn(const void* tile) { return desc_sw128(tile); }

// Two adjacent elements (r, c), (r, c+1) of a 16-bit tile (c even).
template <typename T> __device__ __forceinline__ void st2_tile(unsigned char* tile, int r, int c, float a, float b) {
  *reinterpret_cast<uint32_t*>(tile + toff(r, c)) = pack2<T>(a, b);
}
template <typename T> __device__ __forceinline__ void ld2_tile(const unsigned char* tile, int r, int c, float& a, float& b) {
  unpack2<T>(*reinterpret_cast<const uint32_t*>(tile + toff(r, c)), a, b);
}
template <typename T> __device__ __forceinline__ void st2_global(T* p, float a, float b) {
  *reinterpret_cast<uint32_t*>(p) = pack2<T>(a, b);
}


struct GateSmem {
  float E[BT * LDG];  // exp(gc - ref); dgc scratch in the backward
  float ref[D];       // gc of row 31
  float eref[D];      // exp(ref)
  float egl[D];       // exp(gL - ref), gL = gc of row 63
  float gl[D];        // gL
  float part[NG][D];  // per-group partial sums (gate scan, dg reverse cumsum, dgL)
  unsigned int span_bits;
};
constexpr size_t kGateBytes = sizeof(GateSmem);

// Thread t owns the 16-byte piece of row tr = t % 64, columns tc .. tc+7 (tc = 8 * (t / 64))
// of every 16-bit tile in the gating and state-conversion passes (byte toff(tr, tc)).
struct Own {
  int tr, tc;
  int off;
  __device__ __forceinline__ Own() : tr(threadIdx.x & 63), tc((threadIdx.x >> 6) << 3), off(toff(tr, tc)) {}
};

// Issued by one warp: n16 16-bit tiles (tensor maps m16[i], 3-D views (D, H, T) of the token
// arrays, box 64 x 1 x 64) into dst16 + i*TILE, the raw gate (map mg, unswizzled), and nstate
// fp32 states (2-D map ms over [items * 64 rows, 64], two 32-column boxes each) into sdst[i],
// all completing on `bar`.
__device__ __forceinline__ void issue_loads(unsigned char* dst16, const CUtensorMap* const* m16, int n16,
                                            unsigned char* graw, const CUtensorMap* mg, uint32_t gbytes,
                                            unsigned char* const* sdst, const CUtensorMap* const* ms, int nstate,
                                            int srow, int64_t t0, int head, uint64_t* bar) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) mbar_arrive_expect_tx(bar, n16 * TILE + gbytes + nstate * STATE);
  __syncwarp();
  if (lane < n16) tma_load_3d(dst16 + lane * TILE, m16[lane], 0, head, (int)t0, bar);
  if (lane == 8) tma_load_3d(graw, mg, 0, head, (int)t0, bar);
  if (lane >= 16 && lane < 16 + 2 * nstate) {
    const int j = lane - 16;
    tma_load_2d(sdst[j >> 1] + (j & 1) * (STATE / 2), ms[j >> 1], (j & 1) * 32, srow, bar);
  }
}

// Rows >= len of a partial chunk (the TMA box reads past the chunk): zero them in the 16-bit
// tiles and the raw gate.
template <typename Tg>
__device__ __forceinline__ void zero_tail(unsigned char* dst16, int n16, unsigned char* graw, int len) {
  const Own me;
  if (me.tr >= len)
    for (int i = 0; i < n16; ++i) *reinterpret_cast<uint4*>(dst16 + i * TILE + me.off) = make_uint4(0, 0, 0, 0);
  constexpr int PER_ROW = D * (int)sizeof(Tg) / 16;
#pragma unroll
  for (int j = 0; j < BT * PER_ROW / NT; ++j) {
    const int e = threadIdx.x + j * NT;
    if (e / PER_ROW >= len) *reinterpret_cast<uint4*>(graw + 16 * e) = make_uint4(0, 0, 0, 0);
  }
}

// This thread's 8 values of a staged fp32 state: row tr, columns tc .. tc+7 (two 16-byte
// pieces of a 128-byte-swizzled 32-column half).
__device__ __forceinline__ void state_regs(const unsigned char* src, const Own& me, float* v) {
  const unsigned char* h = src + (me.tc >> 5) * (STATE / 2) + (me.tr << 7);
  const int j = (me.tc & 31) >> 2;
  const float4 a = *reinterpret_cast<const float4*>(h + (((j ^ me.tr) & 7) << 4));
  const float4 b = *reinterpret_cast<const float4*>(h + ((((j + 1) ^ me.tr) & 7) << 4));
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// From the staged raw gate tile: in-chunk cumulative sums gc, ref (gc of row 31), gL (row 63),
// exp(ref), exp(gL - ref), the largest |gc - ref| of the chunk, and E = exp(gc - ref).  Thread (column c = tid % 64, group q = tid / 64) scans rows
// RG*q .. RG*q+RG-1 of its column serially in registers; ref and gL come from the group
// totals, so one barrier combines them.
template <typename Tg>
__device__ __forceinline__ void gate_prep(GateSmem& G, const unsigned char* raw) {
  static_assert(NT % 64 == 0 && 31 % RG == RG - 1, "row 31 must end a group");
  const int tid = threadIdx.x, c = tid & 63, qt = tid >> 6;
  const Tg* gr = reinterpret_cast<const Tg*>(raw);
  if (tid == 0) G.span_bits = 0u;
  float x[RG];
  float run = 0.f;
#pragma unroll
  for (int i = 0; i < RG; ++i) {
    run += ldf(gr + (RG * qt + i) * D + c);
    x[i] = run;
  }
  G.part[qt][c] = run;
  __syncthreads();
  // prefix of this group, ref (rows 0..31) and gL (all rows) from the group totals: one barrier
  float off = 0.f, ref = 0.f, gl = 0.f;
#pragma unroll
  for (int j = 0; j < NG; ++j) {
    const float pj = G.part[j][c];
    if (j < qt) off += pj;
    if (j <= 31 / RG) ref += pj;
    gl += pj;
  }
#pragma unroll
  for (int i = 0; i < RG; ++i) x[i] += off;
  if (qt == 0) {
    G.ref[c] = ref;
    G.gl[c] = gl;
  }
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < RG; ++i) {
    m = fmaxf(m, fabsf(x[i] - ref));
    G.E[(RG * qt + i) * LDG + c] = __expf(x[i] - ref);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((tid & 31) == 0) atomicMax(&G.span_bits, __float_as_uint(m));
  if (qt == 0) {
    G.eref[c] = __expf(ref);
    G.egl[c] = __expf(gl - ref);
  }
  __syncthreads();
}


// Local-state gating fused into the in-chunk prefix sums: thread (column c = tid % 64, group
// q = tid / 64) computes gc for rows RG*q .. RG*q+RG-1 of column c and scales those elements of
// the 16-bit tile in place: mode 0 (state increment) by exp(gL - gc), mode 1 (adjoint
// increment) by scale * exp(gc).  Writes G.gl; one barrier.
template <typename T, typename Tg>
__device__ __forceinline__ void gate_apply_local(GateSmem& G, const unsigned char* raw, unsigned char* tile, int mode,
                                                 float scale) {
  const int tid = threadIdx.x, c = tid & 63, qt = tid >> 6;
  const Tg* gr = reinterpret_cast<const Tg*>(raw);
  float x[RG];
  float run = 0.f;
#pragma unroll
  for (int i = 0; i < RG; ++i) {
    run += ldf(gr + (RG * qt + i) * D + c);
    x[i] = run;
  }
  G.part[qt][c] = run;
  __syncthreads();
  float off = 0.f, gl = 0.f;
#pragma unroll
  for (int j = 0; j < NG; ++j) {
    const float pj = G.part[j][c];
    if (j < qt) off += pj;
    gl += pj;
  }
#pragma unroll
  for (int i = 0; i < RG; ++i) {
    const float gc = x[i] + off;
    T* e = reinterpret_cast<T*>(tile + toff(RG * qt + i, c));
    const float f = mode == 0 ? __expf(gl - gc) : scale * __expf(gc);
    stf(e, ldf(e) * f);
  }
  if (qt == 0) G.gl[c] = gl;
}

// All threads: publish smem operand writes to the tensor core and order them before the MMA.
__device__ __forceinline__ void operands_ready() {
  fence_proxy_async();
  fence_before();
  __syncthreads();
  fence_after();
}

// Bounded waits that give up are counted here (read and reset by ssla_chunk_gla_tc_timeouts);
// a nonzero count means results of that launch are not to be trusted.
__device__ unsigned int g_wait_timeouts = 0;

__device__ __forceinline__ void counted_wait(uint64_t* mbar, uint32_t parity) {
  if (!mbar_wait(mbar, parity)) atomicAdd(&g_wait_timeouts, 1u);
}

__device__ __forceinline__ void wait_mma(uint64_t* mbar, uint32_t& phase) {
  counted_wait(mbar, phase);
  phase ^= 1u;
  fence_after();
}

// Four k-steps (K = 64) of D (+)= A * B^T; operands are 64x64 tiles read K-major or MN-major.
__device__ __forceinline__ void mma64(uint32_t d, const void* a, int a_mn, const void* b, int b_mn,
                                      uint32_t idesc, bool accumulate) {
  const uint64_t da = a_mn ? desc_mn(a) : desc_k(a);
  const uint64_t db = b_mn ? desc_mn(b) : desc_k(b);
  const uint64_t sa = a_mn ? 128u : 2u, sb = b_mn ? 128u : 2u;
#pragma unroll
  for (int s = 0; s < 4; ++s) mma_f16(d, da + s * sa, db + s * sb, idesc, (accumulate || s > 0) ? 1u : 0u);
}

// Gate the staged q and k chunks of this thread: Q^ = scale q E, K^ = k / E, written to dQ /
// dK (which may be the source tiles themselves).
template <typename T>
__device__ __forceinline__ void gate_qk(const unsigned char* sQ, const unsigned char* sK, unsigned char* dQ,
                                        unsigned char* dK, const GateSmem& G, const Own& me, float scale) {
  const int off = me.off;
  const uint4 uq = *reinterpret_cast<const uint4*>(sQ + off);
  const uint4 uk = *reinterpret_cast<const uint4*>(sK + off);
  const T* xq = reinterpret_cast<const T*>(&uq);
  const T* xk = reinterpret_cast<const T*>(&uk);
  const float* e = G.E + me.tr * LDG + me.tc;
  float yq[8], yk[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    yq[i] = ldf(xq + i) * (scale * e[i]);
    yk[i] = __fdividef(ldf(xk + i), e[i]);
  }
  *reinterpret_cast<uint4*>(dQ + off) = pack8<T>(yq);
  *reinterpret_cast<uint4*>(dK + off) = pack8<T>(yk);
}

// Epilogue geometry (16x256b.x2): this warp reads TMEM subpartition sp, columns c0 .. c0+15;
// pair p of the 8 values holds row r0 + 8*(p&1), columns c0 + cc + 8*(p>>1) + {0, 1}.
struct Epi {
  int sp, c0, r0, cc;
  __device__ __forceinline__ Epi() {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    sp = warp & 3;
    c0 = (warp >> 2) * EPI_COLS;
    r0 = 16 * sp + (lane >> 2);
    cc = c0 + 2 * (lane & 3);
  }
  __device__ __forceinline__ int row(int p) const { return r0 + 8 * (p & 1); }
  __device__ __forceinline__ int col(int p) const { return cc + 8 * (p >> 1); }
  __device__ __forceinline__ void load(uint32_t tbase, float* v) const {
    tmem_ld16x256b_x2(tmem_addr(tbase, sp, c0), v);
  }
};

// The 128-byte swizzle is anchored at 1024-byte boundaries: kernels align their dynamic
// shared memory explicitly (launchers reserve kAlignSlack extra bytes).
constexpr size_t kAlignSlack = 1024;
__device__ __forceinline__ unsigned char* align1024(unsigned char* p) {
  return p + ((1024u - (smem_u32(p) & 1023u)) & 1023u);
}

// --------------------------------------------------------------------------- persistent loop
struct Item {
  int64_t t0;  // first token of the chunk
  int cid, head, len;
};

// Item cursor: it = cid * H + head, advanced by gridDim.x without divisions.
struct Cursor {
  int cid, head;
  __device__ __forceinline__ void advance(int gq, int gr, int H) {
    head += gr;
    cid += gq;
    if (head >= H) {
      head -= H;
      ++cid;
    }
  }
};

__device__ __forceinline__ longlong2 item_entry(const Cursor& c, int MC, const longlong2* __restrict__ tab) {
  return c.cid < MC ? tab[c.cid] : make_longlong2(0, -1ll << 32);
}
__device__ __forceinline__ bool decode_item(const Cursor& c, longlong2 e, Item& x) {
  if ((e.y >> 32) < 0) return false;
  x.cid = c.cid;
  x.head = c.head;
  x.t0 = e.x;
  x.len = (int)(e.y & 0xffffffff);
  return true;
}

// Valid chunks form a prefix of the chunk table, so a CTA stops at its first invalid item.
// `issue(item, stage)` runs on the last warp and starts the item's copies on full[stage];
// `zero(item, stage)` clears rows past a partial chunk; `proc(item, stage, next)` computes and
// calls next() (all threads) once its last MMA batch is issued: the last warp then starts the
// next item's copies while the tensor core runs.  If proc returns without calling it, the loop does.
template <class Issue, class Zero, class Proc>
__device__ __forceinline__ void persistent_loop(int MC, int H, const longlong2* __restrict__ tab, uint64_t* full,
                                                Issue issue, Zero zero, Proc proc) {
  const int G = gridDim.x, gq = G / H, gr = G % H;
  const bool w0 = threadIdx.x >= NT - 32;  // the last warp issues copies (thread 0 issues MMAs)
  Cursor c{(int)blockIdx.x / H, (int)blockIdx.x % H};
  Cursor c1 = c, c2;
  c1.advance(gq, gr, H);
  c2 = c1;
  c2.advance(gq, gr, H);
  Item cur;
  bool have = decode_item(c, item_entry(c, MC, tab), cur);
  longlong2 e_next = item_entry(c1, MC, tab);
  if (have && w0) issue(cur, 0);
  for (int i = 0; have; ++i) {
    const longlong2 e_after = item_entry(c2, MC, tab);
    Item nxt;
    const bool nhave = decode_item(c1, e_next, nxt);
    bool issued = false;
    auto next = [&] {
      if (!issued && nhave && w0) issue(nxt, (i + 1) & 1);
      issued = true;
    };
    counted_wait(&full[i & 1], (i >> 1) & 1);
    if (cur.len < BT) {
      zero(cur, i & 1);
      __syncthreads();
    }
    proc(cur, i & 1, next);
    next();
    fence_proxy_async();  // generic writes to this stage before the TMA refills it
    __syncthreads();
    cur = nxt;
    have = nhave;
    e_next = e_after;
    c1 = c2;
    c2.advance(gq, gr, H);
  }
}

// --------------------------------------------------------------------------- local state
// stage: a tile | b tile | raw gate
template <typename Tg> __host__ __device__ constexpr int ls_stage_bytes() { return 2 * TILE + BT * D * (int)sizeof(Tg); }

template <typename T, typename Tg>
__global__ void __launch_bounds__(NT, 2) tc_local_state_kernel(
    const __grid_constant__ CUtensorMap ma, const __grid_constant__ CUtensorMap mb,
    const __grid_constant__ CUtensorMap mg, int mode, const longlong2* __restrict__ chunk_tab, int MC, int H,
    float scale, float* __restrict__ dS, float* __restrict__ decay) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  constexpr int STAGE = ls_stage_bytes<Tg>();
  GateSmem& G = *reinterpret_cast<GateSmem*>(smem + 2 * STAGE);
  __shared__ uint64_t mbar, full[2];
  __shared__ uint32_t tbase_s;
  const int tid = threadIdx.x, warp = tid >> 5;
  griddep_launch_dependents();
  if (warp == 0) tmem_alloc(&tbase_s, 64);
  if (tid == 0) {
    mbar_init(&mbar, 1);
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  fence_after();
  const uint32_t tb = tbase_s;
  uint32_t phase = 0;
  const Epi ep;
  const Own me;
  const CUtensorMap* m16[2] = {&ma, &mb};
  if (tid == 0)
    for (const CUtensorMap* m : {&ma, &mb, &mg}) prefetch_tensormap(m);
  griddep_wait();  // predecessors wrote the chunk table / states this kernel reads
  persistent_loop(
      MC, H, chunk_tab, full,
      [&](const Item& x, int st) {
        unsigned char* b = smem + st * STAGE;
        issue_loads(b, m16, 2, b + 2 * TILE, &mg, BT * D * sizeof(Tg), nullptr, nullptr, 0, 0, x.t0, x.head,
                    &full[st]);
      },
      [&](const Item& x, int st) {
        unsigned char* b = smem + st * STAGE;
        zero_tail<Tg>(b, 2, b + 2 * TILE, x.len);
      },
      [&](const Item& x, int st, auto& next) {
        next();  // short items: the next item's copies start right away
        unsigned char* sA = smem + st * STAGE;
        unsigned char* sB = sA + TILE;
        gate_apply_local<T, Tg>(G, sB + TILE, sA, mode, scale);
        operands_ready();
        if (tid == 0) {
          mma64(tb, sA, 1, sB, 1, idesc_f16(64, 64, Fmt<T>::v, 1, 1), false);
          commit(&mbar);
        }
        wait_mma(&mbar, phase);
        float v[8];
        ep.load(tb, v);
        float* out = dS + ((int64_t)x.cid * H + x.head) * D * D;
#pragma unroll
        for (int p = 0; p < 4; ++p)
          *reinterpret_cast<float2*>(out + ep.row(p) * D + ep.col(p)) = make_float2(v[2 * p], v[2 * p + 1]);
        if (tid < D) decay[((int64_t)x.cid * H + x.head) * D + tid] = __expf(G.gl[tid]);
        fence_before();
      });
  __syncthreads();
  fence_after();
  if (warp == 0) tmem_dealloc(tb, 64);
}

// --------------------------------------------------------------------------- forward output
// stage: q | k | v tiles | fp32 chunk-start state (its first 8 KB become the 16-bit H' tile) |
// raw gate.  Q^ and K^ are gated in place.
template <typename Tg> __host__ __device__ constexpr int fo_stage_bytes() { return 3 * TILE + STATE + BT * D * (int)sizeof(Tg); }

template <typename T, typename Tg>
__global__ void __launch_bounds__(NT, 1) tc_fwd_o_kernel(
    const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
    const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mg,
    const __grid_constant__ CUtensorMap mh, const longlong2* __restrict__ chunk_tab, int MC, int H, float scale,
    T* __restrict__ o, int* __restrict__ flags) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  constexpr int STAGE = fo_stage_bytes<Tg>();
  unsigned char* sA = smem + 2 * STAGE;
  GateSmem& G = *reinterpret_cast<GateSmem*>(sA + TILE);
  __shared__ uint64_t mbar, full[2];
  __shared__ uint32_t tbase_s;
  const int tid = threadIdx.x, warp = tid >> 5;
  griddep_launch_dependents();
  if (warp == 0) tmem_alloc(&tbase_s, 128);
  if (tid == 0) {
    mbar_init(&mbar, 1);
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  fence_after();
  const uint32_t tb = tbase_s;
  uint32_t phase = 0;
  const Epi ep;
  const Own me;
  const CUtensorMap* m16[3] = {&mq, &mk, &mv};
  if (tid == 0)
    for (const CUtensorMap* m : {&mq, &mk, &mv, &mg, &mh}) prefetch_tensormap(m);
  constexpr uint32_t F = Fmt<T>::v;
  griddep_wait();  // predecessors wrote the chunk table / states this kernel reads
  persistent_loop(
      MC, H, chunk_tab, full,
      [&](const Item& x, int st) {
        unsigned char* b = smem + st * STAGE;
        unsigned char* sd[1] = {b + 3 * TILE};
        const CUtensorMap* ms[1] = {&mh};
        issue_loads(b, m16, 3, b + 3 * TILE + STATE, &mg, BT * D * sizeof(Tg), sd, ms, 1, (x.cid * H + x.head) * D,
                    x.t0, x.head, &full[st]);
      },
      [&](const Item& x, int st) {
        unsigned char* b = smem + st * STAGE;
        zero_tail<Tg>(b, 3, b + 3 * TILE + STATE, x.len);
      },
      [&](const Item& x, int st, auto& next) {
        next();  // short items: the next item's copies start right away
        unsigned char* sQ = smem + st * STAGE;
        unsigned char* sK = sQ + TILE;
        unsigned char* sV = sK + TILE;
        unsigned char* sH = sV + TILE;
        float hreg[8];
        state_regs(sH, me, hreg);
        gate_prep<Tg>(G, sH + STATE);  // its barriers order the state reads before sH writes
        const bool exact = __uint_as_float(G.span_bits) > kTcSpan;
        if (exact) {
          if (tid == 0) flags[1 + atomicAdd(flags, 1)] = x.cid * H + x.head;
          return;
        }
        gate_qk<T>(sQ, sK, sQ, sK, G, me, scale);
        operands_ready();
        if (tid == 0) mma64(tb, sQ, 0, sK, 0, idesc_f16(64, 64, F, 0, 0), false);  // A = Q^ K^^T
        {
          const float er = G.eref[me.tr];
#pragma unroll
          for (int i = 0; i < 8; ++i) hreg[i] *= er;
          *reinterpret_cast<uint4*>(sH + me.off) = pack8<T>(hreg);
        }
        operands_ready();
        if (tid == 0) {
          mma64(tb + 64, sQ, 0, sH, 1, idesc_f16(64, 64, F, 0, 1), false);  // O = Q^ H'
          commit(&mbar);
        }
        wait_mma(&mbar, phase);
        {
          float a[8];
          ep.load(tb, a);
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int r = ep.row(p), c = ep.col(p);
            st2_tile<T>(sA, r, c, c > r ? 0.f : a[2 * p], c + 1 > r ? 0.f : a[2 * p + 1]);
          }
        }
        operands_ready();
        if (tid == 0) {
          mma64(tb + 64, sA, 0, sV, 1, idesc_f16(64, 64, F, 0, 1), true);  // O += A V
          commit(&mbar);
        }
        wait_mma(&mbar, phase);
        {
          float y[8];
          ep.load(tb + 64, y);
          T* ob = o + (x.t0 * H + x.head) * D;
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int r = ep.row(p);
            if (r < x.len) st2_global<T>(ob + (int64_t)r * H * D + ep.col(p), y[2 * p], y[2 * p + 1]);
          }
        }
        fence_before();
      });
  __syncthreads();
  fence_after();
  if (warp == 0) tmem_dealloc(tb, 128);
}

// --------------------------------------------------------------------------- backward
// stage: q | k | v | do tiles | fp32 state h | fp32 adjoint dh (the first 8 KB of each become
// the 16-bit H' / dH' tiles) | raw gate.  Gated Q^, K^ and the score tiles A, dA are working
// tiles outside the stages; the raw q and k stay in the stage for dg.
template <typename Tg> __host__ __device__ constexpr int bw_stage_bytes() { return 4 * TILE + 2 * STATE + BT * D * (int)sizeof(Tg); }

template <typename T, typename Tg>
__global__ void __launch_bounds__(NT, 1) tc_bwd_kernel(
    const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
    const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mdo,
    const __grid_constant__ CUtensorMap mg, const __grid_constant__ CUtensorMap mh,
    const __grid_constant__ CUtensorMap mdh, const longlong2* __restrict__ chunk_tab, int MC, int H,
    float scale, T* __restrict__ dq,
    T* __restrict__ dk, T* __restrict__ dv, float* __restrict__ dg, int* __restrict__ flags) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  constexpr int STAGE = bw_stage_bytes<Tg>();
  unsigned char* sQg = smem + 2 * STAGE;
  unsigned char* sKg = sQg + TILE;
  unsigned char* sA = sKg + TILE;
  unsigned char* sdA = sA + TILE;
  GateSmem& G = *reinterpret_cast<GateSmem*>(sdA + TILE);
  __shared__ uint64_t mbar[2], full[2];  // mbar[0]: score batch, then dq / dk;  mbar[1]: dv
  __shared__ uint32_t tbase_s;
  __shared__ float s_hd8[8][D], s_dgl[D];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  griddep_launch_dependents();
  if (warp == 0) tmem_alloc(&tbase_s, 256);
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&mbar[i], 1);
      mbar_init(&full[i], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  fence_after();
  const uint32_t tb = tbase_s;
  uint32_t phase = 0, phase_dv = 0;
  const Epi ep;
  const Own me;
  const CUtensorMap* m16[4] = {&mq, &mk, &mv, &mdo};
  if (tid == 0)
    for (const CUtensorMap* m : {&mq, &mk, &mv, &mdo, &mg, &mh, &mdh}) prefetch_tensormap(m);
  constexpr uint32_t F = Fmt<T>::v;
  griddep_wait();  // predecessors wrote the chunk table / states this kernel reads
  persistent_loop(
      MC, H, chunk_tab, full,
      [&](const Item& x, int st) {
        unsigned char* b = smem + st * STAGE;
        unsigned char* sd[2] = {b + 4 * TILE, b + 4 * TILE + STATE};
        const CUtensorMap* ms[2] = {&mh, &mdh};
        issue_loads(b, m16, 4, b + 4 * TILE + 2 * STATE, &mg, BT * D * sizeof(Tg), sd, ms, 2,
                    (x.cid * H + x.head) * D, x.t0, x.head, &full[st]);
      },
      [&](const Item& x, int st) {
        unsigned char* b = smem + st * STAGE;
        zero_tail<Tg>(b, 4, b + 4 * TILE + 2 * STATE, x.len);
      },
      [&](const Item& x, int st, auto& next) {
        unsigned char* rQ = smem + st * STAGE;
        unsigned char* rK = rQ + TILE;
        unsigned char* sV = rK + TILE;
        unsigned char* sDO = sV + TILE;
        unsigned char* sH = sDO + TILE;
        unsigned char* sDH = sH + STATE;
        float hreg[8], dhreg[8];
        state_regs(sH, me, hreg);
        state_regs(sDH, me, dhreg);
        gate_prep<Tg>(G, sDH + STATE);  // its barriers order the state reads before sH/sDH writes
        const bool exact = __uint_as_float(G.span_bits) > kTcSpan;
        if (exact) {
          if (tid == 0) flags[1 + atomicAdd(flags, 1)] = x.cid * H + x.head;
          return;
        }
        gate_qk<T>(rQ, rK, sQg, sKg, G, me, scale);
        operands_ready();
        if (tid == 0) {
          mma64(tb, sQg, 0, sKg, 0, idesc_f16(64, 64, F, 0, 0), false);       // A  = Q^ K^^T
          mma64(tb + 64, sDO, 0, sV, 0, idesc_f16(64, 64, F, 0, 0), false);   // dA = do v^T
          mma64(tb + 128, sKg, 1, sV, 1, idesc_f16(64, 64, F, 1, 1), false);  // S  = K^^T v
          commit(&mbar[0]);
        }
        // H', dH' tiles and h.dh per row while the score batch runs
        {
          const float er = G.eref[me.tr], egl = G.egl[me.tr];
          float hd = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            hd = fmaf(hreg[i], dhreg[i], hd);
            hreg[i] *= er;
            dhreg[i] *= egl;
          }
          s_hd8[me.tc >> 3][me.tr] = hd;
          *reinterpret_cast<uint4*>(sH + me.off) = pack8<T>(hreg);
          *reinterpret_cast<uint4*>(sDH + me.off) = pack8<T>(dhreg);
        }
        fence_proxy_async();
        __syncthreads();
        wait_mma(&mbar[0], phase);
        {
          float a[8], b[8], z[8];
          ep.load(tb, a);
          ep.load(tb + 64, b);
          ep.load(tb + 128, z);
          float dgl0 = 0.f, dgl1 = 0.f;  // rows r0, r0 + 8
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int r = ep.row(p), c = ep.col(p);
            const bool m0 = c > r, m1 = c + 1 > r;
            st2_tile<T>(sA, r, c, m0 ? 0.f : a[2 * p], m1 ? 0.f : a[2 * p + 1]);
            st2_tile<T>(sdA, r, c, m0 ? 0.f : b[2 * p], m1 ? 0.f : b[2 * p + 1]);
            // row r of S is key index r: dh'[r, :] . S[r, :]
            float d0, d1;
            ld2_tile<T>(sDH, r, c, d0, d1);
            const float t = fmaf(d0, z[2 * p], d1 * z[2 * p + 1]);
            if (p & 1) dgl1 += t; else dgl0 += t;
          }
          dgl0 += __shfl_xor_sync(0xffffffffu, dgl0, 1);
          dgl0 += __shfl_xor_sync(0xffffffffu, dgl0, 2);
          dgl1 += __shfl_xor_sync(0xffffffffu, dgl1, 1);
          dgl1 += __shfl_xor_sync(0xffffffffu, dgl1, 2);
          if ((lane & 3) == 0) {
            G.part[warp >> 2][ep.r0] = dgl0;
            G.part[warp >> 2][ep.r0 + 8] = dgl1;
          }
        }
        operands_ready();
        if (tid == 0) {
          mma64(tb + 192, sA, 1, sDO, 1, idesc_f16(64, 64, F, 1, 1), false);  // dv  = A^T do
          mma64(tb + 192, sKg, 0, sDH, 1, idesc_f16(64, 64, F, 0, 1), true);  //     + K^ dh'
          commit(&mbar[1]);
          mma64(tb, sDO, 0, sH, 0, idesc_f16(64, 64, F, 0, 0), false);        // dq~ = do H'^T
          mma64(tb, sdA, 0, sKg, 1, idesc_f16(64, 64, F, 0, 1), true);        //     + dA K^
          mma64(tb + 64, sV, 0, sDH, 0, idesc_f16(64, 64, F, 0, 0), false);   // dk~ = v dh'^T
          mma64(tb + 64, sdA, 1, sQg, 1, idesc_f16(64, 64, F, 1, 1), true);   //     + dA^T Q^
          commit(&mbar[0]);
        }
        next();
        // dgL per key index: exp(gL) h.dh + dh'.(K^^T v)
        if (tid < D) {
          float sp = 0.f, hdh = 0.f;
#pragma unroll
          for (int j = 0; j < NWARP / 4; ++j) sp += G.part[j][tid];
#pragma unroll
          for (int j = 0; j < 8; ++j) hdh += s_hd8[j][tid];
          s_dgl[tid] = G.eref[tid] * G.egl[tid] * hdh + sp;
        }
        const int64_t base = (x.t0 * H + x.head) * D;
        wait_mma(&mbar[1], phase_dv);
        {
          float z[8];
          ep.load(tb + 192, z);
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int r = ep.row(p);
            if (r < x.len) st2_global<T>(dv + base + (int64_t)r * H * D + ep.col(p), z[2 * p], z[2 * p + 1]);
          }
        }
        wait_mma(&mbar[0], phase);
        {
          float a[8], b[8];
          ep.load(tb, a);
          ep.load(tb + 64, b);
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int r = ep.row(p), c = ep.col(p);
            float* e = G.E + r * LDG + c;
            const float e0 = e[0], e1 = e[1];
            const float q0 = a[2 * p] * (scale * e0), q1 = a[2 * p + 1] * (scale * e1);
            const float k0 = __fdividef(b[2 * p], e0), k1 = __fdividef(b[2 * p + 1], e1);
            float rq0, rq1, rk0, rk1;
            ld2_tile<T>(rQ, r, c, rq0, rq1);
            ld2_tile<T>(rK, r, c, rk0, rk1);
            e[0] = rq0 * q0 - rk0 * k0;  // dgc
            e[1] = rq1 * q1 - rk1 * k1;
            if (r < x.len) {
              const int64_t off = base + (int64_t)r * H * D + c;
              st2_global<T>(dq + off, q0, q1);
              st2_global<T>(dk + off, k0, k1);
            }
          }
        }
        fence_before();
        __syncthreads();
        // dg = reverse cumulative sum over rows of dgc (+ dgL at every row): NG groups of RG rows
        {
          const int c = tid & 63, qt = tid >> 6;
          float y[RG];
          float run = 0.f;
#pragma unroll
          for (int i = RG - 1; i >= 0; --i) {
            run += G.E[(RG * qt + i) * LDG + c];
            y[i] = run;
          }
          G.part[qt][c] = run;
          __syncthreads();
          float after = s_dgl[c];
          for (int j = qt + 1; j < NG; ++j) after += G.part[j][c];
          float* dst = dg + base + (int64_t)RG * qt * H * D + c;
#pragma unroll
          for (int i = 0; i < RG; ++i)
            if (RG * qt + i < x.len) dst[(int64_t)i * H * D] = y[i] + after;
        }
      });
  __syncthreads();
  fence_after();
  if (warp == 0) tmem_dealloc(tb, 256);
}

template <typename K_>
int prepare(K_ kern, size_t smem) {
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
      cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess) {
    set_error("chunk_gla tensor-core kernel: cannot reserve %zu bytes of shared memory", smem);
    return SSLA_ERR_CUDA;
  }
  return SSLA_OK;
}

// Persistent grid: as many CTAs as fit on the device at once (shared memory and TMEM columns
// permitting), capped by the number of items.
template <typename K_>
int persistent_grid(K_ kern, size_t smem, int tmem_cols, int64_t items, unsigned& grid) {
  int rc = prepare(kern, smem);
  if (rc) return rc;
  // CTAs per SM from the kernel's own resources (the occupancy query can report the pre-launch
  // shared-memory configuration on a kernel's first call): 228 KB of shared memory per SM with
  // 1 KB reserved per CTA, 64K registers allocated per warp in multiples of 8 per thread,
  // 2048 threads, 512 TMEM columns.
  int dev = 0, sms = 0;
  cudaFuncAttributes fa;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaFuncGetAttributes(&fa, kern) != cudaSuccess) {
    set_error("chunk_gla tensor-core kernel: attribute query failed");
    return SSLA_ERR_CUDA;
  }
  const int by_smem = (int)((228 * 1024) / (smem + fa.sharedSizeBytes + 1024));
  const int by_regs = 65536 / (((fa.numRegs + 7) / 8) * 8 * NT);
  int per_sm = by_smem < by_regs ? by_smem : by_regs;
  if (per_sm > 2048 / NT) per_sm = 2048 / NT;
  if (per_sm * tmem_cols > 512) per_sm = 512 / tmem_cols;
  if (per_sm < 1) {
    set_error("chunk_gla tensor-core kernel: %zu bytes of shared memory do not fit an SM", smem);
    return SSLA_ERR_CUDA;
  }
  const int64_t cap = (int64_t)per_sm * sms;
  grid = (unsigned)(items < cap ? items : cap);
  return SSLA_OK;
}

// ---------------------------------------------------------------------------- tensor maps
int encode(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
           const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw) {
  return tma::encode(m, dt, rank, base, dims, strides, box, sw, "chunk_gla");
}

// 3-D view (D = 64, H, T) of a [T, H, 64] token array, box 64 x 1 x 64: 16-bit operands with
// the 128-byte swizzle, the gate (any dtype) unswizzled.
int make_map(CUtensorMap* m, const void* base, int dtype, int64_t T, int64_t H, bool swizzle) {
  const int eb = dtype == SSLA_F32 ? 4 : 2;
  const CUtensorMapDataType dt = dtype == SSLA_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == SSLA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T};
  const cuuint64_t strides[2] = {(cuuint64_t)D * eb, (cuuint64_t)H * D * eb};
  const cuuint32_t box[3] = {(cuuint32_t)D, 1u, (cuuint32_t)BT};
  return encode(m, dt, 3, base, dims, strides, box, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
}

// 2-D view [rows, 64] of fp32 states (64 rows per (chunk, head)), box 32 columns x 64 rows,
// 128-byte swizzle.
int make_state_map(CUtensorMap* m, const float* base, int64_t rows) {
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)D * 4};
  const cuuint32_t box[2] = {32u, (cuuint32_t)D};
  return encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
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

// Item indices and TMA row coordinates are 32-bit.
int check_sizes(int64_t T, int64_t MC, int64_t H) {
  if (MC * H * D >= (int64_t)1 << 31 || T >= (int64_t)1 << 31) {
    set_error("chunk_gla tensor-core kernels: T=%lld or %lld chunk-heads x 64 exceed the 2^31 limit",
              (long long)T, (long long)(MC * H));
    return SSLA_ERR_UNSUPPORTED;
  }
  return SSLA_OK;
}

}  // namespace

int tc_supported(int dtype, int dtype_g, int64_t K, int64_t V) {
  return (dtype == SSLA_BF16 || dtype == SSLA_F16) && (dtype_g == dtype || dtype_g == SSLA_F32) &&
         K == D && V == D;
}

int tc_aligned(const void* const* ptrs, int n) {
  for (int i = 0; i < n; ++i)
    if (reinterpret_cast<uintptr_t>(ptrs[i]) % 16) return 0;
  return 1;
}

int tc_local_state(int dtype, int dtype_g, int mode, const void* a_src, const void* b_src, const void* g,
                   const longlong2* chunk_tab, int64_t T, int64_t MC, int64_t H, float scale, float* dS,
                   float* decay, cudaStream_t s) {
  if (MC * H == 0) return SSLA_OK;
  if (int rc = check_sizes(T, MC, H)) return rc;
  CUtensorMap ma, mb, mg;
  int rc;
  if ((rc = make_map(&ma, a_src, dtype, T, H, true)) || (rc = make_map(&mb, b_src, dtype, T, H, true)) ||
      (rc = make_map(&mg, g, dtype_g, T, H, false)))
    return rc;
  return SSLA_DISPATCH_TC(dtype, dtype_g, T_, Tg, [&] {
    auto kern = tc_local_state_kernel<T_, Tg>;
    const size_t smem = 2 * ls_stage_bytes<Tg>() + kGateBytes + kAlignSlack;
    unsigned grid = 0;
    int rc2 = persistent_grid(kern, smem, 64, MC * H, grid);
    if (rc2) return rc2;
    launch_pdl(kern, dim3(grid), dim3(NT), smem, s, ma, mb, mg, mode, chunk_tab, (int)MC, (int)H, scale, dS, decay);
    SSLA_CHECK_LAUNCH("chunk_gla tc_local_state");
    return SSLA_OK;
  });
}

int tc_fwd_o(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
             const longlong2* chunk_tab, int64_t T, int64_t MC, int64_t H, float scale, const float* states,
             void* o, int* flags, cudaStream_t s) {
  if (MC * H == 0) return SSLA_OK;
  if (int rc = check_sizes(T, MC, H)) return rc;
  CUtensorMap mq, mk, mv, mg, mh;
  int rc;
  if ((rc = make_map(&mq, q, dtype, T, H, true)) || (rc = make_map(&mk, k, dtype, T, H, true)) ||
      (rc = make_map(&mv, v, dtype, T, H, true)) || (rc = make_map(&mg, g, dtype_g, T, H, false)) ||
      (rc = make_state_map(&mh, states, MC * H * D)))
    return rc;
  return SSLA_DISPATCH_TC(dtype, dtype_g, T_, Tg, [&] {
    auto kern = tc_fwd_o_kernel<T_, Tg>;
    const size_t smem = 2 * fo_stage_bytes<Tg>() + TILE + kGateBytes + kAlignSlack;
    unsigned grid = 0;
    int rc2 = persistent_grid(kern, smem, 128, MC * H, grid);
    if (rc2) return rc2;
    launch_pdl(kern, dim3(grid), dim3(NT), smem, s, mq, mk, mv, mg, mh, chunk_tab, (int)MC, (int)H, scale, (T_*)o,
               flags);
    SSLA_CHECK_LAUNCH("chunk_gla tc_fwd_o");
    return SSLA_OK;
  });
}

int tc_bwd(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
           const longlong2* chunk_tab, int64_t T, int64_t MC, int64_t H, float scale, const float* states,
           const float* dstates, const void* dout, void* dq, void* dk, void* dv, float* dg, int* flags,
           cudaStream_t s) {
  if (MC * H == 0) return SSLA_OK;
  if (int rc = check_sizes(T, MC, H)) return rc;
  CUtensorMap mq, mk, mv, mdo, mg, mh, mdh;
  int rc;
  if ((rc = make_map(&mq, q, dtype, T, H, true)) || (rc = make_map(&mk, k, dtype, T, H, true)) ||
      (rc = make_map(&mv, v, dtype, T, H, true)) || (rc = make_map(&mdo, dout, dtype, T, H, true)) ||
      (rc = make_map(&mg, g, dtype_g, T, H, false)) || (rc = make_state_map(&mh, states, MC * H * D)) ||
      (rc = make_state_map(&mdh, dstates, MC * H * D)))
    return rc;
  return SSLA_DISPATCH_TC(dtype, dtype_g, T_, Tg, [&] {
    auto kern = tc_bwd_kernel<T_, Tg>;
    const size_t smem = 2 * bw_stage_bytes<Tg>() + 4 * TILE + kGateBytes + kAlignSlack;
    unsigned grid = 0;
    int rc2 = persistent_grid(kern, smem, 256, MC * H, grid);
    if (rc2) return rc2;
    launch_pdl(kern, dim3(grid), dim3(NT), smem, s, mq, mk, mv, mdo, mg, mh, mdh, chunk_tab, (int)MC, (int)H, scale,
               (T_*)dq, (T_*)dk, (T_*)dv, dg, flags);
    SSLA_CHECK_LAUNCH("chunk_gla tc_bwd");
    return SSLA_OK;
  });
}

int tc_timeouts(int reset, unsigned* count) {
  if (cudaMemcpyFromSymbol(count, g_wait_timeouts, sizeof(unsigned)) != cudaSuccess) {
    set_error("chunk_gla: cannot read the wait-timeout counter");
    return SSLA_ERR_CUDA;
  }
  if (reset) {
    const unsigned zero = 0;
    if (cudaMemcpyToSymbol(g_wait_timeouts, &zero, sizeof(unsigned)) != cudaSuccess) {
      set_error("chunk_gla: cannot reset the wait-timeout counter");
      return SSLA_ERR_CUDA;
    }
  }
  return SSLA_OK;
}

}  // namespace chunk
}  // namespace ssla

extern "C" int ssla_chunk_gla_tc_timeouts(int reset, unsigned* count) { return ssla::chunk::tc_timeouts(reset, count); }
