// Tensor-core (tcgen05 / TMEM) kernels of the chunked GLA path for 16-bit inputs, K = V = 64.
//
// Work item = (64-token chunk, head).  CTAs of 256 threads (8 warps), several resident per SM
// so that the serial chain of one item (gate prefix sums, gating, MMA batches, epilogues) of
// one CTA overlaps the chains and copies of the others.  A CTA walks items blockIdx.x,
// blockIdx.x + gridDim.x, ...; with two shared-memory stages the next item's tiles are copied
// while the current one is computed, with one stage the next copy starts when the item is
// done.  Loads are TMA, issued by the last warp: one tensor copy per 64x64 16-bit tile (q, k,
// v, do and the chunk-start states) and one for the raw gate, all completing on the stage's
// mbarrier.  16-bit tiles use the 128-byte swizzle: row r occupies bytes r*128 .. r*128+127
// with its 16-byte piece j at piece position j ^ (r % 8); such a tile is a K-major operand
// (rows = M/N) or an MN-major operand (rows = K) of tcgen05.mma through SWIZZLE_128B
// descriptors.  Thread 0 issues 64x64x16 tcgen05.mma instructions into fp32 TMEM
// accumulators; the epilogues read TMEM with the 16x256b shape (an M=64 accumulator fills
// lanes 0-15 of each TMEM subpartition): warps w and w+4 share subpartition w % 4 and take 32
// accumulator columns each.
//
// Gating: with gc the in-chunk cumulative log decay, ref = gc of the chunk's 32nd row and
// E = exp(gc - ref) (the only exponentials of the output / backward kernels),
//   Q^ = scale q E,  K^ = k / E,  H' = exp(ref) h,  dH' = exp(gL - ref) dh,
// so that (the algebra of ops/gla/chunk.py:23-249 and :253-641)
//   A   = tril(Q^ K^^T)                       o  = Q^ H' + A v
//   dv  = A^T do + K^ dH'                      dq = scale E * (do H'^T + dA K^)
//   dk  = (v dH'^T + dA^T Q^) / E              dA = tril(do v^T)
//   dg  = reverse-cumsum_rows(q dq - k dk) + H'.dH' + dH'.(K^^T v)      (the last two per key)
// H' and dH' arrive ready-made in the operand dtype: the state scans (chunk_gla.cu) multiply
// by the per-chunk factors exp(ref) / exp(gL - ref) that the local-state pass writes.
// Local state: mode 0 dS = (k exp(gL - gc))^T v, mode 1 dS = (scale q exp(gc))^T do, with
// per-element exponents.  Every factor of the output and backward kernels is bounded by
// exp(span/2), span = the chunk's decay range; mode 0 flags (chunk, head) items with span >
// kTcSpan in `xflag`, and the exact CUDA-core kernels (chunk_gla.cu) recompute those.
//
// Bounded waits: a wait that gives up is counted (ssla_chunk_gla_tc_timeouts) and marks the
// CTA bad; a bad CTA writes NaN into the outputs of its current and remaining items, waits
// (bounded) for its copies in flight, releases its tensor memory and exits.
#include <cuda.h>

#include "chunk_gla.cuh"
#include "tc_util.cuh"
#include "tma_map.cuh"

namespace ssla {
namespace chunk {
namespace {

using namespace ssla::tc;

constexpr int NT = 256;
constexpr int D = 64;                 // K = V = 64
constexpr int NWARP = NT / 32;
constexpr int NG = NT / 64;           // gate-scan groups: thread (column, group) owns RG rows
constexpr int RG = BT / NG;
constexpr int LDG = D + 1;            // fp32 gate tile stride
constexpr float kTcSpan = 40.f;
constexpr int TILE = BT * D * 2;      // bytes of one 64x64 16-bit tile
static_assert(NT == 4 * 64 && NWARP == 8, "epilogue / ownership geometry assumes 8 warps");
static_assert(31 % RG == RG - 1, "row 31 must end a gate-scan group");

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

// SWIZZLE_128B descriptor of such a tile (1024-byte aligned).  Within one 64x64x16 MMA the
// only stride the tensor core needs is between groups of 8 rows along the tile (1024 bytes;
// given as both LBO and SBO).  A k-step of 16 elements advances the start address by 32 bytes
// (K-major: within the swizzled row) or 2048 bytes (MN-major: 16 rows).
__device__ __forceinline__ uint64_t desc_sw128(const void* tile) {
  return smem_desc(smem_u32(tile), 1024u, 1024u) | ((uint64_t)2 << 61);
}

template <typename T> __device__ __forceinline__ void st2_tile(unsigned char* tile, int r, int c, float a, float b) {
  *reinterpret_cast<uint32_t*>(tile + toff(r, c)) = pack2<T>(a, b);
}
template <typename T> __device__ __forceinline__ void ld2_tile(const unsigned char* tile, int r, int c, float& a, float& b) {
  unpack2<T>(*reinterpret_cast<const uint32_t*>(tile + toff(r, c)), a, b);
}
template <typename T> __device__ __forceinline__ void st2_global(T* p, float a, float b) {
  *reinterpret_cast<uint32_t*>(p) = pack2<T>(a, b);
}

constexpr float kNaN = __builtin_nanf("");

struct GateSmem {
  float E[BT * LDG];  // exp(gc - ref); dgc scratch in the backward
  float part[NG][D];  // per-group partial sums (gate scan, dgL, dg reverse cumsum)
};

// Barrier over the NT compute threads (named barrier 1; a producer warp, where a kernel has
// one, never joins it).
__device__ __forceinline__ void cbar() { named_barrier(1, NT); }

// Thread t owns row tr = t % 64, 16-byte pieces at columns tc .. tc+7 and tc+32 .. tc+39
// (tc = 8 * (t / 64)) of every 16-bit tile in the gating and tail-zeroing passes.
struct Own {
  int tr, tc, off0, off1;
  __device__ __forceinline__ Own()
      : tr(threadIdx.x & 63), tc((threadIdx.x >> 6) << 3), off0(toff(tr, tc)), off1(toff(tr, tc + 32)) {}
};

// Epilogue geometry (16x256b.x4): this warp reads TMEM subpartition sp, accumulator columns
// c0 .. c0+31; pair p (0..7) of the 16 values holds row r0 + 8*(p&1), columns
// cc + 8*(p>>1) + {0, 1}.
struct Epi {
  int sp, c0, r0, cc;
  __device__ __forceinline__ Epi() {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    sp = warp & 3;
    c0 = (warp >> 2) * 32;
    r0 = 16 * sp + (lane >> 2);
    cc = c0 + 2 * (lane & 3);
  }
  __device__ __forceinline__ int row(int p) const { return r0 + 8 * (p & 1); }
  __device__ __forceinline__ int col(int p) const { return cc + 8 * (p >> 1); }
  __device__ __forceinline__ uint32_t addr(uint32_t tbase) const { return tmem_addr(tbase, sp, c0); }
};

template <int N>
__device__ __forceinline__ void ld_acc(const Epi& ep, const uint32_t (&tb)[N], float (&v)[N][16]) {
  uint32_t r[N][16];
#pragma unroll
  for (int i = 0; i < N; ++i) tmem_ld16x256b_x4_nowait(ep.addr(tb[i]), r[i]);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < N; ++i) {
    reg_fence16(r[i]);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[i][j] = __uint_as_float(r[i][j]);
  }
}

// Issued by one warp: n16 16-bit tiles (3-D token maps m16[i], views (D, H, T), box 64 x 1 x
// 64) into dst16 + i*TILE, the raw gate (map mg, unswizzled) and nst 16-bit state tiles (2-D
// map over [items * 64 rows, 64], rows srow..srow+63) into sdst[i], all completing on `bar`.
__device__ __forceinline__ void issue_loads(unsigned char* dst16, const CUtensorMap* const* m16, int n16,
                                            unsigned char* graw, const CUtensorMap* mg, uint32_t gbytes,
                                            unsigned char* const* sdst, const CUtensorMap* const* ms, int nst,
                                            int srow, int64_t t0, int head, uint64_t* bar) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) mbar_arrive_expect_tx(bar, (n16 + nst) * TILE + gbytes);
  __syncwarp();
  if (lane < n16) tma_load_3d(dst16 + lane * TILE, m16[lane], 0, head, (int)t0, bar);
  if (lane == 8) tma_load_3d(graw, mg, 0, head, (int)t0, bar);
  if (lane >= 16 && lane < 16 + nst) tma_load_2d(sdst[lane - 16], ms[lane - 16], 0, srow, bar);
}

// Rows >= len of a partial chunk (the TMA box reads past the chunk): zero them in the n16
// token tiles and the raw gate.
template <typename Tg>
__device__ __forceinline__ void zero_tail(unsigned char* dst16, int n16, unsigned char* graw, int len, const Own& me) {
  if (me.tr >= len)
    for (int i = 0; i < n16; ++i) {
      *reinterpret_cast<uint4*>(dst16 + i * TILE + me.off0) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(dst16 + i * TILE + me.off1) = make_uint4(0, 0, 0, 0);
    }
  constexpr int PER_ROW = D * (int)sizeof(Tg) / 16;
#pragma unroll
  for (int j = 0; j < BT * PER_ROW / NT; ++j) {
    const int e = threadIdx.x + j * NT;
    if (e / PER_ROW >= len) *reinterpret_cast<uint4*>(graw + 16 * e) = make_uint4(0, 0, 0, 0);
  }
}

// E = exp(gc - ref) from the staged raw gate tile.  Thread (column c = tid % 64, group
// q = tid / 64) scans rows RG*q .. RG*q+RG-1 of its column serially in registers; the group
// offsets and ref (gc of row 31, the end of group 31 / RG) come from the group totals.
template <typename Tg>
__device__ __forceinline__ void gate_prep(float* __restrict__ E, float (*part)[D], const unsigned char* raw) {
  const int tid = threadIdx.x, c = tid & 63, qt = tid >> 6;
  const Tg* gr = reinterpret_cast<const Tg*>(raw);
  float x[RG];
  float run = 0.f;
#pragma unroll
  for (int i = 0; i < RG; ++i) {
    run += ldf(gr + (RG * qt + i) * D + c);
    x[i] = run;
  }
  part[qt][c] = run;
  cbar();
  float off = 0.f, ref = 0.f;
#pragma unroll
  for (int j = 0; j < NG; ++j) {
    const float pj = part[j][c];
    if (j < qt) off += pj;
    if (j <= 31 / RG) ref += pj;
  }
#pragma unroll
  for (int i = 0; i < RG; ++i) E[(RG * qt + i) * LDG + c] = __expf((x[i] + off) - ref);
  cbar();
}

// Gate the staged q and k chunks of this thread: Q^ = scale q E, K^ = k / E, written to dQ /
// dK (which may be the source tiles themselves).
template <typename T>
__device__ __forceinline__ void gate_qk(const unsigned char* sQ, const unsigned char* sK, unsigned char* dQ,
                                        unsigned char* dK, const float* __restrict__ E, const Own& me, float scale) {
  // loads of both pieces before any store (dQ, dK may be the source tiles)
  uint4 uq[2], uk[2];
  float e[2][8];
#pragma unroll
  for (int pc = 0; pc < 2; ++pc) {
    const int off = pc ? me.off1 : me.off0;
    uq[pc] = *reinterpret_cast<const uint4*>(sQ + off);
    uk[pc] = *reinterpret_cast<const uint4*>(sK + off);
    const float* ep = E + me.tr * LDG + me.tc + 32 * pc;
#pragma unroll
    for (int i = 0; i < 8; ++i) e[pc][i] = ep[i];
  }
#pragma unroll
  for (int pc = 0; pc < 2; ++pc) {
    const int off = pc ? me.off1 : me.off0;
    const T* xq = reinterpret_cast<const T*>(&uq[pc]);
    const T* xk = reinterpret_cast<const T*>(&uk[pc]);
    float yq[8], yk[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      yq[i] = ldf(xq + i) * (scale * e[pc][i]);
      yk[i] = __fdividef(ldf(xk + i), e[pc][i]);
    }
    *reinterpret_cast<uint4*>(dQ + off) = pack8<T>(yq);
    *reinterpret_cast<uint4*>(dK + off) = pack8<T>(yk);
  }
}

// All threads: publish smem operand writes to the tensor core and order them before the MMA.
__device__ __forceinline__ void operands_ready() {
  fence_proxy_async();
  fence_before();
  cbar();
  fence_after();
}

// Bounded waits that give up are counted here (read and reset by ssla_chunk_gla_tc_timeouts)
// and mark the CTA bad (its outputs become NaN).  Once the CTA is bad no thread waits again.
__device__ unsigned int g_wait_timeouts = 0;

__device__ __forceinline__ void counted_wait(uint64_t* mbar, uint32_t parity, volatile int* bad) {
  if (*bad) return;
  if (!mbar_wait(mbar, parity)) {
    atomicAdd(&g_wait_timeouts, 1u);
    *bad = 1;
  }
}

__device__ __forceinline__ void wait_mma(uint64_t* mbar, uint32_t& phase, volatile int* bad) {
  counted_wait(mbar, phase, bad);
  phase ^= 1u;
  fence_after();
}

// Four k-steps (K = 64) of D (+)= A * B^T; operands are 64x64 tiles read K-major or MN-major.
__device__ __forceinline__ void mma64(uint32_t d, const void* a, int a_mn, const void* b, int b_mn,
                                      uint32_t idesc, bool accumulate) {
  const uint64_t da = desc_sw128(a), db = desc_sw128(b);
  const uint64_t sa = a_mn ? 128u : 2u, sb = b_mn ? 128u : 2u;
#pragma unroll
  for (int s = 0; s < 4; ++s) mma_f16(d, da + s * sa, db + s * sb, idesc, (accumulate || s > 0) ? 1u : 0u);
}

// The 128-byte swizzle is anchored at 1024-byte boundaries: kernels align their dynamic
// shared memory explicitly (launchers reserve kAlignSlack extra bytes).
constexpr size_t kAlignSlack = 1024;
__device__ __forceinline__ unsigned char* align1024(unsigned char* p) {
  return p + ((1024u - (smem_u32(p) & 1023u)) & 1023u);
}

// Phase timing (built only with -DSSLA_PHASE_PROF, for kernel development): thread 0 of each
// CTA records clock64() at numbered points of its first kPhaseItems items into g_phase
// [CTA][item][point]; ssla_chunk_gla_phase_dump copies the table out.
#ifdef SSLA_PHASE_PROF
constexpr int kPhaseItems = 8, kPhasePts = 32, kPhaseCtas = 1024;
__device__ long long g_phase[kPhaseCtas * kPhaseItems * kPhasePts];
#define PHASE(item, k)                                                                                  \
  do {                                                                                                  \
    if (threadIdx.x == 0 && (item) < kPhaseItems && blockIdx.x < kPhaseCtas)                            \
      g_phase[(blockIdx.x * kPhaseItems + (item)) * kPhasePts + (k)] = clock64();                       \
  } while (0)
#else
#define PHASE(item, k) \
  do {                 \
  } while (0)
#endif

// --------------------------------------------------------------------------- persistent loop
struct Item {
  int64_t t0;  // first token of the chunk
  int cid, head, len;
  __device__ __forceinline__ int64_t id(int H) const { return (int64_t)cid * H + head; }
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

// Common prologue: TMEM columns, barriers, bad flag; ends with griddepcontrol.wait (the
// predecessors wrote the chunk table / states this kernel reads).
template <int NBAR>
__device__ __forceinline__ void prologue(uint32_t* tbase_s, uint32_t ncols, uint64_t* bars, volatile int* bad) {
  griddep_launch_dependents();
  if ((threadIdx.x >> 5) == 0) tmem_alloc(tbase_s, ncols);
  if (threadIdx.x == 0) {
    for (int i = 0; i < NBAR; ++i) mbar_init(&bars[i], 1);
    *bad = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  fence_after();
}


// --------------------------------------------------------------------------- local state
// stage: a tile | b tile | raw gate
template <typename Tg> __host__ __device__ constexpr int gate_bytes() { return BT * D * (int)sizeof(Tg); }
template <typename Tg> __host__ __device__ constexpr int ls_stage_bytes() { return 2 * TILE + gate_bytes<Tg>(); }

// Local-state gate scan: thread (column pair 2 * (t % 32), group t / 32) scans LS_RG rows.
constexpr int LS_NG = NT / 32, LS_RG = BT / LS_NG;
struct LsSmem {
  alignas(16) float part[LS_NG][D];
  unsigned int span_bits;
};

// Two consecutive gate values (columns c, c + 1) of a raw, unswizzled 64 x 64 gate tile.
template <typename Tg> __device__ __forceinline__ float2 ld2_gate(const unsigned char* raw, int r, int c) {
  const Tg* p = reinterpret_cast<const Tg*>(raw) + r * D + c;
  return make_float2(ldf(p), ldf(p + 1));
}
template <> __device__ __forceinline__ float2 ld2_gate<float>(const unsigned char* raw, int r, int c) {
  return *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(raw) + r * D + c);
}

// Byte offset of fp32 element (r, c) of a 64 x 64 tile kept as two 32-column halves, each in
// the 128-byte-swizzled layout of a TMA box of 32 fp32 columns x 64 rows.
__device__ __forceinline__ int toff32(int r, int c) {
  return ((c >> 5) << 13) + (r << 7) + (((((c & 31) >> 2) ^ r) & 7) << 4) + ((c & 3) << 2);
}

// --------------------------------------------------------------------------- pipelined kernels
// tc_fwd_o (three CTAs per SM) and tc_bwd (two) run NT compute threads plus one producer warp
// per CTA.  The producer fills a ring of NS shared-memory stages by TMA, each once the consumer
// released it (the `empty` barrier: the tensor core's completion of the last MMA batch that
// reads the stage, or an arrive for items left to the exact kernels).  The compute threads run
// their items one after another; the other CTAs of the SM overlap their chains.  Outputs of whole chunks are
// staged in shared memory as swizzled tiles and written by TMA stores; rows of a partial chunk
// (the next sequence's tokens follow them) are stored directly.

// Producer: for the CTA's j-th item, wait until stage j % NS is released by item j - NS, then
// issue the item's copies on full[j % NS].
template <int NS, class Issue>
__device__ __forceinline__ void producer_loop(int MC, int H, const longlong2* __restrict__ tab, uint64_t* full,
                                              uint64_t* empty, volatile int* bad, Issue issue) {
  const int G = gridDim.x, gq = G / H, gr = G % H;
  Cursor c{(int)blockIdx.x / H, (int)blockIdx.x % H};
  Item x;
  for (int j = 0; decode_item(c, item_entry(c, MC, tab), x); ++j, c.advance(gq, gr, H)) {
    const int s = j % NS;
    if (j >= NS && !mbar_wait(&empty[s], (uint32_t)(((j - NS) / NS) & 1))) {
      if ((threadIdx.x & 31) == 0) atomicAdd(&g_wait_timeouts, 1u);
      *bad = 1;
      break;
    }
    issue(x, s);
  }
}

// Consumer item walk: calls body(item, stage, parity, exact) for the CTA's items in order;
// `exact` is the item's exact-path flag (xflag, when given).  The next item's chunk-table entry
// and flag are loaded before the current body runs, so no global-load latency sits between two
// items.
template <int NS, class Body>
__device__ __forceinline__ void consumer_loop(int MC, int H, const longlong2* __restrict__ tab,
                                              const unsigned char* __restrict__ xflag, Body body) {
  const int G = gridDim.x, gq = G / H, gr = G % H;
  Cursor c{(int)blockIdx.x / H, (int)blockIdx.x % H};
  auto flag_of = [&](const Cursor& k) -> bool {
    return xflag && k.cid < MC && xflag[(int64_t)k.cid * H + k.head] != 0;
  };
  longlong2 e = item_entry(c, MC, tab);
  bool f = flag_of(c);
  Item x;
  for (int i = 0; decode_item(c, e, x); ++i) {
    Cursor cn = c;
    cn.advance(gq, gr, H);
    const longlong2 en = item_entry(cn, MC, tab);
    const bool fn = flag_of(cn);
    body(x, i % NS, (uint32_t)((i / NS) & 1), f);
    c = cn;
    e = en;
    f = fn;
  }
}

// End of a producer/consumer kernel: every thread (producer included) meets; the TMA stores of
// the last epilogue are waited for; TMEM is released.
__device__ __forceinline__ void pipeline_end(uint32_t tb, uint32_t ncols) {
  if (threadIdx.x == 0) bulk_wait_all();
  fence_before();
  __syncthreads();
  fence_after();
  if ((threadIdx.x >> 5) == 0) tmem_dealloc(tb, ncols);
}

// --------------------------------------------------------------------------- local state (pipelined)
// Four CTAs per SM, each NT compute threads + a producer warp keeping LS_NS stages of (a tile,
// b tile, raw gate) in flight; a stage is released by the tensor core's commit of the item's
// MMA.  Per item: gate prefix sums fused with the in-place scaling of the a tile, one 64x64x64
// MMA, the fp32 increment staged from TMEM into shared memory and written by a TMA store (the
// load/store unit stays free for the next item's shared-memory work).
constexpr int LS_NS = 1;

template <typename T, typename Tg>
__global__ void __launch_bounds__(NT + 32, 4) tc_local_state_kernel(
    const __grid_constant__ CUtensorMap ma, const __grid_constant__ CUtensorMap mb,
    const __grid_constant__ CUtensorMap mg, const __grid_constant__ CUtensorMap mds, int mode,
    const longlong2* __restrict__ chunk_tab, int MC, int H, float scale, float* __restrict__ dS,
    float* __restrict__ decay, float* __restrict__ escale, unsigned char* __restrict__ xflag,
    int* __restrict__ xlist) {
  constexpr int NS = LS_NS;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  constexpr int STAGE = ls_stage_bytes<Tg>();
  unsigned char* sOut = smem + NS * STAGE;  // 16 KB fp32 staging tile
  LsSmem& S = *reinterpret_cast<LsSmem*>(sOut + 2 * TILE);
  __shared__ uint64_t bars[1 + 2 * NS];  // mma, full[NS], empty[NS]
  __shared__ uint32_t tbase_s;
  __shared__ int s_bad;
  volatile int* bad = &s_bad;
  uint64_t* mma = bars;
  uint64_t* full = bars + 1;
  uint64_t* empty = bars + 1 + NS;
  const int tid = threadIdx.x;
  prologue<1 + 2 * NS>(&tbase_s, 64, bars, bad);
  const uint32_t tb = tbase_s;
  if (tid == 0)
    for (const CUtensorMap* m : {&ma, &mb, &mg, &mds}) prefetch_tensormap(m);
  int pitem = -1;
  (void)pitem;
  griddep_wait();
  if (tid >= NT) {  // producer warp
    const CUtensorMap* m16[2] = {&ma, &mb};
    producer_loop<NS>(MC, H, chunk_tab, full, empty, bad, [&](const Item& x, int st) {
      unsigned char* b = smem + st * STAGE;
      issue_loads(b, m16, 2, b + 2 * TILE, &mg, gate_bytes<Tg>(), nullptr, nullptr, 0, 0, x.t0, x.head, &full[st]);
    });
  } else {
    uint32_t phase = 0;
    const Epi ep;
    const Own me;
    consumer_loop<NS>(MC, H, chunk_tab, nullptr, [&](const Item& x, int st, uint32_t par, bool) {
      ++pitem;
      PHASE(pitem, 21);
      counted_wait(&full[st], par, bad);
      PHASE(pitem, 16);
      unsigned char* sA = smem + st * STAGE;
      unsigned char* sB = sA + TILE;
      const int64_t item = x.id(H);
      float* out = dS + item * D * D;
      if (*bad) {  // the CTA gave up: NaN outputs, stage released
        for (int e = tid; e < D * D; e += NT) out[e] = kNaN;
        if (tid < D) decay[item * D + tid] = kNaN;
        cbar();
        if (tid == 0) mbar_arrive(&empty[st]);
        return;
      }
      if (x.len < BT) {
        zero_tail<Tg>(sA, 2, sB + TILE, x.len, me);
        cbar();
      }
      // in-chunk prefix sums of the gate, fused with the in-place scaling of the a tile:
      // mode 0 (state increment) by exp(gL - gc), mode 1 (adjoint increment) by scale exp(gc).
      // Thread (column pair c, c + 1; group qt) scans rows LS_RG * qt .. + LS_RG - 1, so every
      // shared-memory access moves two elements.
      {
        const int c = 2 * (tid & 31), qt = tid >> 5;
        if (tid == 0) S.span_bits = 0u;
        float2 xs[LS_RG];
        float r0 = 0.f, r1 = 0.f;
#pragma unroll
        for (int i = 0; i < LS_RG; ++i) {
          const float2 gv = ld2_gate<Tg>(sB + TILE, LS_RG * qt + i, c);
          r0 += gv.x;
          r1 += gv.y;
          xs[i] = make_float2(r0, r1);
        }
        PHASE(pitem, 24);
        *reinterpret_cast<float2*>(&S.part[qt][c]) = make_float2(r0, r1);
        cbar();
        PHASE(pitem, 25);
        float off0 = 0.f, off1 = 0.f, gl0 = 0.f, gl1 = 0.f, ref0 = 0.f, ref1 = 0.f;
#pragma unroll
        for (int j = 0; j < LS_NG; ++j) {
          const float2 pj = *reinterpret_cast<const float2*>(&S.part[j][c]);
          const float p0 = pj.x, p1 = pj.y;
          if (j < qt) {
            off0 += p0;
            off1 += p1;
          }
          if (j <= 31 / LS_RG) {
            ref0 += p0;
            ref1 += p1;
          }
          gl0 += p0;
          gl1 += p1;
        }
        // all loads before any store: the compiler cannot tell the tile elements apart, so
        // an interleaved load / store loop would run one pair at a time
        float m = 0.f, a0[LS_RG], a1[LS_RG];
#pragma unroll
        for (int i = 0; i < LS_RG; ++i) ld2_tile<T>(sA, LS_RG * qt + i, c, a0[i], a1[i]);
#pragma unroll
        for (int i = 0; i < LS_RG; ++i) {
          const float gc0 = xs[i].x + off0, gc1 = xs[i].y + off1;
          a0[i] *= mode == 0 ? __expf(gl0 - gc0) : scale * __expf(gc0);
          a1[i] *= mode == 0 ? __expf(gl1 - gc1) : scale * __expf(gc1);
          m = fmaxf(m, fmaxf(fabsf(gc0 - ref0), fabsf(gc1 - ref1)));
        }
#pragma unroll
        for (int i = 0; i < LS_RG; ++i) st2_tile<T>(sA, LS_RG * qt + i, c, a0[i], a1[i]);
        PHASE(pitem, 26);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((tid & 31) == 0) atomicMax(&S.span_bits, __float_as_uint(m));
        PHASE(pitem, 27);
        if (qt == 0) {
          decay[item * D + c] = __expf(gl0);
          decay[item * D + c + 1] = __expf(gl1);
          escale[item * D + c] = mode == 0 ? __expf(ref0) : __expf(gl0 - ref0);
          escale[item * D + c + 1] = mode == 0 ? __expf(ref1) : __expf(gl1 - ref1);
        }
      }
      PHASE(pitem, 17);
      if (tid == 0) bulk_wait_read_all();  // the previous item's staged tile has been stored
      operands_ready();
      if (tid == 0) {
        mma64(tb, sA, 1, sB, 1, idesc_f16(64, 64, Fmt<T>::v, 1, 1), false);
        commit(mma);
        commit(&empty[st]);  // the stage is free once the MMA has read it
        if (xflag) {
          const bool exact = __uint_as_float(S.span_bits) > kTcSpan;
          xflag[item] = exact ? 1 : 0;
          if (exact) xlist[1 + atomicAdd(xlist, 1)] = (int)item;
        }
      }
      PHASE(pitem, 18);
      wait_mma(mma, phase, bad);
      PHASE(pitem, 19);
      float v[1][16];
      ld_acc<1>(ep, {tb}, v);
      const bool poisoned = *bad;
#pragma unroll
      for (int p = 0; p < 8; ++p)
        *reinterpret_cast<float2*>(sOut + toff32(ep.row(p), ep.col(p))) =
            poisoned ? make_float2(kNaN, kNaN) : make_float2(v[0][2 * p], v[0][2 * p + 1]);
      fence_proxy_async();
      fence_before();
      cbar();
      if (tid == 0) {
        tma_store_2d(&mds, sOut, 0, (int)(item * D));
        tma_store_2d(&mds, sOut + TILE, 32, (int)(item * D));
        bulk_commit_group();
      }
      PHASE(pitem, 20);
    });
  }
  pipeline_end(tb, 64);
}

// --------------------------------------------------------------------------- forward output
// stage: q | k | v | H' tiles | raw gate.  Q^ and K^ are gated in place.
// Three CTAs per SM (three independent item pipelines): one stage and 128 TMEM columns each;
// a CTA runs its items one after another and the staged output tile shares its buffer with the
// score tile A.
template <typename Tg> __host__ __device__ constexpr int fo_stage_bytes() { return 4 * TILE + gate_bytes<Tg>(); }
constexpr int FO_NS = 1;

template <typename T, typename Tg>
__global__ void __launch_bounds__(NT + 32, 3) tc_fwd_o_kernel(
    const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
    const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mg,
    const __grid_constant__ CUtensorMap mh, const __grid_constant__ CUtensorMap mo,
    const longlong2* __restrict__ chunk_tab, int MC, int H, float scale, const unsigned char* __restrict__ xflag,
    T* __restrict__ o) {
  constexpr int NS = FO_NS;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  constexpr int STAGE = fo_stage_bytes<Tg>();
  unsigned char* sA = smem + NS * STAGE;
  unsigned char* sOut = sA;  // the previous item's output is staged in the score tile's buffer
  GateSmem& G = *reinterpret_cast<GateSmem*>(sA + TILE);
  __shared__ uint64_t bars[2 + 2 * NS];  // batch 1, batch 2, full[NS], empty[NS]
  __shared__ uint32_t tbase_s;
  __shared__ int s_bad;
  volatile int* bad = &s_bad;
  uint64_t* full = bars + 2;
  uint64_t* empty = bars + 2 + NS;
  const int tid = threadIdx.x;
  prologue<2 + 2 * NS>(&tbase_s, 128, bars, bad);
  const uint32_t tb = tbase_s;
  if (tid == 0)
    for (const CUtensorMap* m : {&mq, &mk, &mv, &mg, &mh, &mo}) prefetch_tensormap(m);
  constexpr uint32_t F = Fmt<T>::v;
  griddep_wait();
  if (tid >= NT) {  // producer warp
    const CUtensorMap* m16[3] = {&mq, &mk, &mv};
    producer_loop<NS>(MC, H, chunk_tab, full, empty, bad, [&](const Item& x, int st) {
      unsigned char* b = smem + st * STAGE;
      unsigned char* sd[1] = {b + 3 * TILE};
      const CUtensorMap* ms[1] = {&mh};
      issue_loads(b, m16, 3, b + 4 * TILE, &mg, gate_bytes<Tg>(), sd, ms, 1, (int)(x.id(H) * D), x.t0, x.head,
                  &full[st]);
    });
  } else {
    const Epi ep;
    const Own me;
    uint32_t ph1 = 0, ph2 = 0;
    const uint32_t tA = tb, tO = tb + 64;
    // epilogue of the item: O from TMEM -> staged tile + TMA store (whole chunks) or direct
    // stores (partial chunks)
    auto finish = [&](const Item& x) {
      wait_mma(&bars[1], ph2, bad);
      float y[1][16];
      ld_acc<1>(ep, {tO}, y);
      const bool poisoned = *bad;
      if (x.len == BT) {
#pragma unroll
        for (int p = 0; p < 8; ++p)
          st2_tile<T>(sOut, ep.row(p), ep.col(p), poisoned ? kNaN : y[0][2 * p], poisoned ? kNaN : y[0][2 * p + 1]);
        fence_proxy_async();
        cbar();
        if (tid == 0) {
          tma_store_3d(&mo, sOut, 0, x.head, (int)x.t0);
          bulk_commit_group();
        }
      } else {
        T* ob = o + (x.t0 * H + x.head) * D;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const int r = ep.row(p);
          if (r < x.len)
            st2_global<T>(ob + (int64_t)r * H * D + ep.col(p), poisoned ? kNaN : y[0][2 * p],
                          poisoned ? kNaN : y[0][2 * p + 1]);
        }
      }
    };
    consumer_loop<NS>(MC, H, chunk_tab, xflag, [&](const Item& x, int st, uint32_t par, bool exact) {
      counted_wait(&full[st], par, bad);
      unsigned char* sQ = smem + st * STAGE;
      unsigned char* sK = sQ + TILE;
      unsigned char* sV = sK + TILE;
      unsigned char* sH = sV + TILE;
      if (x.len < BT) {
        zero_tail<Tg>(sQ, 3, sH + TILE, x.len, me);
        cbar();
      }
      if (exact || *bad) {  // left to the exact kernel (or the CTA gave up: NaN outputs)
        if (*bad) {
          T* ob = o + (x.t0 * H + x.head) * D;
          for (int e = tid; e < x.len * D; e += NT) stf(ob + (int64_t)(e / D) * H * D + (e % D), kNaN);
        }
        cbar();
        if (tid == 0) mbar_arrive(&empty[st]);
        return;
      }
      // the previous item's output store has read A's buffer before the score epilogue below
      // writes it (gate_prep's barriers order it for every thread)
      if (tid == 0) bulk_wait_read_all();
      gate_prep<Tg>(G.E, G.part, sH + TILE);
      gate_qk<T>(sQ, sK, sQ, sK, G.E, me, scale);
      operands_ready();
      if (tid == 0) {
        mma64(tA, sQ, 0, sK, 0, idesc_f16(64, 64, F, 0, 0), false);  // A = Q^ K^^T
        mma64(tO, sQ, 0, sH, 1, idesc_f16(64, 64, F, 0, 1), false);  // O = Q^ H'
        commit(&bars[0]);
      }
      wait_mma(&bars[0], ph1, bad);
      {
        float a[1][16];
        ld_acc<1>(ep, {tA}, a);
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const int r = ep.row(p), c = ep.col(p);
          st2_tile<T>(sA, r, c, c > r ? 0.f : a[0][2 * p], c + 1 > r ? 0.f : a[0][2 * p + 1]);
        }
      }
      operands_ready();
      if (tid == 0) {
        mma64(tO, sA, 0, sV, 1, idesc_f16(64, 64, F, 0, 1), true);  // O += A V
        commit(&bars[1]);
        commit(&empty[st]);  // the stage is free once this batch has read it
      }
      finish(x);
    });
  }
  pipeline_end(tb, 128);
}

// --------------------------------------------------------------------------- backward
// stage: q | k | v | do | H' | dH' tiles | raw gate.  Work tiles: gated Q^, K^ (which become
// the staged dq, dk tiles of the item's epilogue), the score tiles A and dA (A's buffer then
// stages dv), gate factors E (then dgc).  Two CTAs per SM, one stage and 256 TMEM columns each:
// a CTA runs its items one after another (the second MMA batch reuses the first batch's TMEM
// columns once their epilogue has read them), and the two CTAs of an SM overlap each other's
// chains; the producer refills the stage while the CTA writes the item's outputs.
template <typename Tg> __host__ __device__ constexpr int bw_stage_bytes() { return 6 * TILE + gate_bytes<Tg>(); }
constexpr int BW_NS = 1;

struct BwSmem {
  float E[BT * LDG];   // exp(gc - ref); dgc scratch in the epilogue
  float part[NG][D];   // gate-scan group sums
  float dpart[NG][D];  // dg reverse-cumsum group sums
  float hd[NG][D];     // H'.dH' partial sums per key row
  float gp[2][D];      // dH'.S partial sums per key row, per column half
  float dgl[D];        // dgL per key index
};

template <typename T, typename Tg>
__global__ void __launch_bounds__(NT + 32, 2) tc_bwd_kernel(
    const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
    const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mdo,
    const __grid_constant__ CUtensorMap mg, const __grid_constant__ CUtensorMap mh,
    const __grid_constant__ CUtensorMap mdh, const __grid_constant__ CUtensorMap mdq,
    const __grid_constant__ CUtensorMap mdk, const __grid_constant__ CUtensorMap mdv,
    const longlong2* __restrict__ chunk_tab, int MC, int H, float scale, const unsigned char* __restrict__ xflag,
    T* __restrict__ dq, T* __restrict__ dk, T* __restrict__ dv, float* __restrict__ dg) {
  constexpr int NS = BW_NS;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  constexpr int STAGE = bw_stage_bytes<Tg>();
  unsigned char* gQ = smem + NS * STAGE;
  unsigned char* gK = gQ + TILE;
  unsigned char* sA = gK + TILE;
  unsigned char* sdA = sA + TILE;
  unsigned char* sOut = sA;  // dv is staged in A's buffer once the second batch has read A
  BwSmem& W = *reinterpret_cast<BwSmem*>(sdA + TILE);
  __shared__ uint64_t bars[2 + 2 * NS];  // batch 1, batch 2, full[NS], empty[NS]
  __shared__ uint32_t tbase_s;
  __shared__ int s_bad;
  volatile int* bad = &s_bad;
  uint64_t* full = bars + 2;
  uint64_t* empty = bars + 2 + NS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  prologue<2 + 2 * NS>(&tbase_s, 256, bars, bad);
  const uint32_t tb = tbase_s;
  if (tid == 0)
    for (const CUtensorMap* m : {&mq, &mk, &mv, &mdo, &mg, &mh, &mdh, &mdq, &mdk, &mdv}) prefetch_tensormap(m);
  constexpr uint32_t F = Fmt<T>::v;
  // TMEM: batch 1 (A, dA, S) and then batch 2 (dv, dq~, dk~) at columns 0..191
  const uint32_t tA = tb, tdA = tb + 64, tS = tb + 128, tV = tb, tQ = tb + 64, tK = tb + 128;
  griddep_wait();
  if (tid >= NT) {  // producer warp
    const CUtensorMap* m16[4] = {&mq, &mk, &mv, &mdo};
    producer_loop<NS>(MC, H, chunk_tab, full, empty, bad, [&](const Item& x, int st) {
      unsigned char* b = smem + st * STAGE;
      unsigned char* sd[2] = {b + 4 * TILE, b + 5 * TILE};
      const CUtensorMap* ms[2] = {&mh, &mdh};
      issue_loads(b, m16, 4, b + 6 * TILE, &mg, gate_bytes<Tg>(), sd, ms, 2, (int)(x.id(H) * D), x.t0, x.head,
                  &full[st]);
    });
  } else {
    const Epi ep;
    const Own me;
    uint32_t ph1 = 0, ph2 = 0;
    int ci = 0;
    auto poison_rows = [&](const Item& x) {
      const int64_t base = (x.t0 * H + x.head) * D;
      for (int e = tid; e < x.len * D; e += NT) {
        const int64_t off = base + (int64_t)(e / D) * H * D + (e % D);
        stf(dq + off, kNaN);
        stf(dk + off, kNaN);
        stf(dv + off, kNaN);
        dg[off] = kNaN;
      }
    };
    // epilogue of the item: dv, dq, dk and dg (after its second MMA batch)
    auto finish = [&](const Item& x) {
      PHASE(ci - 1, 10);
      wait_mma(&bars[1], ph2, bad);
      PHASE(ci - 1, 11);
      const bool poisoned = *bad;
      const bool whole = x.len == BT;
      const int64_t base = (x.t0 * H + x.head) * D;
      float* E = W.E;
      {
        float z[1][16];
        ld_acc<1>(ep, {tV}, z);
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const int r = ep.row(p), c = ep.col(p);
          const float z0 = poisoned ? kNaN : z[0][2 * p], z1 = poisoned ? kNaN : z[0][2 * p + 1];
          if (whole) st2_tile<T>(sOut, r, c, z0, z1);
          else if (r < x.len) st2_global<T>(dv + base + (int64_t)r * H * D + c, z0, z1);
        }
      }
      {
        float acc[2][16];
        ld_acc<2>(ep, {tQ, tK}, acc);
        // loads of all pairs first, then the stores (see the local-state scaling loop)
        float ee[16], gq[16], gk[16];
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const int r = ep.row(p), c = ep.col(p);
          ee[2 * p] = E[r * LDG + c];
          ee[2 * p + 1] = E[r * LDG + c + 1];
          ld2_tile<T>(gQ, r, c, gq[2 * p], gq[2 * p + 1]);
          ld2_tile<T>(gK, r, c, gk[2 * p], gk[2 * p + 1]);
        }
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const int r = ep.row(p), c = ep.col(p);
          float q0 = acc[0][2 * p] * (scale * ee[2 * p]), q1 = acc[0][2 * p + 1] * (scale * ee[2 * p + 1]);
          float k0 = __fdividef(acc[1][2 * p], ee[2 * p]), k1 = __fdividef(acc[1][2 * p + 1], ee[2 * p + 1]);
          if (poisoned) q0 = q1 = k0 = k1 = kNaN;
          // dgc = q dq - k dk = Q^ dq~ - K^ dk~ (the gated tiles of this item)
          E[r * LDG + c] = gq[2 * p] * acc[0][2 * p] - gk[2 * p] * acc[1][2 * p];
          E[r * LDG + c + 1] = gq[2 * p + 1] * acc[0][2 * p + 1] - gk[2 * p + 1] * acc[1][2 * p + 1];
          if (whole) {  // the gated tiles become the staged outputs
            st2_tile<T>(gQ, r, c, q0, q1);
            st2_tile<T>(gK, r, c, k0, k1);
          } else if (r < x.len) {
            const int64_t off = base + (int64_t)r * H * D + c;
            st2_global<T>(dq + off, q0, q1);
            st2_global<T>(dk + off, k0, k1);
          }
        }
      }
      fence_proxy_async();
      fence_before();
      cbar();
      PHASE(ci - 1, 12);
      if (whole && tid == 0) {
        tma_store_3d(&mdv, sOut, 0, x.head, (int)x.t0);
        tma_store_3d(&mdq, gQ, 0, x.head, (int)x.t0);
        tma_store_3d(&mdk, gK, 0, x.head, (int)x.t0);
        bulk_commit_group();
      }
      // dg = reverse cumulative sum over rows of dgc (+ dgL at every row): NG groups of RG rows
      {
        const int c = tid & 63, qt = tid >> 6;
        float y[RG];
        float run = 0.f;
#pragma unroll
        for (int i = RG - 1; i >= 0; --i) {
          run += E[(RG * qt + i) * LDG + c];
          y[i] = run;
        }
        W.dpart[qt][c] = run;
        cbar();
        float after = W.dgl[c];
#pragma unroll
        for (int j = 0; j < NG; ++j)
          if (j > qt) after += W.dpart[j][c];
        float* dst = dg + base + (int64_t)RG * qt * H * D + c;
#pragma unroll
        for (int i = 0; i < RG; ++i)
          if (RG * qt + i < x.len) dst[(int64_t)i * H * D] = poisoned ? kNaN : y[i] + after;
      }
      PHASE(ci - 1, 13);
    };
    consumer_loop<NS>(MC, H, chunk_tab, xflag, [&](const Item& x, int st, uint32_t par, bool exact) {
      PHASE(ci, 0);
      counted_wait(&full[st], par, bad);
      PHASE(ci, 1);
      unsigned char* rQ = smem + st * STAGE;
      unsigned char* rK = rQ + TILE;
      unsigned char* sV = rK + TILE;
      unsigned char* sDO = sV + TILE;
      unsigned char* sH = sDO + TILE;
      unsigned char* sDH = sH + TILE;
      if (x.len < BT) {
        zero_tail<Tg>(rQ, 4, sDH + TILE, x.len, me);
        cbar();
      }
      if (exact || *bad) {  // left to the exact kernel (or the CTA gave up: NaN outputs)
        if (*bad) poison_rows(x);
        cbar();
        if (tid == 0) mbar_arrive(&empty[st]);
        return;
      }
      // the previous item's output stores have read gQ, gK and A before they are written again
      // (gate_qk and the score epilogue come after gate_prep's barriers)
      if (tid == 0) bulk_wait_read_all();
      gate_prep<Tg>(W.E, W.part, sDH + TILE);
      PHASE(ci, 2);
      gate_qk<T>(rQ, rK, gQ, gK, W.E, me, scale);
      operands_ready();
      PHASE(ci, 3);
      if (tid == 0) {
        mma64(tA, gQ, 0, gK, 0, idesc_f16(64, 64, F, 0, 0), false);    // A  = Q^ K^^T
        mma64(tdA, sDO, 0, sV, 0, idesc_f16(64, 64, F, 0, 0), false);  // dA = do v^T
        mma64(tS, gK, 1, sV, 1, idesc_f16(64, 64, F, 1, 1), false);    // S  = K^^T v
        commit(&bars[0]);
      }
      // H'.dH' per key row (this thread's 16 elements) while the batch runs
      {
        float hd = 0.f;
#pragma unroll
        for (int pc = 0; pc < 2; ++pc) {
          const int off = pc ? me.off1 : me.off0;
          const uint4 uh = *reinterpret_cast<const uint4*>(sH + off);
          const uint4 ud = *reinterpret_cast<const uint4*>(sDH + off);
          const T* xh = reinterpret_cast<const T*>(&uh);
          const T* xd = reinterpret_cast<const T*>(&ud);
#pragma unroll
          for (int i = 0; i < 8; ++i) hd = fmaf(ldf(xh + i), ldf(xd + i), hd);
        }
        W.hd[me.tc >> 3][me.tr] = hd;
      }
      PHASE(ci, 4);
      wait_mma(&bars[0], ph1, bad);
      PHASE(ci, 6);
      {
        float acc[3][16];
        ld_acc<3>(ep, {tA, tdA, tS}, acc);
        float dgl0 = 0.f, dgl1 = 0.f;  // rows r0, r0 + 8
        float dh[16];  // dH' pairs, loaded before the tile stores (see the local-state loop)
#pragma unroll
        for (int p = 0; p < 8; ++p) ld2_tile<T>(sDH, ep.row(p), ep.col(p), dh[2 * p], dh[2 * p + 1]);
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const int r = ep.row(p), c = ep.col(p);
          const bool m0 = c > r, m1 = c + 1 > r;
          st2_tile<T>(sA, r, c, m0 ? 0.f : acc[0][2 * p], m1 ? 0.f : acc[0][2 * p + 1]);
          st2_tile<T>(sdA, r, c, m0 ? 0.f : acc[1][2 * p], m1 ? 0.f : acc[1][2 * p + 1]);
          // row r of S is key index r: dH'[r, :] . S[r, :]
          const float t = fmaf(dh[2 * p], acc[2][2 * p], dh[2 * p + 1] * acc[2][2 * p + 1]);
          if (p & 1) dgl1 += t; else dgl0 += t;
        }
        dgl0 += __shfl_xor_sync(0xffffffffu, dgl0, 1);
        dgl0 += __shfl_xor_sync(0xffffffffu, dgl0, 2);
        dgl1 += __shfl_xor_sync(0xffffffffu, dgl1, 1);
        dgl1 += __shfl_xor_sync(0xffffffffu, dgl1, 2);
        if ((lane & 3) == 0) {
          W.gp[warp >> 2][ep.r0] = dgl0;
          W.gp[warp >> 2][ep.r0 + 8] = dgl1;
        }
      }
      PHASE(ci, 7);
      // every thread's TMEM reads of batch 1 are complete before batch 2 overwrites its columns
      operands_ready();
      if (tid == 0) {
        mma64(tV, sA, 1, sDO, 1, idesc_f16(64, 64, F, 1, 1), false);  // dv  = A^T do
        mma64(tV, gK, 0, sDH, 1, idesc_f16(64, 64, F, 0, 1), true);   //     + K^ dH'
        mma64(tQ, sDO, 0, sH, 0, idesc_f16(64, 64, F, 0, 0), false);  // dq~ = do H'^T
        mma64(tQ, sdA, 0, gK, 1, idesc_f16(64, 64, F, 0, 1), true);   //     + dA K^
        mma64(tK, sV, 0, sDH, 0, idesc_f16(64, 64, F, 0, 0), false);  // dk~ = v dH'^T
        mma64(tK, sdA, 1, gQ, 1, idesc_f16(64, 64, F, 1, 1), true);   //     + dA^T Q^
        commit(&bars[1]);
        commit(&empty[st]);  // the stage is free once this batch has read it
      }
      PHASE(ci, 8);
      // dgL per key index: H'.dH' + dH'.(K^^T v)
      if (tid < D) {
        float s2 = W.gp[0][tid] + W.gp[1][tid];
#pragma unroll
        for (int j = 0; j < NG; ++j) s2 += W.hd[j][tid];
        W.dgl[tid] = s2;
      }
      PHASE(ci, 9);
      ++ci;
      finish(x);
    });
  }
  pipeline_end(tb, 256);
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

// Grid: as many CTAs as fit on the device at once (shared memory, registers and TMEM columns
// permitting), capped by the number of items.
template <typename K_>
int persistent_grid(K_ kern, size_t smem, int tmem_cols, int64_t items, unsigned& grid, int nthreads = NT) {
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
  const int by_regs = 65536 / (((fa.numRegs + 7) / 8) * 8 * nthreads);
  int per_sm = by_smem < by_regs ? by_smem : by_regs;
  if (per_sm > 2048 / nthreads) per_sm = 2048 / nthreads;
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

CUtensorMapDataType tmap_dtype(int dtype) {
  return dtype == SSLA_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
         : dtype == SSLA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// 3-D view (D = 64, H, T) of a [T, H, 64] token array, box 64 x 1 x 64: 16-bit operands with
// the 128-byte swizzle, the gate (any dtype) unswizzled.
int make_map(CUtensorMap* m, const void* base, int dtype, int64_t T, int64_t H, bool swizzle) {
  const int eb = dtype == SSLA_F32 ? 4 : 2;
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T};
  const cuuint64_t strides[2] = {(cuuint64_t)D * eb, (cuuint64_t)H * D * eb};
  const cuuint32_t box[3] = {(cuuint32_t)D, 1u, (cuuint32_t)BT};
  return encode(m, tmap_dtype(dtype), 3, base, dims, strides, box,
                swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
}

// 2-D view [rows, 64] of 16-bit chunk states (64 rows per (chunk, head)), box 64 x 64,
// 128-byte swizzle (the layout of the token tiles).
int make_state_map(CUtensorMap* m, const void* base, int dtype, int64_t rows) {
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  const cuuint32_t box[2] = {(cuuint32_t)D, (cuuint32_t)D};
  return encode(m, tmap_dtype(dtype), 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// 2-D view [rows, 64] of fp32 per-item tiles (64 rows per (chunk, head)), box of 32 columns x
// 64 rows with the 128-byte swizzle (a tile is stored as two column halves).
int make_f32_rows_map(CUtensorMap* m, const float* base, int64_t rows) {
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

int tc_aligned(const void* const* ptrs, int n) {
  for (int i = 0; i < n; ++i)
    if (reinterpret_cast<uintptr_t>(ptrs[i]) % 16) return 0;
  return 1;
}

int tc_local_state(int dtype, int dtype_g, int mode, const void* a_src, const void* b_src, const void* g,
                   const longlong2* chunk_tab, int64_t T, int64_t MC, int64_t H, float scale, float* dS,
                   float* decay, float* escale, unsigned char* xflag, int* xlist, cudaStream_t s) {
  if (MC * H == 0) return SSLA_OK;
  if (int rc = check_sizes(T, MC, H)) return rc;
  CUtensorMap ma, mb, mg, mds;
  int rc;
  if ((rc = make_map(&ma, a_src, dtype, T, H, true)) || (rc = make_map(&mb, b_src, dtype, T, H, true)) ||
      (rc = make_map(&mg, g, dtype_g, T, H, false)) || (rc = make_f32_rows_map(&mds, dS, MC * H * D)))
    return rc;
  return SSLA_DISPATCH_TC(dtype, dtype_g, T_, Tg, [&] {
    auto kern = tc_local_state_kernel<T_, Tg>;
    const size_t smem = LS_NS * ls_stage_bytes<Tg>() + 2 * TILE + sizeof(LsSmem) + kAlignSlack;
    unsigned grid = 0;
    int rc2 = persistent_grid(kern, smem, 64, MC * H, grid, NT + 32);
    if (rc2) return rc2;
    launch_pdl(kern, dim3(grid), dim3(NT + 32), smem, s, ma, mb, mg, mds, mode, chunk_tab, (int)MC, (int)H, scale,
               dS, decay, escale, xflag, xlist);
    SSLA_CHECK_LAUNCH("chunk_gla tc_local_state");
    return SSLA_OK;
  });
}

int tc_fwd_o(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
             const longlong2* chunk_tab, int64_t T, int64_t MC, int64_t H, float scale, const void* h16,
             const unsigned char* xflag, void* o, cudaStream_t s) {
  if (MC * H == 0) return SSLA_OK;
  if (int rc = check_sizes(T, MC, H)) return rc;
  CUtensorMap mq, mk, mv, mg, mh, mo;
  int rc;
  if ((rc = make_map(&mq, q, dtype, T, H, true)) || (rc = make_map(&mk, k, dtype, T, H, true)) ||
      (rc = make_map(&mv, v, dtype, T, H, true)) || (rc = make_map(&mg, g, dtype_g, T, H, false)) ||
      (rc = make_state_map(&mh, h16, dtype, MC * H * D)) || (rc = make_map(&mo, o, dtype, T, H, true)))
    return rc;
  return SSLA_DISPATCH_TC(dtype, dtype_g, T_, Tg, [&] {
    auto kern = tc_fwd_o_kernel<T_, Tg>;
    const size_t smem = FO_NS * fo_stage_bytes<Tg>() + TILE + sizeof(GateSmem) + kAlignSlack;
    unsigned grid = 0;
    int rc2 = persistent_grid(kern, smem, 128, MC * H, grid, NT + 32);
    if (rc2) return rc2;
    launch_pdl(kern, dim3(grid), dim3(NT + 32), smem, s, mq, mk, mv, mg, mh, mo, chunk_tab, (int)MC, (int)H, scale,
               xflag, (T_*)o);
    SSLA_CHECK_LAUNCH("chunk_gla tc_fwd_o");
    return SSLA_OK;
  });
}

int tc_bwd(int dtype, int dtype_g, const void* q, const void* k, const void* v, const void* g,
           const longlong2* chunk_tab, int64_t T, int64_t MC, int64_t H, float scale, const void* h16,
           const void* dh16, const unsigned char* xflag, const void* dout, void* dq, void* dk, void* dv,
           float* dg, cudaStream_t s) {
  if (MC * H == 0) return SSLA_OK;
  if (int rc = check_sizes(T, MC, H)) return rc;
  CUtensorMap mq, mk, mv, mdo, mg, mh, mdh, mdq, mdk, mdv;
  int rc;
  if ((rc = make_map(&mq, q, dtype, T, H, true)) || (rc = make_map(&mk, k, dtype, T, H, true)) ||
      (rc = make_map(&mv, v, dtype, T, H, true)) || (rc = make_map(&mdo, dout, dtype, T, H, true)) ||
      (rc = make_map(&mg, g, dtype_g, T, H, false)) || (rc = make_state_map(&mh, h16, dtype, MC * H * D)) ||
      (rc = make_state_map(&mdh, dh16, dtype, MC * H * D)) || (rc = make_map(&mdq, dq, dtype, T, H, true)) ||
      (rc = make_map(&mdk, dk, dtype, T, H, true)) || (rc = make_map(&mdv, dv, dtype, T, H, true)))
    return rc;
  return SSLA_DISPATCH_TC(dtype, dtype_g, T_, Tg, [&] {
    auto kern = tc_bwd_kernel<T_, Tg>;
    const size_t smem = BW_NS * bw_stage_bytes<Tg>() + 4 * TILE + sizeof(BwSmem) + kAlignSlack;
    unsigned grid = 0;
    int rc2 = persistent_grid(kern, smem, 256, MC * H, grid, NT + 32);
    if (rc2) return rc2;
    launch_pdl(kern, dim3(grid), dim3(NT + 32), smem, s, mq, mk, mv, mdo, mg, mh, mdh, mdq, mdk, mdv, chunk_tab,
               (int)MC, (int)H, scale, xflag, (T_*)dq, (T_*)dk, (T_*)dv, dg);
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

#ifdef SSLA_PHASE_PROF
// Development build only: copy (and clear) the phase-timing table; `out` holds
// kPhaseCtas * kPhaseItems * kPhasePts int64.
extern "C" int ssla_chunk_gla_phase_dump(long long* out) {
  using namespace ssla::chunk;
  if (cudaMemcpyFromSymbol(out, g_phase, sizeof(g_phase)) != cudaSuccess) return SSLA_ERR_CUDA;
  static long long zero[kPhaseCtas * kPhaseItems * kPhasePts];
  return cudaMemcpyToSymbol(g_phase, zero, sizeof(g_phase)) == cudaSuccess ? SSLA_OK : SSLA_ERR_CUDA;
}
#endif
