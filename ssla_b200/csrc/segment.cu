// Deterministic segment reductions, row gathers and index_add for sparse pooling and the
// sparse-token routing (layers/sparse_pooling.py:14-51 with torch_scatter.scatter_max /
// scatter_mean; utils/async_utils.py:243-264 index_add_).
//
// The reference reduces with torch_scatter / index_add_, whose GPU kernels use atomics and
// so sum in an unspecified order.  Here every reduction walks the rows of a segment in
// ascending row order with an fp32 accumulator, which reproduces the CPU PyTorch /
// torch_scatter result bit for bit for fp32 data:
//   * sorted indices (the pooling case: unique_consecutive inverse ids are non-decreasing):
//     segment boundaries come from one pass over the index, no sort at all;
//   * arbitrary indices: a counting sort builds a CSR (count -> exclusive scan -> scatter),
//     and each segment's row list is then put in ascending order by a warp-level rank sort,
//     so the result never depends on atomic arrival order.
// Rows are moved 16 B (fp32) or 8 B (16-bit) per thread; consecutive threads cover
// consecutive channel vectors of the same row.
#include <float.h>

#include "common.cuh"
#include "vec.cuh"

namespace ssla {
namespace {

inline size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

// off[s] = first row r with index[r] >= s, for s in [0, S]; index non-decreasing.
__global__ void offsets_sorted_kernel(const int64_t* __restrict__ index, int64_t R, int64_t S,
                                      int64_t* __restrict__ off) {
  griddep_launch_dependents();
  griddep_wait();
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r > R) return;
  int64_t prev = r == 0 ? -1 : index[r - 1];
  int64_t cur = r == R ? S : index[r];
  if (prev < -1) prev = -1;
  if (cur > S) cur = S;
  for (int64_t s = prev + 1; s <= cur; ++s) off[s] = r;
}

__global__ void count_kernel(const int64_t* __restrict__ index, int64_t R, int64_t S,
                             int* __restrict__ counts) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= R) return;
  const int64_t s = index[r];
  if (s >= 0 && s < S) atomicAdd(&counts[s], 1);
}

// Block-wise exclusive scan of int counts into int64 offsets (+ per-block totals).
__global__ void __launch_bounds__(1024) scan_blocks_kernel(const int* __restrict__ counts,
                                                           int64_t S, int64_t* __restrict__ off,
                                                           int64_t* __restrict__ block_sums) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ int64_t ws[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t i = (int64_t)blockIdx.x * 1024 + tid;
  const int64_t x = i < S ? counts[i] : 0;
  int64_t incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) ws[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int64_t w = ws[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    ws[lane] = w;
  }
  __syncthreads();
  const int64_t before = warp > 0 ? ws[warp - 1] : 0;
  if (i < S) off[i] = before + incl - x;
  if (tid == 1023) block_sums[blockIdx.x] = before + incl;
}

// Exclusive scan of the block totals in place, by one CTA of 1024 threads walking them 1024 at a
// time with a running carry, then off[S] = number of rows (for nb > 1024; fewer blocks use
// add_block_prefix_kernel).
__global__ void __launch_bounds__(1024) scan_totals_kernel(int64_t* __restrict__ block_sums, int64_t nb,
                                                           int64_t S, int64_t* __restrict__ off) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ int64_t ws[32];
  __shared__ int64_t carry_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int64_t carry = 0;
  for (int64_t base = 0; base < nb; base += 1024) {
    const int64_t i = base + tid;
    const int64_t x = i < nb ? block_sums[i] : 0;
    int64_t incl = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) ws[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int64_t w = ws[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      ws[lane] = w;
    }
    __syncthreads();
    const int64_t before = carry + (warp > 0 ? ws[warp - 1] : 0);
    if (i < nb) block_sums[i] = before + incl - x;
    if (tid == 1023) carry_s = before + incl;
    __syncthreads();
    carry = carry_s;
  }
  if (tid == 0) off[S] = carry;
}

__global__ void add_block_base_kernel(int64_t* __restrict__ off, int64_t S,
                                      const int64_t* __restrict__ block_sums,
                                      int* __restrict__ counts) {
  griddep_launch_dependents();
  griddep_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= S) return;
  off[i] += block_sums[i / 1024];
  counts[i] = 0;  // reused as the fill cursor
}

// Adds to each 1024-entry block of `off` the sum of all earlier blocks' totals (each block
// reduces the prefix of block_sums itself, so no sequential pass is needed), resets `counts`
// to zero for use as the fill cursor and writes off[S] = number of rows.  For nb <= 1024.
__global__ void __launch_bounds__(1024) add_block_prefix_kernel(int64_t* __restrict__ off, int64_t S,
                                                                const int64_t* __restrict__ block_sums,
                                                                int64_t nb, int* __restrict__ counts) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ int64_t red[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int64_t part = 0;
  for (int64_t j = tid; j < blockIdx.x; j += 1024) part += block_sums[j];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if (lane == 0) red[warp] = part;
  __syncthreads();
  int64_t base = 0;
#pragma unroll
  for (int w = 0; w < 32; ++w) base += red[w];
  const int64_t i = (int64_t)blockIdx.x * 1024 + tid;
  if (i < S) {
    off[i] += base;
    counts[i] = 0;
  }
  if (blockIdx.x == nb - 1 && tid == 0) off[S] = base + block_sums[nb - 1];
}

__global__ void fill_kernel(const int64_t* __restrict__ index, int64_t R, int64_t S,
                            const int64_t* __restrict__ off, int* __restrict__ cursor,
                            int64_t* __restrict__ tmp) {
  griddep_launch_dependents();
  griddep_wait();
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= R) return;
  const int64_t s = index[r];
  if (s < 0 || s >= S) return;
  const int64_t pos = off[s] + atomicAdd(&cursor[s], 1);
  tmp[pos] = r;
}

// One warp per segment: rows[off[s] + rank(x)] = x, rank = #{y in segment : y < x}.
__global__ void rank_sort_kernel(const int64_t* __restrict__ off, int64_t S,
                                 const int64_t* __restrict__ tmp, int64_t* __restrict__ rows) {
  griddep_launch_dependents();
  griddep_wait();
  const int64_t s = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (s >= S) return;
  const int64_t b = off[s], e = off[s + 1], n = e - b;
  if (n <= 32) {
    const int64_t x = lane < n ? tmp[b + lane] : INT64_MAX;
    int rank = 0;
    for (int j = 0; j < n; ++j) {
      const int64_t y = __shfl_sync(0xffffffffu, x, j);
      rank += (y < x);
    }
    if (lane < n) rows[b + rank] = x;
  } else {
    for (int64_t i = lane; i < n; i += 32) {
      const int64_t x = tmp[b + i];
      int64_t rank = 0;
      for (int64_t j = 0; j < n; ++j) rank += (tmp[b + j] < x);
      rows[b + rank] = x;
    }
  }
}

template <typename T> __device__ __forceinline__ float lowest_of();
template <> __device__ __forceinline__ float lowest_of<float>() { return -FLT_MAX; }
template <> __device__ __forceinline__ float lowest_of<__nv_bfloat16>() { return -3.38953139e38f; }
template <> __device__ __forceinline__ float lowest_of<__half>() { return -65504.f; }

// Block = (CV channel vectors) x (segments): threadIdx.x picks VEC channels, threadIdx.y the
// segment, so a warp reads whole rows of consecutive segments and no index division is needed.
// Rows are visited in ascending order; loads are issued 8 rows at a time (predicated), then
// combined in row order.  op: 0 sum, 1 mean, 2 max.
template <typename T, int VEC, int OP>
__global__ void __launch_bounds__(256) reduce_kernel(const T* __restrict__ src,
                                                     const int64_t* __restrict__ off,
                                                     const int64_t* __restrict__ rows, int64_t R,
                                                     int64_t S, int64_t C, T* __restrict__ out,
                                                     int64_t* __restrict__ arg) {
  griddep_launch_dependents();
  griddep_wait();
  constexpr int U = 4;
  const int64_t s = (int64_t)blockIdx.x * blockDim.y + threadIdx.y;
  if (s >= S) return;
  const int64_t c = (int64_t)threadIdx.x * VEC;
  const int64_t b = off[s], e = off[s + 1];
  float acc[VEC];
  int64_t am[VEC];
  const float lo = lowest_of<T>();
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    acc[i] = OP == 2 ? lo : 0.f;
    am[i] = R;
  }
  for (int64_t p = b; p < e; p += U) {
    float x[U][VEC];
    int64_t rr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (p + u < e) {
        rr[u] = rows ? rows[p + u] : p + u;
        Vec<T, VEC>::load(src + rr[u] * C + c, x[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (p + u < e) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          if (OP == 2) {
            if (x[u][i] > acc[i]) { acc[i] = x[u][i]; am[i] = rr[u]; }
          } else {
            acc[i] = __fadd_rn(acc[i], x[u][i]);
          }
        }
      }
    }
  }
  if (OP == 1) {
    const float cnt = (float)(e - b > 0 ? e - b : 1);
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = __fdiv_rn(acc[i], cnt);
  }
  if (OP == 2) {
#pragma unroll
    for (int i = 0; i < VEC; ++i)
      if (acc[i] == lo) acc[i] = 0.f;
    if (arg) {
#pragma unroll
      for (int i = 0; i < VEC; ++i) arg[s * C + c + i] = am[i];
    }
  }
  Vec<T, VEC>::store(out + s * C + c, acc);
}

// Sorted segments (rows == nullptr): a block owns 256 / CV consecutive segments, whose rows
// are one contiguous byte range.  The range is staged into shared memory with coalesced 16-byte
// loads (all issued before any is consumed), in windows of at most `win_rows` rows; each thread
// then reduces its (segment, channel vector) from shared memory in ascending row order.
template <typename T, int VEC, int OP>
__global__ void __launch_bounds__(256) reduce_sorted_tiled_kernel(const T* __restrict__ src,
                                                                  const int64_t* __restrict__ off,
                                                                  int64_t R, int64_t S, int64_t C,
                                                                  int win_rows, T* __restrict__ out,
                                                                  int64_t* __restrict__ arg) {
  griddep_launch_dependents();
  griddep_wait();
  extern __shared__ uint4 stage4[];
  const T* stage = reinterpret_cast<const T*>(stage4);
  const int CV = (int)(C / VEC);
  const int segs = 256 / CV;
  const int64_t s0 = (int64_t)blockIdx.x * segs;
  const int tid = threadIdx.x;
  const int js = tid / CV, jv = tid - js * CV;
  const int64_t s = s0 + js;
  const bool mine = js < segs && s < S;
  const int64_t sl = (s0 + segs < S) ? s0 + segs : S;
  const int64_t r0 = off[s0], r1 = off[sl];
  int64_t b = 0, e = 0;
  if (mine) { b = off[s]; e = off[s + 1]; }
  const int64_t c = (int64_t)jv * VEC;
  float acc[VEC];
  int64_t am[VEC];
  const float lo = lowest_of<T>();
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    acc[i] = OP == 2 ? lo : 0.f;
    am[i] = R;
  }
  const int64_t row16 = C * (int64_t)sizeof(T) / 16;  // 16-byte words per row
  for (int64_t w0 = r0; w0 < r1; w0 += win_rows) {
    const int64_t w1 = (w0 + win_rows < r1) ? w0 + win_rows : r1;
    const int64_t n16 = (w1 - w0) * row16;
    const uint4* g4 = reinterpret_cast<const uint4*>(src + w0 * C);
    __syncthreads();
    for (int64_t i = tid; i < n16; i += 256) stage4[i] = __ldg(g4 + i);
    __syncthreads();
    const int64_t pb = b > w0 ? b : w0, pe = e < w1 ? e : w1;
    for (int64_t p = pb; p < pe; ++p) {
      float x[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) x[i] = ldf(stage + (p - w0) * C + c + i);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        if (OP == 2) {
          if (x[i] > acc[i]) { acc[i] = x[i]; am[i] = p; }
        } else {
          acc[i] = __fadd_rn(acc[i], x[i]);
        }
      }
    }
  }
  if (!mine) return;
  if (OP == 1) {
    const float cnt = (float)(e - b > 0 ? e - b : 1);
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = __fdiv_rn(acc[i], cnt);
  }
  if (OP == 2) {
#pragma unroll
    for (int i = 0; i < VEC; ++i)
      if (acc[i] == lo) acc[i] = 0.f;
    if (arg) {
#pragma unroll
      for (int i = 0; i < VEC; ++i) arg[s * C + c + i] = am[i];
    }
  }
  Vec<T, VEC>::store(out + s * C + c, acc);
}

template <typename T, int VEC>
__global__ void __launch_bounds__(256) gather_kernel(const T* __restrict__ src,
                                                     const int64_t* __restrict__ index, int64_t R,
                                                     int64_t C, T* __restrict__ out) {
  griddep_launch_dependents();
  griddep_wait();
  const int64_t CV = C / VEC;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= R * CV) return;
  const int64_t r = idx / CV;
  const int64_t c = (idx - r * CV) * VEC;
  float x[VEC];
  Vec<T, VEC>::load(src + index[r] * C + c, x);
  Vec<T, VEC>::store(out + r * C + c, x);
}

// 16 bytes of T as floats (raw vector already loaded).
template <typename T> struct Row16 {
  static constexpr int V = 8;
  static __device__ __forceinline__ void unpack(uint4 r, float* x) { Vec8x16<T>::unpack(r, x); }
};
template <> struct Row16<float> {
  static constexpr int V = 4;
  static __device__ __forceinline__ void unpack(uint4 r, float* x) {
    x[0] = __uint_as_float(r.x); x[1] = __uint_as_float(r.y);
    x[2] = __uint_as_float(r.z); x[3] = __uint_as_float(r.w);
  }
};

// Scatter max + mean of every segment and the gather of the max back to its rows, in one
// pass over the rows (the sparse pooling of layers/sparse_pooling.py:33 followed by the
// inverse lookup pooled[index]); with MODE kPoolSum, the plain ascending-order sum
// (the index_add_ gather-back of utils/async_utils.py:243-264).  A group of GP lanes (GP the
// power of two >= G) owns one segment; lane gl < G holds 16 bytes (V channels) of a row, so
// G * V == C.  The segment's row ids arrive unsorted from the counting-sort fill; up to
// kSlots * GP of them are ranked in registers (each lane keeps kSlots ids, every id is
// compared with every other through shuffles) and handed to the lanes in ascending order,
// longer segments by a rank count over the list written to `sorted`.  Rows are loaded kWin at
// a time (all loads issued before any is combined) and reduced in ascending row order: max
// keeps the first maximal row (strict >), the sum is fp32 with round-to-nearest adds, mean =
// sum / max(count, 1), empty segments give 0 (arg R).  (A persistent variant walking segments
// with a grid stride and prefetching the next segment's offsets and row ids measured slower:
// 51 vs 42 us on the config-4 k=2 pooling.)
constexpr int kPoolMaxMean = 0, kPoolArg = 1, kPoolSum = 2;

template <typename T, int G, int MODE>
__global__ void __launch_bounds__(256, MODE == kPoolArg ? 2 : 4) pool_fused_kernel(
    const T* __restrict__ src, const int64_t* __restrict__ off, const int64_t* __restrict__ tmp,
    int64_t* __restrict__ sorted, int R, int S, T* __restrict__ out_max, int64_t* __restrict__ arg,
    T* __restrict__ out_mean, T* __restrict__ back, bool presorted) {
  griddep_launch_dependents();
  griddep_wait();
  // presorted: the ids of each segment are already ascending in `tmp` (a sorted CSR), or, with
  // tmp == nullptr, the segment is the row range itself (sorted index: ids b .. b+n-1).
  // Row ids, offsets and counts fit in 32 bits (the launcher checks R < 2^31); the row width
  // C = G * V is a compile-time constant, so no 64-bit index arithmetic is issued per row.
  constexpr int V = Row16<T>::V;
  constexpr int C = G * V;
  constexpr int GP = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : G <= 8 ? 8 : G <= 16 ? 16 : 32;
  constexpr int kSlots = GP >= 8 ? 2 : 4;
  constexpr int kWin = 4;
  constexpr int kNone = 0x7fffffff;
  constexpr bool ARG = MODE == kPoolArg, SUM = MODE == kPoolSum;
  const int lane = threadIdx.x & 31, gl = lane & (GP - 1);
  const unsigned gmask = GP == 32 ? 0xffffffffu : (((1u << GP) - 1u) << (lane & ~(GP - 1)));
  const int s = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / GP);
  if (s >= S) return;  // the whole group leaves together
  const int b = (int)off[s], n = (int)off[s + 1] - b;
  const bool data = gl < G;  // lanes G..GP-1 only take part in the shuffles
  const int c = (data ? gl : 0) * V;
  const float lo = lowest_of<T>();
  float mx[V], sm[V];
  int am[ARG ? V : 1];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    mx[i] = lo;
    sm[i] = 0.f;
    if (ARG) am[i] = R;
  }
  const bool small = n <= kSlots * GP;
  int mine[kSlots];  // small: slot k of lane gl holds the (k * GP + gl)-th smallest row id
#pragma unroll
  for (int k = 0; k < kSlots; ++k) mine[k] = kNone;
  auto id_at = [&](int i) -> int { return tmp ? (int)tmp[b + i] : b + i; };
  if (small && presorted) {
#pragma unroll
    for (int k = 0; k < kSlots; ++k) mine[k] = k * GP + gl < n ? id_at(k * GP + gl) : kNone;
  } else if (small) {
    int id[kSlots], rank[kSlots];
#pragma unroll
    for (int k = 0; k < kSlots; ++k) {
      id[k] = k * GP + gl < n ? (int)tmp[b + k * GP + gl] : kNone;
      rank[k] = 0;
    }
#pragma unroll
    for (int kk = 0; kk < kSlots; ++kk) {
      if (kk * GP < n) {  // uniform over the group
#pragma unroll
        for (int j = 0; j < GP; ++j) {
          const int y = __shfl_sync(gmask, id[kk], j, GP);
#pragma unroll
          for (int k = 0; k < kSlots; ++k) rank[k] += y < id[k];
        }
      }
    }
#pragma unroll
    for (int kk = 0; kk < kSlots; ++kk) {
      if (kk * GP < n) {
#pragma unroll
        for (int j = 0; j < GP; ++j) {
          const int rj = __shfl_sync(gmask, rank[kk], j, GP);
          const int yj = __shfl_sync(gmask, id[kk], j, GP);
#pragma unroll
          for (int k = 0; k < kSlots; ++k)
            if (rj == k * GP + gl) mine[k] = yj;
        }
      }
    }
  } else if (!presorted) {
    for (int i = gl; i < n; i += GP) {
      const int x = (int)tmp[b + i];
      int rank = 0;
      for (int j = 0; j < n; ++j) rank += (int)tmp[b + j] < x;
      sorted[b + rank] = x;
    }
    __syncwarp(gmask);
  }
  // the rows of slot window p0 (GP rows, ascending) as one lane value each
  auto window_ids = [&](int p0, int k) -> int {
    if (small) return mine[k];
    if (p0 + gl >= n) return kNone;
    return presorted ? id_at(p0 + gl) : (int)sorted[b + p0 + gl];
  };
#pragma unroll 1
  for (int k = 0, p0 = 0; p0 < n; ++k, p0 += GP) {
    int w = kNone;
#pragma unroll
    for (int kk = 0; kk < kSlots; ++kk)
      if (kk == (small ? k : 0)) w = window_ids(p0, kk);
    const int m = n - p0 < GP ? n - p0 : GP;
    for (int w0 = 0; w0 < m; w0 += kWin) {
      int rid[kWin];
      uint4 raw[kWin];
#pragma unroll
      for (int u = 0; u < kWin; ++u) {
        rid[u] = __shfl_sync(gmask, w, (w0 + u) & (GP - 1), GP);
        if (data && w0 + u < m) raw[u] = __ldg(reinterpret_cast<const uint4*>(src + (size_t)rid[u] * C + c));
      }
#pragma unroll
      for (int u = 0; u < kWin; ++u) {
        if (data && w0 + u < m) {
          float x[V];
          Row16<T>::unpack(raw[u], x);
#pragma unroll
          for (int i = 0; i < V; ++i) {
            if (!SUM && x[i] > mx[i]) {
              mx[i] = x[i];
              if (ARG) am[i] = rid[u];
            }
            sm[i] = __fadd_rn(sm[i], x[i]);
          }
        }
      }
    }
  }
  if (!data) return;
  const size_t o = (size_t)s * C + c;
  if (SUM) {
    Vec<T, V>::store(out_mean + o, sm);
    return;
  }
#pragma unroll
  for (int i = 0; i < V; ++i)
    if (mx[i] == lo) mx[i] = 0.f;
  if (out_max) Vec<T, V>::store(out_max + o, mx);
  if (ARG) {
#pragma unroll
    for (int i = 0; i < V; ++i) arg[o + i] = am[i];
  }
  if (out_mean) {
    const float cnt = (float)(n > 0 ? n : 1);
#pragma unroll
    for (int i = 0; i < V; ++i) sm[i] = __fdiv_rn(sm[i], cnt);
    Vec<T, V>::store(out_mean + o, sm);
  }
  if (back) {
    // row ids straight from the list (in any order: each row's store is independent)
    for (int u = 0; u < n; ++u) {
      const int r = id_at(u);
      Vec<T, V>::store(back + (size_t)r * C + c, mx);
    }
  }
}

template <typename T>
int run_reduce(const void* src, const int64_t* off, const int64_t* rows, int64_t R, int64_t S,
               int64_t C, int op, void* out, int64_t* arg, cudaStream_t s) {
  if (S == 0 || C == 0) return SSLA_OK;
  const bool v4 = C % 4 == 0 && aligned_to(src, 4 * sizeof(T)) && aligned_to(out, 4 * sizeof(T));
  const int64_t CV = v4 ? C / 4 : C;
  if (CV > 256) {
    set_error("ssla_segment_reduce: C=%lld too wide (at most %d)", (long long)C, v4 ? 1024 : 256);
    return SSLA_ERR_UNSUPPORTED;
  }
  const int segs = (int)(256 / CV);
  const unsigned grid = (unsigned)ceil_div(S, segs);
  const bool tiled = rows == nullptr && (C * (int64_t)sizeof(T)) % 16 == 0 && aligned_to(src, 16);
  if (tiled) {
    constexpr int kStageBytes = 48 * 1024;
    const int win = (int)(kStageBytes / (C * (int64_t)sizeof(T)));
    if (win < 1) {
      set_error("ssla_segment_reduce: row of %lld bytes exceeds the staging buffer", (long long)(C * sizeof(T)));
      return SSLA_ERR_UNSUPPORTED;
    }
    const size_t smem = (size_t)win * C * sizeof(T);
#define SSLA_RED(VEC, OP)                                                                   \
  launch_pdl(reduce_sorted_tiled_kernel<T, VEC, OP>, dim3(grid), dim3(256), smem, s, (const T*)src, off, R, S, C, win, \
                                                                 (T*)out, arg)
    if (v4) {
      if (op == 0) SSLA_RED(4, 0); else if (op == 1) SSLA_RED(4, 1); else SSLA_RED(4, 2);
    } else {
      if (op == 0) SSLA_RED(1, 0); else if (op == 1) SSLA_RED(1, 1); else SSLA_RED(1, 2);
    }
#undef SSLA_RED
  } else {
    const dim3 block((unsigned)CV, (unsigned)segs);
#define SSLA_RED(VEC, OP) \
  launch_pdl(reduce_kernel<T, VEC, OP>, dim3(grid), block, 0, s, (const T*)src, off, rows, R, S, C, (T*)out, arg)
    if (v4) {
      if (op == 0) SSLA_RED(4, 0); else if (op == 1) SSLA_RED(4, 1); else SSLA_RED(4, 2);
    } else {
      if (op == 0) SSLA_RED(1, 0); else if (op == 1) SSLA_RED(1, 1); else SSLA_RED(1, 2);
    }
#undef SSLA_RED
  }
  SSLA_CHECK_LAUNCH("ssla_segment_reduce");
  return SSLA_OK;
}

int build_csr(const int64_t* index, int64_t R, int64_t S, int64_t* off, int64_t* rows, void* ws,
              cudaStream_t s) {
  char* p = (char*)ws;
  int* counts = (int*)p;
  p += a256(4 * (size_t)S);
  const int64_t nb = (S + 1023) / 1024;
  int64_t* block_sums = (int64_t*)p;
  p += a256(8 * (size_t)(nb + 1));
  int64_t* tmp = (int64_t*)p;
  if (S > 0) {
    if (cudaMemsetAsync(counts, 0, 4 * (size_t)S, s) != cudaSuccess) {
      set_error("ssla_segment_csr: memset failed");
      return SSLA_ERR_CUDA;
    }
    if (R > 0) count_kernel<<<ceil_div(R, 256), 256, 0, s>>>(index, R, S, counts);
    launch_pdl(scan_blocks_kernel, dim3((unsigned)nb), dim3(1024), 0, s, (const int*)counts, S, off, block_sums);
  }
  if (S > 0 && nb <= 1024) {
    launch_pdl(add_block_prefix_kernel, dim3((unsigned)nb), dim3(1024), 0, s, off, S, (const int64_t*)block_sums, nb, counts);
  } else {
    launch_pdl(scan_totals_kernel, dim3(1), dim3(1024), 0, s, block_sums, nb, S, off);
    if (S > 0)
      launch_pdl(add_block_base_kernel, dim3(ceil_div(S, 256)), dim3(256), 0, s, off, S, (const int64_t*)block_sums,
                 counts);
  }
  if (S > 0) {
    if (R > 0) {
      launch_pdl(fill_kernel, dim3(ceil_div(R, 256)), dim3(256), 0, s, index, R, S, (const int64_t*)off, counts, tmp);
      launch_pdl(rank_sort_kernel, dim3(ceil_div(S * 32, 256)), dim3(256), 0, s, (const int64_t*)off, S, (const int64_t*)tmp, rows);
    }
  }
  SSLA_CHECK_LAUNCH("ssla_segment_csr");
  return SSLA_OK;
}

size_t csr_ws_bytes(int64_t R, int64_t S) {
  const int64_t nb = (S + 1023) / 1024;
  return a256(4 * (size_t)S) + a256(8 * (size_t)(nb + 1)) + a256(8 * (size_t)R);
}

}  // namespace
}  // namespace ssla

namespace ssla {
namespace {
template <typename T>
int reduce_one_pass(const void* src, const int64_t* off, const int64_t* rows, int64_t R, int64_t S, int64_t C,
                    int op, void* out, int64_t* arg, cudaStream_t s);
}  // namespace
}  // namespace ssla

using namespace ssla;

extern "C" int ssla_segment_offsets_sorted(const int64_t* index, int64_t R, int64_t S,
                                           int64_t* seg_offsets, ssla_stream_t stream) {
  SSLA_CHECK_ARG(R >= 0 && S >= 0, "ssla_segment_offsets_sorted: negative size");
  SSLA_CHECK_ARG(seg_offsets && (R == 0 || index), "ssla_segment_offsets_sorted: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  launch_pdl(offsets_sorted_kernel, dim3(ceil_div(R + 1, 256)), dim3(256), 0, s, index, R, S, seg_offsets);
  SSLA_CHECK_LAUNCH("ssla_segment_offsets_sorted");
  return SSLA_OK;
}

extern "C" size_t ssla_segment_csr_workspace_bytes(int64_t R, int64_t S) { return csr_ws_bytes(R, S); }

extern "C" int ssla_segment_csr(const int64_t* index, int64_t R, int64_t S, int64_t* seg_offsets,
                                int64_t* rows, void* workspace, size_t workspace_bytes,
                                ssla_stream_t stream) {
  SSLA_CHECK_ARG(R >= 0 && S >= 0, "ssla_segment_csr: negative size");
  SSLA_CHECK_ARG(seg_offsets && workspace && (R == 0 || (index && rows)),
                 "ssla_segment_csr: null pointer");
  if (workspace_bytes < csr_ws_bytes(R, S)) {
    set_error("ssla_segment_csr: workspace of %zu bytes < %zu needed", workspace_bytes,
              csr_ws_bytes(R, S));
    return SSLA_ERR_WORKSPACE;
  }
  return build_csr(index, R, S, seg_offsets, rows, workspace, (cudaStream_t)stream);
}

extern "C" int ssla_segment_reduce(const void* src, int dtype, const int64_t* seg_offsets,
                                   const int64_t* rows, int64_t R, int64_t S, int64_t C, int op,
                                   void* out, int64_t* arg, ssla_stream_t stream) {
  SSLA_CHECK_ARG(dtype_ok(dtype), "ssla_segment_reduce: bad dtype");
  SSLA_CHECK_ARG(op >= 0 && op <= 2, "ssla_segment_reduce: bad op %d", op);
  SSLA_CHECK_ARG(R >= 0 && S >= 0 && C >= 0, "ssla_segment_reduce: negative size");
  if (S == 0 || C == 0) return SSLA_OK;
  SSLA_CHECK_ARG(seg_offsets && out && (R == 0 || src), "ssla_segment_reduce: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  return SSLA_DISPATCH_DTYPE(dtype, T, [&] {
    const int rc = reduce_one_pass<T>(src, seg_offsets, rows, R, S, C, op, out, arg, s);
    return rc != SSLA_ERR_UNSUPPORTED ? rc : run_reduce<T>(src, seg_offsets, rows, R, S, C, op, out, arg, s);
  });
}

extern "C" int ssla_gather_rows(const void* src, int dtype, const int64_t* index, int64_t R,
                                int64_t C, void* out, ssla_stream_t stream) {
  SSLA_CHECK_ARG(dtype_ok(dtype), "ssla_gather_rows: bad dtype");
  SSLA_CHECK_ARG(R >= 0 && C >= 0, "ssla_gather_rows: negative size");
  if (R == 0 || C == 0) return SSLA_OK;
  SSLA_CHECK_ARG(src && index && out, "ssla_gather_rows: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  return SSLA_DISPATCH_DTYPE(dtype, T, [&] {
    const bool v4 = C % 4 == 0 && aligned_to(src, 4 * sizeof(T)) && aligned_to(out, 4 * sizeof(T));
    const int64_t threads = R * (v4 ? C / 4 : C);
    if (v4)
      launch_pdl(gather_kernel<T, 4>, dim3(ceil_div(threads, 256)), dim3(256), 0, s, (const T*)src, index, R, C, (T*)out);
    else
      launch_pdl(gather_kernel<T, 1>, dim3(ceil_div(threads, 256)), dim3(256), 0, s, (const T*)src, index, R, C, (T*)out);
    SSLA_CHECK_LAUNCH("ssla_gather_rows");
    return SSLA_OK;
  });
}

extern "C" size_t ssla_index_add_rows_workspace_bytes(int64_t P, int64_t D) {
  return a256(8 * (size_t)(D + 1)) + a256(8 * (size_t)P) + csr_ws_bytes(P, D);
}

namespace ssla {
namespace {
template <typename T, int G>
void launch_pool(int mode, cudaStream_t s, const void* src, const int64_t* off, const int64_t* tmp,
                 int64_t* sorted, int64_t R, int64_t S, void* out_max, int64_t* arg, void* out_mean, void* back,
                 bool presorted = false) {
  constexpr int GP = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : G <= 8 ? 8 : G <= 16 ? 16 : 32;
  const dim3 grid((unsigned)ceil_div(S * GP, 256));
  if (mode == kPoolArg)
    launch_pdl(pool_fused_kernel<T, G, kPoolArg>, grid, dim3(256), 0, s, (const T*)src, off, tmp, sorted, (int)R,
               (int)S, (T*)out_max, arg, (T*)out_mean, (T*)back, presorted);
  else if (mode == kPoolSum)
    launch_pdl(pool_fused_kernel<T, G, kPoolSum>, grid, dim3(256), 0, s, (const T*)src, off, tmp, sorted, (int)R,
               (int)S, (T*)nullptr, (int64_t*)nullptr, (T*)out_mean, (T*)nullptr, presorted);
  else
    launch_pdl(pool_fused_kernel<T, G, kPoolMaxMean>, grid, dim3(256), 0, s, (const T*)src, off, tmp, sorted,
               (int)R, (int)S, (T*)out_max, (int64_t*)nullptr, (T*)out_mean, (T*)back, presorted);
}

// One reduction over segments whose ids are already ascending (a sorted CSR, or the row ranges of
// a sorted index when rows == nullptr) by the one-pass kernel: no sort, 16-byte lanes.
// SSLA_ERR_UNSUPPORTED (nothing launched) when the row width or alignment does not fit it.
template <typename T>
int reduce_one_pass(const void* src, const int64_t* off, const int64_t* rows, int64_t R, int64_t S, int64_t C,
                    int op, void* out, int64_t* arg, cudaStream_t s) {
  constexpr int V = 16 / (int)sizeof(T);
  const int64_t G = C / V;
  const bool ok = C % V == 0 &&
                  (G == 1 || G == 2 || G == 3 || G == 4 || G == 6 || G == 8 || G == 12 || G == 16 || G == 24 ||
                   G == 32) &&
                  aligned_to(src, 16) && aligned_to(out, 16) && R < (int64_t)INT32_MAX && S < (int64_t)INT32_MAX;
  if (!ok) return SSLA_ERR_UNSUPPORTED;
  const int mode = op == SSLA_REDUCE_SUM ? kPoolSum : (op == SSLA_REDUCE_MAX && arg ? kPoolArg : kPoolMaxMean);
  void* mx = op == SSLA_REDUCE_MAX ? out : nullptr;
  void* mean = op == SSLA_REDUCE_MAX ? nullptr : out;
#define SSLA_RED1(GG) \
  case GG: launch_pool<T, GG>(mode, s, src, off, rows, nullptr, R, S, mx, arg, mean, nullptr, true); break
  switch (G) {
    SSLA_RED1(1);
    SSLA_RED1(2);
    SSLA_RED1(3);
    SSLA_RED1(4);
    SSLA_RED1(6);
    SSLA_RED1(8);
    SSLA_RED1(12);
    SSLA_RED1(16);
    SSLA_RED1(24);
    default: launch_pool<T, 32>(mode, s, src, off, rows, nullptr, R, S, mx, arg, mean, nullptr, true); break;
  }
#undef SSLA_RED1
  SSLA_CHECK_LAUNCH("ssla_segment_reduce");
  return SSLA_OK;
}

// Counting sort of the row ids by segment (offsets + ids in arrival order), then the one-pass
// kernel.  Row widths whose 16-byte lane count G is not in {1, 2, 3, 4, 6, 8, 12, 16, 24, 32}
// take the sorted-CSR sequence (reductions + row gather) instead.  mode kPoolSum writes the
// segment sums to out_mean.
template <typename T>
int run_pool(int mode, const void* src, int dtype, const int64_t* index, int64_t R, int64_t S, int64_t C,
             void* out_max, int64_t* arg, void* out_mean, void* back, int64_t* off, int64_t* sorted, char* p,
             int* counts, int64_t nb, int64_t* block_sums, int64_t* tmp, cudaStream_t s) {
  constexpr int V = 16 / (int)sizeof(T);
  const int64_t G = C / V;
  const bool g_ok = G == 1 || G == 2 || G == 3 || G == 4 || G == 6 || G == 8 || G == 12 || G == 16 || G == 24 ||
                    G == 32;
  const bool fused = C % V == 0 && g_ok && aligned_to(src, 16) && aligned_to(out_max, 16) &&
                     aligned_to(out_mean, 16) && aligned_to(back, 16) && R < (int64_t)INT32_MAX &&
                     S < (int64_t)INT32_MAX;
  if (!fused) {
    // general widths: sorted CSR, one reduction per output, then the row gather
    int rc = build_csr(index, R, S, off, sorted, p, s);
    if (!rc && mode == kPoolSum) return run_reduce<T>(src, off, sorted, R, S, C, SSLA_REDUCE_SUM, out_mean, nullptr, s);
    if (!rc && (out_max || arg)) {
      T* mx = (T*)out_max;
      if (!mx) {
        set_error("ssla_scatter_pool: C=%lld needs out_max for arg", (long long)C);
        return SSLA_ERR_UNSUPPORTED;
      }
      rc = run_reduce<T>(src, off, sorted, R, S, C, SSLA_REDUCE_MAX, mx, arg, s);
    }
    if (!rc && out_mean) rc = run_reduce<T>(src, off, sorted, R, S, C, SSLA_REDUCE_MEAN, out_mean, nullptr, s);
    if (!rc && back) return ssla_gather_rows(out_max, dtype, index, R, C, back, (ssla_stream_t)s);
    return rc;
  }
  if (cudaMemsetAsync(counts, 0, 4 * (size_t)S, s) != cudaSuccess) {
    set_error("ssla_scatter_pool: memset failed");
    return SSLA_ERR_CUDA;
  }
  if (R > 0) count_kernel<<<ceil_div(R, 256), 256, 0, s>>>(index, R, S, counts);
  launch_pdl(scan_blocks_kernel, dim3((unsigned)nb), dim3(1024), 0, s, (const int*)counts, S, off, block_sums);
  if (nb <= 1024) {
    launch_pdl(add_block_prefix_kernel, dim3((unsigned)nb), dim3(1024), 0, s, off, S, (const int64_t*)block_sums, nb, counts);
  } else {
    launch_pdl(scan_totals_kernel, dim3(1), dim3(1024), 0, s, block_sums, nb, S, off);
    launch_pdl(add_block_base_kernel, dim3(ceil_div(S, 256)), dim3(256), 0, s, off, S, (const int64_t*)block_sums,
               counts);
  }
  if (R > 0) launch_pdl(fill_kernel, dim3(ceil_div(R, 256)), dim3(256), 0, s, index, R, S, (const int64_t*)off, counts, tmp);
  if (mode != kPoolSum) mode = arg ? kPoolArg : kPoolMaxMean;
#define SSLA_POOL_G(GG) \
  case GG: launch_pool<T, GG>(mode, s, src, off, tmp, sorted, R, S, out_max, arg, out_mean, back); break
  switch (G) {
    SSLA_POOL_G(1);
    SSLA_POOL_G(2);
    SSLA_POOL_G(3);
    SSLA_POOL_G(4);
    SSLA_POOL_G(6);
    SSLA_POOL_G(8);
    SSLA_POOL_G(12);
    SSLA_POOL_G(16);
    SSLA_POOL_G(24);
    default: launch_pool<T, 32>(mode, s, src, off, tmp, sorted, R, S, out_max, arg, out_mean, back); break;
  }
#undef SSLA_POOL_G
  SSLA_CHECK_LAUNCH("ssla_scatter_pool");
  return SSLA_OK;
}

}  // namespace
}  // namespace ssla

extern "C" size_t ssla_scatter_pool_workspace_bytes(int64_t R, int64_t S) {
  return a256(8 * (size_t)(S + 1)) + a256(8 * (size_t)R) + csr_ws_bytes(R, S);
}

extern "C" int ssla_scatter_pool(const void* src, int dtype, const int64_t* index, int64_t R, int64_t S,
                                 int64_t C, void* out_max, int64_t* arg, void* out_mean, void* back,
                                 int64_t* seg_offsets, void* workspace, size_t workspace_bytes,
                                 ssla_stream_t stream) {
  SSLA_CHECK_ARG(dtype_ok(dtype), "ssla_scatter_pool: bad dtype");
  SSLA_CHECK_ARG(R >= 0 && S >= 0 && C >= 0, "ssla_scatter_pool: negative size");
  if (S == 0) return SSLA_OK;  // no segment: nothing to write (back rows are all out of range)
  SSLA_CHECK_ARG(out_max || out_mean || arg || seg_offsets, "ssla_scatter_pool: no output requested");
  SSLA_CHECK_ARG(!back || out_max, "ssla_scatter_pool: back needs out_max");
  SSLA_CHECK_ARG(workspace && (R == 0 || (src && index)), "ssla_scatter_pool: null pointer");
  const size_t need = ssla_scatter_pool_workspace_bytes(R, S);
  if (workspace_bytes < need) {
    set_error("ssla_scatter_pool: workspace of %zu bytes < %zu needed", workspace_bytes, need);
    return SSLA_ERR_WORKSPACE;
  }
  cudaStream_t s = (cudaStream_t)stream;
  char* p = (char*)workspace;
  int64_t* off = seg_offsets ? seg_offsets : (int64_t*)p;
  p += a256(8 * (size_t)(S + 1));
  int64_t* sorted = (int64_t*)p;
  p += a256(8 * (size_t)R);
  int* counts = (int*)p;
  const int64_t nb = (S + 1023) / 1024;
  int64_t* block_sums = (int64_t*)(p + a256(4 * (size_t)S));
  int64_t* tmp = (int64_t*)((char*)block_sums + a256(8 * (size_t)(nb + 1)));
  if (C == 0) return build_csr(index, R, S, off, sorted, p, s);
  return SSLA_DISPATCH_DTYPE(dtype, T, [&] {
    return run_pool<T>(kPoolMaxMean, src, dtype, index, R, S, C, out_max, arg, out_mean, back, off, sorted, p, counts,
                       nb, block_sums, tmp, s);
  });
}

// Deterministic index_add: the one-pass kernel in sum mode over the counting-sorted row lists
// (same workspace layout as ssla_scatter_pool).
extern "C" int ssla_index_add_rows(const void* src, int dtype, const int64_t* index, int64_t P,
                                   int64_t D, int64_t C, void* out, void* workspace,
                                   size_t workspace_bytes, ssla_stream_t stream) {
  SSLA_CHECK_ARG(dtype_ok(dtype), "ssla_index_add_rows: bad dtype");
  SSLA_CHECK_ARG(P >= 0 && D >= 0 && C >= 0, "ssla_index_add_rows: negative size");
  if (D == 0 || C == 0) return SSLA_OK;
  SSLA_CHECK_ARG(out && workspace && (P == 0 || (src && index)), "ssla_index_add_rows: null pointer");
  const size_t need = ssla_index_add_rows_workspace_bytes(P, D);
  if (workspace_bytes < need) {
    set_error("ssla_index_add_rows: workspace of %zu bytes < %zu needed", workspace_bytes, need);
    return SSLA_ERR_WORKSPACE;
  }
  cudaStream_t s = (cudaStream_t)stream;
  char* p = (char*)workspace;
  int64_t* off = (int64_t*)p;
  p += a256(8 * (size_t)(D + 1));
  int64_t* sorted = (int64_t*)p;
  p += a256(8 * (size_t)P);
  int* counts = (int*)p;
  const int64_t nb = (D + 1023) / 1024;
  int64_t* block_sums = (int64_t*)(p + a256(4 * (size_t)D));
  int64_t* tmp = (int64_t*)((char*)block_sums + a256(8 * (size_t)(nb + 1)));
  return SSLA_DISPATCH_DTYPE(dtype, T, [&] {
    return run_pool<T>(kPoolSum, src, dtype, index, P, D, C, nullptr, nullptr, out, nullptr, off, sorted, p, counts,
                       nb, block_sums, tmp, s);
  });
}
