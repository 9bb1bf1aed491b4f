// Pixel grouping of padded event batches (group_events, utils/farsecnn_utils.py:130-174 and
// utils/async_utils.py:10-84), without a sort.
//
// The reference orders all events by (sample, pixel) with a stable sort, finds the groups with
// unique_consecutive and keeps the last max_events_per_px events of each group; the model then
// keeps the first hot_pixel_thres of those (truncate_packed_sequence, model_mos.py:173-209).
// Here, with P = H * W pixels per sample and one counter per (sample, pixel) id:
//   1. count:  events per id (atomics on integer counters, exact);
//   2. scan:   exclusive scans over the ids of the event count, of the non-empty flag (group
//              index) and of the kept count, in 2048-id tiles (tile sums, one scan of the tile
//              sums, tile-local scans); the totals (events, groups, kept events) go to the host;
//   3. place:  every event takes a slot in its id's range by an atomic cursor (unordered);
//   4. order:  every id's slot range is put back in event order (row index): for up to kShort
//              events one thread ranks each event by counting the smaller row indices of its
//              range, otherwise one CTA per id sorts the range in shared memory (bitonic; past
//              kLongMax events, radix selection of the kept ranks first); the kept ranks are
//              written out;
//   5. emit:   per group batch id, h, w, length; per kept event its time and features, and
//              optionally the model's per-pixel delay feature (model_mos.py:190-200).
// The result equals the reference's stable-sort formulation exactly (integer work only).
#include <climits>

#include "common.cuh"

namespace ssla {
namespace group {
namespace {

constexpr int kTile = 2048;      // ids per scan tile
constexpr int kShort = 32;       // longest id range ordered by one thread
constexpr int kLongMax = 4096;   // longest id range sorted whole in shared memory

__device__ __forceinline__ int kept_of(int c, int maxpp, int keep_first) {
  int k = c < maxpp ? c : maxpp;
  return k < keep_first ? k : keep_first;
}

struct Ws {
  int* cnt;        // [NI] events per id
  int* cursor;     // [NI] placement cursor
  int* off;        // [NI] first slot of the id
  int* goff;       // [NI] group index of the id
  int* koff;       // [NI] first kept index of the id
  int* tile_sum;   // [3][nt]
  int* rows;       // [R] placed row indices
  int* krow;       // [R] kept rows in order
  unsigned char* kfirst;  // [R] 1 for the first kept event of a group
  int* nlong;      // [1] number of ids with more than kShort events
  int* longs;      // [R / (kShort + 1) + 1] those ids
};

inline size_t al(size_t x) { return (x + 255) & ~size_t(255); }

inline size_t ws_bytes(int64_t NI, int64_t R) {
  const int64_t nt = (NI + kTile - 1) / kTile;
  return 5 * al(4 * NI) + al(12 * nt) + 2 * al(4 * R) + al(R) + al(4) + al(4 * (R / (kShort + 1) + 1));
}

inline Ws carve(void* base, int64_t NI, int64_t R) {
  const int64_t nt = (NI + kTile - 1) / kTile;
  char* p = (char*)base;
  Ws w;
  auto take = [&](size_t n) {
    char* q = p;
    p += al(n);
    return q;
  };
  w.cnt = (int*)take(4 * NI);
  w.cursor = (int*)take(4 * NI);
  w.nlong = (int*)take(4);  // zeroed together with cnt / cursor (adjacent)
  w.off = (int*)take(4 * NI);
  w.goff = (int*)take(4 * NI);
  w.koff = (int*)take(4 * NI);
  w.tile_sum = (int*)take(12 * nt);
  w.rows = (int*)take(4 * R);
  w.krow = (int*)take(4 * R);
  w.kfirst = (unsigned char*)take(R);
  w.longs = (int*)take(4 * (R / (kShort + 1) + 1));
  return w;
}

__device__ __forceinline__ int64_t pixel_id(const float* __restrict__ ev, int64_t r, int64_t C, int64_t b, int64_t H,
                                            int64_t W) {
  const int64_t x = (int64_t)ev[r * C + 0], y = (int64_t)ev[r * C + 1];
  return b * H * W + y * W + x;
}

__global__ void count_kernel(const float* __restrict__ ev, int64_t B, int64_t Nmax, int64_t C,
                             const int64_t* __restrict__ lengths, int64_t H, int64_t W, int* __restrict__ cnt) {
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < B * Nmax; r += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = r / Nmax, n = r - b * Nmax;
    if (n < lengths[b]) atomicAdd(&cnt[pixel_id(ev, r, C, b, H, W)], 1);
  }
}

// Inclusive block scan of three int values (1024 threads).
__device__ __forceinline__ void block_scan3(int v[3], int tot[3], int (*ws)[32]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < 3; ++k)
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, v[k], o);
      if (lane >= o) v[k] += y;
    }
  if (lane == 31)
    for (int k = 0; k < 3; ++k) ws[k][warp] = v[k];
  __syncthreads();
  if (warp == 0)
    for (int k = 0; k < 3; ++k) {
      int w = ws[k][lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      ws[k][lane] = w;
    }
  __syncthreads();
  for (int k = 0; k < 3; ++k) {
    if (warp > 0) v[k] += ws[k][warp - 1];
    tot[k] = ws[k][31];
  }
  __syncthreads();
}

// 1024 threads, 2 ids per thread: per-tile sums of (events, non-empty, kept).
__global__ void __launch_bounds__(1024) tile_sum_kernel(const int* __restrict__ cnt, int64_t NI, int maxpp,
                                                        int keep_first, int* __restrict__ tile_sum, int64_t nt) {
  __shared__ int ws[3][32];
  const int64_t base = blockIdx.x * (int64_t)kTile;
  int v[3] = {0, 0, 0};
  for (int j = 0; j < 2; ++j) {
    const int64_t i = base + 2 * threadIdx.x + j;
    const int c = i < NI ? cnt[i] : 0;
    v[0] += c;
    v[1] += c > 0;
    v[2] += kept_of(c, maxpp, keep_first);
  }
  int tot[3];
  block_scan3(v, tot, ws);
  if (threadIdx.x == 0)
    for (int k = 0; k < 3; ++k) tile_sum[k * nt + blockIdx.x] = tot[k];
}

// One block: exclusive scan of the tile sums in place; totals.
__global__ void __launch_bounds__(1024) tile_scan_kernel(int* __restrict__ tile_sum, int64_t nt, int* __restrict__ totals) {
  __shared__ int ws[3][32];
  __shared__ int carry[3];
  if (threadIdx.x < 3) carry[threadIdx.x] = 0;
  __syncthreads();
  for (int64_t base = 0; base < nt; base += 1024) {
    const int64_t i = base + threadIdx.x;
    int v[3], x[3];
    for (int k = 0; k < 3; ++k) x[k] = v[k] = i < nt ? tile_sum[k * nt + i] : 0;
    int tot[3];
    block_scan3(v, tot, ws);
    if (i < nt)
      for (int k = 0; k < 3; ++k) tile_sum[k * nt + i] = carry[k] + v[k] - x[k];
    __syncthreads();
    if (threadIdx.x < 3) carry[threadIdx.x] += tot[threadIdx.x];
    __syncthreads();
  }
  if (threadIdx.x < 3) totals[threadIdx.x] = carry[threadIdx.x];
}

// Tile-local exclusive scans + tile offsets -> off, goff, koff; ids with long ranges listed.
__global__ void __launch_bounds__(1024) tile_apply_kernel(const int* __restrict__ cnt, int64_t NI, int maxpp,
                                                          int keep_first, const int* __restrict__ tile_sum, int64_t nt,
                                                          int* __restrict__ off, int* __restrict__ goff,
                                                          int* __restrict__ koff, int* __restrict__ nlong,
                                                          int* __restrict__ longs) {
  __shared__ int ws[3][32];
  const int64_t base = blockIdx.x * (int64_t)kTile;
  int c2[2], v[3] = {0, 0, 0};
  for (int j = 0; j < 2; ++j) {
    const int64_t i = base + 2 * threadIdx.x + j;
    c2[j] = i < NI ? cnt[i] : 0;
    v[0] += c2[j];
    v[1] += c2[j] > 0;
    v[2] += kept_of(c2[j], maxpp, keep_first);
  }
  int inc[3] = {v[0], v[1], v[2]}, tot[3];
  block_scan3(inc, tot, ws);
  int e[3];
  for (int k = 0; k < 3; ++k) e[k] = tile_sum[k * nt + blockIdx.x] + inc[k] - v[k];
  for (int j = 0; j < 2; ++j) {
    const int64_t i = base + 2 * threadIdx.x + j;
    if (i < NI) {
      off[i] = e[0];
      goff[i] = e[1];
      koff[i] = e[2];
      if (c2[j] > kShort) longs[atomicAdd(nlong, 1)] = (int)i;
    }
    e[0] += c2[j];
    e[1] += c2[j] > 0;
    e[2] += kept_of(c2[j], maxpp, keep_first);
  }
}

__global__ void place_kernel(const float* __restrict__ ev, int64_t B, int64_t Nmax, int64_t C,
                             const int64_t* __restrict__ lengths, int64_t H, int64_t W, const int* __restrict__ off,
                             int* __restrict__ cursor, int* __restrict__ rows) {
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < B * Nmax; r += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = r / Nmax, n = r - b * Nmax;
    if (n < lengths[b]) {
      const int64_t id = pixel_id(ev, r, C, b, H, W);
      rows[off[id] + atomicAdd(&cursor[id], 1)] = (int)r;
    }
  }
}

// Ids with 1..kShort events: each event's rank in its range is the number of smaller row
// indices there (rows are distinct); the kept ranks are written in order.
__global__ void order_short_kernel(const int* __restrict__ cnt, const int* __restrict__ off,
                                   const int* __restrict__ koff, int64_t NI, int maxpp, int keep_first,
                                   const int* __restrict__ rows, int* __restrict__ krow,
                                   unsigned char* __restrict__ kfirst) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < NI; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = cnt[i];
    if (c == 0 || c > kShort) continue;
    const int o = off[i], ko = koff[i];
    const int start = c > maxpp ? c - maxpp : 0;
    const int n = kept_of(c, maxpp, keep_first);
    for (int j = 0; j < c; ++j) {
      const int x = rows[o + j];
      int rank = 0;
      for (int m = 0; m < c; ++m) rank += rows[o + m] < x;
      if (rank >= start && rank < start + n) {
        krow[ko + rank - start] = x;
        kfirst[ko + rank - start] = rank == start;
      }
    }
  }
}

// Bitonic sort of s[0 .. n) (n a power of two) by the block.
__device__ void block_bitonic(int* s, int n) {
  for (int k = 2; k <= n; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int t = threadIdx.x; t < n; t += blockDim.x) {
        const int p = t ^ j;
        if (p > t) {
          const int a = s[t], b = s[p];
          const bool up = (t & k) == 0;
          if ((a > b) == up) {
            s[t] = b;
            s[p] = a;
          }
        }
      }
      __syncthreads();
    }
}

// Value of rank `rank` (0-based, ascending) among the distinct non-negative ints v[0 .. c),
// by bitwise radix selection (31 counting passes over the range).
__device__ int block_select(const int* __restrict__ v, int c, int rank, int* red) {
  int prefix = 0;
  for (int bit = 30; bit >= 0; --bit) {
    const int cand = prefix | (1 << bit);
    // values below cand sharing the decided high bits... count values < cand among those
    // whose bits above `bit` equal prefix's
    int n = 0;
    for (int t = threadIdx.x; t < c; t += blockDim.x) {
      const int x = v[t];
      n += ((x >> (bit + 1)) == (prefix >> (bit + 1))) && x < cand;
    }
    for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(red, n);
    __syncthreads();
    const int below = *red;
    __syncthreads();
    if (threadIdx.x == 0) *red = 0;
    __syncthreads();
    // `rank` counts from the smallest value sharing the prefix: subtract those already below
    if (rank >= below) {
      prefix = cand;
      rank -= below;
    }
  }
  return prefix;
}

// Ids with more than kShort events: one CTA per id (listed by tile_apply).
__global__ void __launch_bounds__(512) order_long_kernel(const int* __restrict__ cnt, const int* __restrict__ off,
                                                         const int* __restrict__ koff, int maxpp, int keep_first,
                                                         const int* __restrict__ nlong, const int* __restrict__ longs,
                                                         const int* __restrict__ rows, int* __restrict__ krow,
                                                         unsigned char* __restrict__ kfirst) {
  __shared__ int s[kLongMax];
  __shared__ int red;
  if (threadIdx.x == 0) red = 0;
  __syncthreads();
  const int nl = *nlong;
  for (int li = blockIdx.x; li < nl; li += gridDim.x) {
    const int id = longs[li];
    const int c = cnt[id], o = off[id], ko = koff[id];
    const int start = c > maxpp ? c - maxpp : 0;
    const int n = kept_of(c, maxpp, keep_first);
    if (c <= kLongMax) {
      int p2 = 1;
      while (p2 < c) p2 <<= 1;
      for (int t = threadIdx.x; t < p2; t += blockDim.x) s[t] = t < c ? rows[o + t] : INT_MAX;
      __syncthreads();
      block_bitonic(s, p2);
      for (int t = threadIdx.x; t < n; t += blockDim.x) {
        krow[ko + t] = s[start + t];
        kfirst[ko + t] = t == 0;
      }
      __syncthreads();
    } else {
      // kept ranks [start, start + n) in windows of kLongMax: select the window's smallest and
      // largest values, collect the values between them, sort them
      for (int w0 = 0; w0 < n; w0 += kLongMax) {
        const int wn = (n - w0) < kLongMax ? (n - w0) : kLongMax;
        const int lo = block_select(rows + o, c, start + w0, &red);
        const int hi = block_select(rows + o, c, start + w0 + wn - 1, &red);
        int p2 = 1;
        while (p2 < wn) p2 <<= 1;
        for (int t = threadIdx.x; t < p2; t += blockDim.x) s[t] = INT_MAX;
        __syncthreads();
        for (int t = threadIdx.x; t < c; t += blockDim.x) {
          const int x = rows[o + t];
          if (x >= lo && x <= hi) s[atomicAdd(&red, 1)] = x;
        }
        __syncthreads();
        if (threadIdx.x == 0) red = 0;
        __syncthreads();
        block_bitonic(s, p2);
        for (int t = threadIdx.x; t < wn; t += blockDim.x) {
          krow[ko + w0 + t] = s[t];
          kfirst[ko + w0 + t] = w0 + t == 0;
        }
        __syncthreads();
      }
    }
  }
}

__global__ void emit_groups_kernel(const int* __restrict__ cnt, const int* __restrict__ goff, int64_t NI,
                                   int64_t H, int64_t W, int maxpp, int keep_first, int64_t* __restrict__ batch_id,
                                   int64_t* __restrict__ gh, int64_t* __restrict__ gw, int64_t* __restrict__ glen) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < NI; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = cnt[i];
    if (c == 0) continue;
    const int64_t g = goff[i], P = H * W, pix = i % P;
    batch_id[g] = i / P;
    gh[g] = pix / W;
    gw[g] = pix % W;
    glen[g] = kept_of(c, maxpp, keep_first);
  }
}

// Per kept event: time (column 2, as int64) and features (columns 3..C-1); with dt_col >= 0
// feature dt_col is replaced by the pixel delay of model_mos.py:190-200: 1 for the first event
// of a group, else min((t - t_prev) / 1e5, 1) (IEEE division) with t the time column.
__global__ void emit_events_kernel(const float* __restrict__ ev, int64_t C, const int* __restrict__ krow,
                                   const unsigned char* __restrict__ kfirst, int64_t K, int dt_col,
                                   int64_t* __restrict__ time, float* __restrict__ feats) {
  const int64_t F = C - 3;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < K; j += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = krow[j];
    const float t = ev[r * C + 2];
    time[j] = (int64_t)t;
    for (int64_t f = 0; f < F; ++f) feats[j * F + f] = ev[r * C + 3 + f];
    if (dt_col >= 0) {
      float dt = 1.f;
      if (!kfirst[j]) {
        const float d = t - ev[(int64_t)krow[j - 1] * C + 2];
        dt = fminf(__fdiv_rn(d, 1e5f), 1.f);
      }
      feats[j * F + dt_col] = dt;
    }
  }
}

inline unsigned grid_for(int64_t n, int per = 256) {
  int64_t g = (n + per - 1) / per;
  const int64_t cap = (int64_t)kNumSMs * 16;
  return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace
}  // namespace group
}  // namespace ssla

using namespace ssla;
using namespace ssla::group;

extern "C" size_t ssla_group_events_workspace_bytes(int64_t B, int64_t Nmax, int64_t H, int64_t W) {
  return ws_bytes(B * H * W, B * Nmax);
}

extern "C" int ssla_group_events_count(const float* events, int64_t B, int64_t Nmax, int64_t C,
                                       const int64_t* lengths, int64_t H, int64_t W, int64_t max_per_px,
                                       int64_t keep_first, void* workspace, size_t workspace_bytes, int* totals,
                                       ssla_stream_t stream) {
  SSLA_CHECK_ARG(B >= 0 && Nmax >= 0 && C >= 4 && H > 0 && W > 0 && max_per_px > 0 && keep_first > 0,
                 "ssla_group_events_count: bad size");
  SSLA_CHECK_ARG(B * H * W < ((int64_t)1 << 31) && B * Nmax < ((int64_t)1 << 31),
                 "ssla_group_events_count: B*H*W and B*Nmax must stay below 2^31");
  SSLA_CHECK_ARG(workspace_bytes >= ws_bytes(B * H * W, B * Nmax), "ssla_group_events_count: workspace too small");
  SSLA_CHECK_ARG((B * Nmax == 0 || (events && lengths)) && workspace && totals, "ssla_group_events_count: null pointer");
  const int64_t NI = B * H * W, R = B * Nmax, nt = (NI + kTile - 1) / kTile;
  cudaStream_t s = (cudaStream_t)stream;
  Ws w = carve(workspace, NI, R);
  // cnt, cursor and nlong are adjacent: one clear
  if (cudaMemsetAsync(w.cnt, 0, (char*)(w.nlong + 1) - (char*)w.cnt, s) != cudaSuccess) {
    set_error("ssla_group_events_count: memset failed");
    return SSLA_ERR_CUDA;
  }
  const int mp = (int)(max_per_px < INT32_MAX ? max_per_px : INT32_MAX);
  const int kf = (int)(keep_first < INT32_MAX ? keep_first : INT32_MAX);
  if (R) count_kernel<<<grid_for(R), 256, 0, s>>>(events, B, Nmax, C, lengths, H, W, w.cnt);
  tile_sum_kernel<<<(unsigned)nt, 1024, 0, s>>>(w.cnt, NI, mp, kf, w.tile_sum, nt);
  tile_scan_kernel<<<1, 1024, 0, s>>>(w.tile_sum, nt, totals);
  tile_apply_kernel<<<(unsigned)nt, 1024, 0, s>>>(w.cnt, NI, mp, kf, w.tile_sum, nt, w.off, w.goff, w.koff, w.nlong,
                                                 w.longs);
  if (R) place_kernel<<<grid_for(R), 256, 0, s>>>(events, B, Nmax, C, lengths, H, W, w.off, w.cursor, w.rows);
  order_short_kernel<<<grid_for(NI), 256, 0, s>>>(w.cnt, w.off, w.koff, NI, mp, kf, w.rows, w.krow, w.kfirst);
  order_long_kernel<<<kNumSMs, 512, 0, s>>>(w.cnt, w.off, w.koff, mp, kf, w.nlong, w.longs, w.rows, w.krow,
                                             w.kfirst);
  SSLA_CHECK_LAUNCH("ssla_group_events_count");
  return SSLA_OK;
}

extern "C" int ssla_group_events_emit(const float* events, int64_t B, int64_t Nmax, int64_t C, int64_t H, int64_t W,
                                      int64_t max_per_px, int64_t keep_first, const void* workspace, int64_t G,
                                      int64_t K, int dt_col, int64_t* batch_id, int64_t* h, int64_t* w_,
                                      int64_t* lengths_out, int64_t* time, float* feats, ssla_stream_t stream) {
  SSLA_CHECK_ARG(G >= 0 && K >= 0 && dt_col < C - 3, "ssla_group_events_emit: bad size");
  const int64_t NI = B * H * W;
  cudaStream_t s = (cudaStream_t)stream;
  Ws w = carve(const_cast<void*>(workspace), NI, B * Nmax);
  const int mp = (int)(max_per_px < INT32_MAX ? max_per_px : INT32_MAX);
  const int kf = (int)(keep_first < INT32_MAX ? keep_first : INT32_MAX);
  if (G) emit_groups_kernel<<<grid_for(NI), 256, 0, s>>>(w.cnt, w.goff, NI, H, W, mp, kf, batch_id, h, w_, lengths_out);
  if (K) emit_events_kernel<<<grid_for(K), 256, 0, s>>>(events, C, w.krow, w.kfirst, K, dt_col, time, feats);
  SSLA_CHECK_LAUNCH("ssla_group_events_emit");
  return SSLA_OK;
}
