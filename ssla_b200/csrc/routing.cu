// Event routing of the sparse layers on the GPU: pixel groups -> receptive fields (MoS patches,
// pooling windows) with each field's events in time order (utils/async_utils.py:125-240,
// utils/farsecnn_utils.py:177-265).
//
// The reference builds dense [batch * fields, kh*kw] masks, replicates events with
// repeat_interleave and orders every field's events with a sort.  Here:
//   1. pixel_map: a dense [B, H, W] int32 map of the active pixel groups (-1 elsewhere);
//   2. field_lengths: one thread per field adds the lengths of the groups in its window
//      (window pixel (dy, dx) of field (oy, ox) = (oy*sh - pt + dy, ox*sw - pl + dx));
//   3. (host) the non-empty fields in ascending id order and their output offsets;
//   4. fill: one thread per non-empty field merges the time-ordered event lists of its window's
//      groups, smallest (time, window position, event order) first -- the order a stable sort
//      by time of the (position, event)-ordered rows gives.
// A group's events must be in non-decreasing time order (time-ordered event streams keep it
// through every layer); groups_time_sorted checks it so the caller can fall back otherwise.
#include "common.cuh"

namespace ssla {
namespace {

constexpr int kMaxArea = 32;

struct Geo {
  int B, H, W, kh, kw, sh, sw, pt, pl, oh, ow;
};

// Groups with coordinates outside [B, H, W] are skipped and counted in *bad.
__global__ void pixel_map_kernel(const int64_t* __restrict__ bid, const int64_t* __restrict__ h,
                                 const int64_t* __restrict__ w, int64_t G, int B, int H, int W, int* __restrict__ map,
                                 int* __restrict__ bad) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= G) return;
  const int64_t b = bid[g], y = h[g], x = w[g];
  if (b < 0 || b >= B || y < 0 || y >= H || x < 0 || x >= W) {
    atomicAdd(bad, 1);
    return;
  }
  map[(b * H + y) * W + x] = (int)g;
}

__global__ void time_sorted_kernel(const int64_t* __restrict__ start, const int64_t* __restrict__ len,
                                   const int64_t* __restrict__ t, int64_t G, int* __restrict__ bad) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= G) return;
  const int64_t s = start[g], e = s + len[g];
  for (int64_t i = s + 1; i < e; ++i)
    if (t[i] < t[i - 1]) {
      atomicExch(bad, 1);
      return;
    }
}

// Window pixel p of field (b, oy, ox) -> group id (-1 if outside the frame or inactive).
__device__ __forceinline__ int window_group(const int* __restrict__ map, const Geo& g, int b, int oy, int ox, int p) {
  const int y = oy * g.sh - g.pt + p / g.kw;
  const int x = ox * g.sw - g.pl + p % g.kw;
  if (y < 0 || y >= g.H || x < 0 || x >= g.W) return -1;
  return map[((int64_t)b * g.H + y) * g.W + x];
}

__global__ void field_lengths_kernel(const int* __restrict__ map, const int64_t* __restrict__ glen, Geo geo,
                                     int64_t* __restrict__ flen) {
  const int64_t nf = (int64_t)geo.oh * geo.ow;
  const int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= geo.B * nf) return;
  const int b = (int)(f / nf);
  const int r = (int)(f - b * nf);
  const int oy = r / geo.ow, ox = r - oy * geo.ow;
  int64_t n = 0;
  for (int p = 0; p < geo.kh * geo.kw; ++p) {
    const int gi = window_group(map, geo, b, oy, ox, p);
    if (gi >= 0) n += glen[gi];
  }
  flen[f] = n;
}

// Outputs of a block's fields form one contiguous range; up to kStage of them are staged in
// shared memory and written out coalesced (the rest, for blocks with very long fields, go
// straight to global memory).
constexpr int kFillThreads = 128, kStage = 2048;

// A >= window size: the per-list state lives in registers (every access is an unrolled loop
// over compile-time indices).
template <int A>
__global__ void __launch_bounds__(kFillThreads) fill_kernel(
    const int* __restrict__ map, const int64_t* __restrict__ gstart, const int64_t* __restrict__ glen,
    const int64_t* __restrict__ gtime, Geo geo, const int64_t* __restrict__ field_ids,
    const int64_t* __restrict__ field_off, int64_t F, int64_t* __restrict__ src, int64_t* __restrict__ pos,
    int64_t* __restrict__ time) {
  __shared__ int64_t s_src[kStage], s_time[kStage];
  __shared__ unsigned char s_pos[kStage];
  const int64_t f0 = (int64_t)blockIdx.x * kFillThreads;
  const int64_t i = f0 + threadIdx.x;
  const int64_t flast = (f0 + kFillThreads < F ? f0 + kFillThreads : F);
  const int64_t base = field_off[f0], span = field_off[flast] - base;
  if (i < F) {
    const int64_t nf = (int64_t)geo.oh * geo.ow;
    const int64_t f = field_ids[i];
    const int b = (int)(f / nf);
    const int r = (int)(f - b * nf);
    const int oy = r / geo.ow, ox = r - oy * geo.ow;
    // list j = window position j: events [cur, end) of the group there (empty if none)
    int64_t cur[A], end[A], head[A];
#pragma unroll
    for (int j = 0; j < A; ++j) {
      cur[j] = end[j] = head[j] = 0;
      if (j < geo.kh * geo.kw) {
        const int gi = window_group(map, geo, b, oy, ox, j);
        if (gi >= 0) {
          cur[j] = gstart[gi];
          end[j] = cur[j] + glen[gi];
          if (end[j] > cur[j]) head[j] = gtime[cur[j]];
        }
      }
    }
    const int64_t oe = field_off[i + 1];
    for (int64_t o = field_off[i]; o < oe; ++o) {
      // smallest head time; ties -> lowest position
      int best = -1;
      int64_t bt = 0;
#pragma unroll
      for (int j = 0; j < A; ++j)
        if (cur[j] < end[j] && (best < 0 || head[j] < bt)) {
          best = j;
          bt = head[j];
        }
      if (best < 0) break;  // offsets inconsistent with the lists (not produced by field_lengths)
      int64_t sidx = 0;
#pragma unroll
      for (int j = 0; j < A; ++j)
        if (j == best) {
          sidx = cur[j]++;
          if (cur[j] < end[j]) head[j] = gtime[cur[j]];
        }
      const int64_t so = o - base;
      if (so < kStage) {
        s_src[so] = sidx;
        s_pos[so] = (unsigned char)best;
        s_time[so] = bt;
      } else {
        src[o] = sidx;
        pos[o] = best;
        time[o] = bt;
      }
    }
  }
  __syncthreads();
  const int64_t ns = span < kStage ? span : kStage;
  for (int64_t k = threadIdx.x; k < ns; k += kFillThreads) {
    src[base + k] = s_src[k];
    pos[base + k] = s_pos[k];
    time[base + k] = s_time[k];
  }
}

// Compaction of the non-empty fields (flen > 0) in ascending field order, three passes:
// per-block (1024 fields) exclusive prefixes of the non-empty count and of the event count,
// one CTA scanning the block totals in place (1024 at a time with a carry), and a scatter of
// field id, length and event offset to each non-empty field's rank.
__device__ __forceinline__ void block_scan2(int64_t& a, int64_t& b, int64_t* wa, int64_t* wb, int64_t& ta,
                                            int64_t& tb) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int64_t ia = a, ib = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t ya = __shfl_up_sync(0xffffffffu, ia, o), yb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) {
      ia += ya;
      ib += yb;
    }
  }
  if (lane == 31) {
    wa[warp] = ia;
    wb[warp] = ib;
  }
  __syncthreads();
  if (warp == 0) {
    int64_t xa = wa[lane], xb = wb[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t ya = __shfl_up_sync(0xffffffffu, xa, o), yb = __shfl_up_sync(0xffffffffu, xb, o);
      if (lane >= o) {
        xa += ya;
        xb += yb;
      }
    }
    wa[lane] = xa;
    wb[lane] = xb;
  }
  __syncthreads();
  const int64_t pa = warp > 0 ? wa[warp - 1] : 0, pb = warp > 0 ? wb[warp - 1] : 0;
  ta = wa[31];
  tb = wb[31];
  a = pa + ia - a;  // exclusive
  b = pb + ib - b;
  __syncthreads();
}

__global__ void __launch_bounds__(1024) field_block_scan_kernel(const int64_t* __restrict__ flen, int64_t nf,
                                                                int64_t* __restrict__ pre_cnt,
                                                                int64_t* __restrict__ pre_len,
                                                                int64_t* __restrict__ bsum) {
  __shared__ int64_t wa[32], wb[32];
  const int64_t f = (int64_t)blockIdx.x * 1024 + threadIdx.x;
  const int64_t l = f < nf ? flen[f] : 0;
  int64_t a = l > 0 ? 1 : 0, b = l, ta, tb;
  block_scan2(a, b, wa, wb, ta, tb);
  if (f < nf) {
    pre_cnt[f] = a;
    pre_len[f] = b;
  }
  if (threadIdx.x == 0) {
    bsum[2 * blockIdx.x] = ta;
    bsum[2 * blockIdx.x + 1] = tb;
  }
}

// stats = {flags[0], flags[1], non-empty fields, routed events}
__global__ void __launch_bounds__(1024) field_totals_kernel(int64_t* __restrict__ bsum, int64_t nb,
                                                            const int* __restrict__ flags,
                                                            int64_t* __restrict__ stats) {
  __shared__ int64_t wa[32], wb[32];
  int64_t ca = 0, cb = 0;
  for (int64_t base = 0; base < nb; base += 1024) {
    const int64_t i = base + threadIdx.x;
    int64_t a = i < nb ? bsum[2 * i] : 0, b = i < nb ? bsum[2 * i + 1] : 0, ta, tb;
    block_scan2(a, b, wa, wb, ta, tb);
    if (i < nb) {
      bsum[2 * i] = ca + a;
      bsum[2 * i + 1] = cb + b;
    }
    ca += ta;
    cb += tb;
  }
  if (threadIdx.x == 0) {
    stats[0] = flags ? flags[0] : 0;
    stats[1] = flags ? flags[1] : 0;
    stats[2] = ca;
    stats[3] = cb;
  }
}

__global__ void field_scatter_kernel(const int64_t* __restrict__ flen, int64_t nf,
                                     const int64_t* __restrict__ pre_cnt, const int64_t* __restrict__ pre_len,
                                     const int64_t* __restrict__ bsum, const int64_t* __restrict__ stats,
                                     int64_t* __restrict__ field_ids, int64_t* __restrict__ lengths,
                                     int64_t* __restrict__ off) {
  const int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (f == 0) off[stats[2]] = stats[3];
  if (f >= nf) return;
  const int64_t l = flen[f];
  if (l <= 0) return;
  const int64_t blk = f >> 10;
  const int64_t k = bsum[2 * blk] + pre_cnt[f];
  field_ids[k] = f;
  lengths[k] = l;
  off[k] = bsum[2 * blk + 1] + pre_len[f];
}

int check_geo(const Geo& g) {
  SSLA_CHECK_ARG(g.B >= 0 && g.H > 0 && g.W > 0 && g.kh > 0 && g.kw > 0 && g.sh > 0 && g.sw > 0 && g.oh >= 0 &&
                     g.ow >= 0,
                 "ssla_route: bad geometry");
  SSLA_CHECK_ARG(g.kh * g.kw <= kMaxArea, "ssla_route: window of %d pixels exceeds %d", g.kh * g.kw, kMaxArea);
  return SSLA_OK;
}

}  // namespace
}  // namespace ssla

using namespace ssla;

extern "C" int ssla_route_pixel_map(const int64_t* batch_id, const int64_t* h, const int64_t* w, int64_t G, int64_t B,
                                    int64_t H, int64_t W, int* map, int* bad, ssla_stream_t stream) {
  SSLA_CHECK_ARG(G >= 0 && B >= 0 && H > 0 && W > 0, "ssla_route_pixel_map: bad sizes");
  if (G == 0) return SSLA_OK;
  SSLA_CHECK_ARG(batch_id && h && w && map && bad, "ssla_route_pixel_map: null pointer");
  pixel_map_kernel<<<(unsigned)ceil_div(G, 256), 256, 0, (cudaStream_t)stream>>>(batch_id, h, w, G, (int)B, (int)H,
                                                                                  (int)W, map, bad);
  SSLA_CHECK_LAUNCH("ssla_route_pixel_map");
  return SSLA_OK;
}

extern "C" int ssla_route_groups_time_sorted(const int64_t* gstart, const int64_t* glen, const int64_t* gtime,
                                             int64_t G, int* bad, ssla_stream_t stream) {
  SSLA_CHECK_ARG(G >= 0, "ssla_route_groups_time_sorted: bad sizes");
  if (G == 0) return SSLA_OK;
  time_sorted_kernel<<<(unsigned)ceil_div(G, 256), 256, 0, (cudaStream_t)stream>>>(gstart, glen, gtime, G, bad);
  SSLA_CHECK_LAUNCH("ssla_route_groups_time_sorted");
  return SSLA_OK;
}

extern "C" int ssla_route_field_lengths(const int* map, const int64_t* glen, int64_t B, int64_t H, int64_t W,
                                        int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t pt, int64_t pl,
                                        int64_t oh, int64_t ow, int64_t* flen, ssla_stream_t stream) {
  const Geo geo{(int)B, (int)H, (int)W, (int)kh, (int)kw, (int)sh, (int)sw, (int)pt, (int)pl, (int)oh, (int)ow};
  int rc = check_geo(geo);
  if (rc) return rc;
  const int64_t n = B * oh * ow;
  if (n == 0) return SSLA_OK;
  field_lengths_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, (cudaStream_t)stream>>>(map, glen, geo, flen);
  SSLA_CHECK_LAUNCH("ssla_route_field_lengths");
  return SSLA_OK;
}

extern "C" int ssla_route_fill(const int* map, const int64_t* gstart, const int64_t* glen, const int64_t* gtime,
                               int64_t B, int64_t H, int64_t W, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                               int64_t pt, int64_t pl, int64_t oh, int64_t ow, const int64_t* field_ids,
                               const int64_t* field_off, int64_t F, int64_t* src, int64_t* pos, int64_t* time,
                               ssla_stream_t stream) {
  const Geo geo{(int)B, (int)H, (int)W, (int)kh, (int)kw, (int)sh, (int)sw, (int)pt, (int)pl, (int)oh, (int)ow};
  int rc = check_geo(geo);
  if (rc) return rc;
  if (F == 0) return SSLA_OK;
  const unsigned grid = (unsigned)ceil_div(F, kFillThreads);
  const int area = (int)(kh * kw);
  cudaStream_t s = (cudaStream_t)stream;
#define SSLA_FILL(A) fill_kernel<A><<<grid, kFillThreads, 0, s>>>(map, gstart, glen, gtime, geo, field_ids, field_off, F, src, pos, time)
  if (area <= 4) SSLA_FILL(4);
  else if (area <= 9) SSLA_FILL(9);
  else if (area <= 16) SSLA_FILL(16);
  else SSLA_FILL(32);
#undef SSLA_FILL
  SSLA_CHECK_LAUNCH("ssla_route_fill");
  return SSLA_OK;
}

extern "C" size_t ssla_route_compact_fields_workspace_bytes(int64_t nf) {
  const int64_t nb = (nf + 1023) / 1024;
  return (size_t)(2 * nf + 2 * nb + 2) * sizeof(int64_t);
}

extern "C" int ssla_route_compact_fields(const int64_t* flen, int64_t nf, const int* flags, int64_t* field_ids,
                                         int64_t* lengths, int64_t* field_off, int64_t* stats, void* workspace,
                                         size_t workspace_bytes, ssla_stream_t stream) {
  SSLA_CHECK_ARG(nf >= 0, "ssla_route_compact_fields: bad size");
  SSLA_CHECK_ARG(stats && field_off && (nf == 0 || (flen && field_ids && lengths && workspace)),
                 "ssla_route_compact_fields: null pointer");
  if (workspace_bytes < ssla_route_compact_fields_workspace_bytes(nf)) {
    set_error("ssla_route_compact_fields: workspace of %zu bytes < %zu needed", workspace_bytes,
              ssla_route_compact_fields_workspace_bytes(nf));
    return SSLA_ERR_WORKSPACE;
  }
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t nb = (nf + 1023) / 1024;
  int64_t* pre_cnt = (int64_t*)workspace;
  int64_t* pre_len = pre_cnt + nf;
  int64_t* bsum = pre_len + nf;
  if (nb > 0)
    field_block_scan_kernel<<<(unsigned)nb, 1024, 0, s>>>(flen, nf, pre_cnt, pre_len, bsum);
  field_totals_kernel<<<1, 1024, 0, s>>>(bsum, nb, flags, stats);
  field_scatter_kernel<<<(unsigned)(nf > 0 ? ceil_div(nf, 256) : 1), 256, 0, s>>>(flen, nf, pre_cnt, pre_len, bsum,
                                                                                   stats, field_ids, lengths,
                                                                                   field_off);
  SSLA_CHECK_LAUNCH("ssla_route_compact_fields");
  return SSLA_OK;
}
