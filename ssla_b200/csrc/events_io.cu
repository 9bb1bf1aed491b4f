// Event-stream input on the GPU: Prophesee .dat (Event2D) payloads resident in device memory,
// sliced into per-sample time windows and decoded straight into the padded model batch.
//
// A .dat event is two little-endian 32-bit words: the timestamp t (u32, microseconds) and a
// packed word with x in bits 0-13, y in bits 14-27 and the polarity in bit 28
// (utils/io/dat_events_tools.py:14, :40-44).  The Gen1 dataset takes, for a label at time ts,
// the events the stream loader returns after seek_time(ts - window) and
// load_delta_t(window + 1) (dataset/gen1.py:190-193, utils/io/psee_loader.py:109-219), and the
// batch collation stacks them as float32 <t, x, y, p>, zero-pads to the longest sample,
// reorders to <x, y, t, p> and maps p to 2p - 1, padding rows included
// (model_base.py:82-117).
//
//   1. window_ranges: one warp per sample reproduces the loader's cursor arithmetic on the
//      resident timestamps: the interval bisection of seek_time (stopping at term_criterion
//      events, an exact timestamp hit leaving the cursor one event past the hit), the
//      bisect-left of the remaining interval, and load_delta_t's walk over 100000-event
//      buffers that cuts the last buffer with a bisect-left of final_time.  Result: the
//      [begin, end) event range of every sample.
//   2. decode_windows: one thread per output row of [B, Nmax, 4] decodes its event (8-byte
//      load) and stores one float4; rows past a sample's length get the padding row
//      (0, 0, 0, -1).  Pure streaming work: 8 bytes read and 16 written per row.
#include "common.cuh"

namespace ssla {
namespace {

constexpr int64_t kLoadBatch = 100000;  // events per buffer of load_delta_t

// The cursor searches are chains of dependent loads (one per bisection level); a warp takes
// one sample and evaluates them five levels at a time: lane j (0..30) follows the path of node
// j + 1 of the next five levels (heap order: the bits after the leading one pick the lower or
// upper half), loads that node's probe, and the walk then reads the probes from registers.
// The visited probes, the comparisons and hence the results are those of the one-at-a-time
// loop, only the loads overlap.
constexpr int kLevels = 5;
constexpr unsigned kFull = 0xffffffffu;

// First index in [lo, hi) whose timestamp is not below `key` (numpy searchsorted, side left,
// for one key: plain bisection mid = lo + (hi - lo) / 2, defined for any data).
__device__ int64_t warp_bisect_left(const uint2* ev, int64_t lo, int64_t hi, int64_t key) {
  const int lane = threadIdx.x & 31;
  while (lo < hi) {
    // this lane's node: apply the path bits of heap index lane + 1 from (lo, hi)
    int64_t l = lo, h = hi;
    const int node = lane + 1;
    const int depth = 31 - __clz(node);
    bool valid = lane < (1 << kLevels) - 1;
    for (int d = depth - 1; d >= 0 && valid; --d) {
      if (l >= h) { valid = false; break; }
      const int64_t m = l + ((h - l) >> 1);
      if ((node >> d) & 1) l = m + 1;  // upper half: t[m] < key
      else h = m;
    }
    valid = valid && l < h;
    const int64_t m = l + ((h - l) >> 1);
    const int64_t v = valid ? (int64_t)__ldg(&ev[m].x) : 0;
    int cur = 0;  // walk the five levels with the gathered probes
    for (int lev = 0; lev < kLevels && lo < hi; ++lev) {
      const int64_t vm = __shfl_sync(kFull, v, cur);
      const int64_t mid = lo + ((hi - lo) >> 1);
      if (vm < key) { lo = mid + 1; cur = 2 * cur + 2; }
      else { hi = mid; cur = 2 * cur + 1; }
    }
  }
  return lo;
}

__global__ void window_ranges_kernel(const uint2* __restrict__ ev, const int64_t* __restrict__ rec_start,
                                     const int64_t* __restrict__ rec_count, const int64_t* __restrict__ t_end,
                                     int64_t B, int64_t window, int64_t term, int64_t* __restrict__ range,
                                     int64_t* __restrict__ lengths) {
  const int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (b >= B) return;  // whole warps exit together
  const uint2* e = ev + rec_start[b];
  const int64_t n = rec_count[b];
  const int64_t total = n ? (int64_t)__ldg(&e[n - 1].x) : 0;  // total_time(): last timestamp
  const int64_t ft = t_end[b] - window;                         // seek_time target
  int64_t pos = 0, cur = 0;
  bool done = false;
  if (ft > total) {
    done = true;  // cursor at the end of the stream
    pos = n;
  } else if (ft > 0) {
    int64_t low = 0, high = n;
    bool hit = false;
    // seek_time's bisection: mid = (low + high) / 2 while more than `term` events remain
    while (!hit && high - low > term) {
      int64_t l = low, h = high;
      const int node = lane + 1;
      const int depth = 31 - __clz(node);
      bool valid = lane < (1 << kLevels) - 1;
      for (int d = depth - 1; d >= 0 && valid; --d) {
        if (h - l <= term) { valid = false; break; }
        const int64_t m = (l + h) / 2;
        if ((node >> d) & 1) l = m + 1;  // t[m] < ft
        else h = m;                      // t[m] > ft
      }
      valid = valid && h - l > term;
      const int64_t v = valid ? (int64_t)__ldg(&e[(l + h) / 2].x) : 0;
      int c = 0;
      for (int lev = 0; lev < kLevels && high - low > term; ++lev) {
        const int64_t tm = __shfl_sync(kFull, v, c);
        const int64_t mid = (low + high) / 2;
        if (tm > ft) { high = mid; c = 2 * c + 1; }
        else if (tm < ft) { low = mid + 1; c = 2 * c + 2; }
        else {
          pos = mid + 1;  // the probe read leaves the cursor one event past the hit
          hit = true;
          break;
        }
      }
    }
    if (!hit) {
      pos = warp_bisect_left(e, low, high, ft);
      if (pos < 0) pos = 0;
      if (pos > n) pos = n;
    }
    cur = ft;
    done = pos >= n;
  }
  int64_t begin = pos, end = pos;
  if (!done && pos < n) {
    // load_delta_t(window + 1): buffers of kLoadBatch events from the cursor until one ends at
    // or after fin (or the stream ends); 32 buffer ends are probed per round
    const int64_t fin = cur + window + 1;
    int64_t first = pos;  // start of the 32 buffers of this round
    int64_t last_lo = pos, last_hi = pos;
    for (;;) {
      const int64_t lo = first + (int64_t)lane * kLoadBatch;
      const int64_t hi = lo + kLoadBatch < n ? lo + kLoadBatch : n;
      const bool exists = lo < n;
      const bool stop = exists && ((int64_t)__ldg(&e[hi - 1].x) >= fin || hi >= n);
      const unsigned m = __ballot_sync(kFull, stop);
      if (m) {
        const int k = __ffs(m) - 1;
        last_lo = first + (int64_t)k * kLoadBatch;
        last_hi = last_lo + kLoadBatch < n ? last_lo + kLoadBatch : n;
        break;
      }
      first += 32 * kLoadBatch;
    }
    end = warp_bisect_left(e, last_lo, last_hi, fin);
  }
  if (lane == 0) {
    range[2 * b] = begin;
    range[2 * b + 1] = end;
    lengths[b] = end - begin;
  }
}

__global__ void decode_windows_kernel(const uint2* __restrict__ ev, const int64_t* __restrict__ rec_start,
                                      const int64_t* __restrict__ range, int64_t B, int64_t Nmax,
                                      float4* __restrict__ out) {
  const int64_t rows = B * Nmax;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / Nmax, j = i - b * Nmax;
    const int64_t beg = range[2 * b], len = range[2 * b + 1] - beg;
    float4 r = make_float4(0.f, 0.f, 0.f, -1.f);
    if (j < len) {
      const uint2 w = __ldg(ev + rec_start[b] + beg + j);
      r.x = (float)(w.y & 16383u);
      r.y = (float)((w.y & 268419072u) >> 14);
      r.z = __uint2float_rn(w.x);
      r.w = (float)((w.y & 268435456u) >> 28) * 2.f - 1.f;
    }
    out[i] = r;
  }
}

}  // namespace
}  // namespace ssla

using namespace ssla;

extern "C" int ssla_dat_window_ranges(const uint32_t* words, const int64_t* rec_start, const int64_t* rec_count,
                                      const int64_t* t_end, int64_t B, int64_t window, int64_t term_criterion,
                                      int64_t* range, int64_t* lengths, ssla_stream_t stream) {
  SSLA_CHECK_ARG(B >= 0 && window >= 0 && term_criterion >= 0, "ssla_dat_window_ranges: bad sizes");
  if (B == 0) return SSLA_OK;
  SSLA_CHECK_ARG(words && rec_start && rec_count && t_end && range && lengths, "ssla_dat_window_ranges: null pointer");
  SSLA_CHECK_ARG(reinterpret_cast<uintptr_t>(words) % 8 == 0, "ssla_dat_window_ranges: words must be 8-byte aligned");
  window_ranges_kernel<<<(unsigned)ceil_div(B, 4), 128, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint2*>(words), rec_start, rec_count, t_end, B, window, term_criterion, range, lengths);
  SSLA_CHECK_LAUNCH("ssla_dat_window_ranges");
  return SSLA_OK;
}

extern "C" int ssla_dat_decode_windows(const uint32_t* words, const int64_t* rec_start, const int64_t* range,
                                       int64_t B, int64_t Nmax, float* out, ssla_stream_t stream) {
  SSLA_CHECK_ARG(B >= 0 && Nmax >= 0, "ssla_dat_decode_windows: bad sizes");
  if (B * Nmax == 0) return SSLA_OK;
  SSLA_CHECK_ARG(words && rec_start && range && out, "ssla_dat_decode_windows: null pointer");
  SSLA_CHECK_ARG(reinterpret_cast<uintptr_t>(words) % 8 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0,
                 "ssla_dat_decode_windows: words must be 8-byte and out 16-byte aligned");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = ceil_div(B * Nmax, (int64_t)256);
  const int64_t cap = (int64_t)sms * 8;
  decode_windows_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint2*>(words), rec_start, range, B, Nmax, reinterpret_cast<float4*>(out));
  SSLA_CHECK_LAUNCH("ssla_dat_decode_windows");
  return SSLA_OK;
}
