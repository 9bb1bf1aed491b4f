// fp32 GEMM on the tensor cores by split TF32 ("3xTF32"): C[M, N] = A[M, K] * B[N, K]^T.
//
// The MoS layers' projections are fp32 GEMMs with a huge M (patch or pixel events) and small
// K, N (<= a few thousand): on the CUDA cores they are FMA-bound.  Each fp32 operand x is split
// as x = hi + lo with hi = x rounded to TF32 (cvt.rna) and lo = x - hi (exact in fp32), and
// A B^T ~= Ahi Bhi^T + Ahi Blo^T + Alo Bhi^T, accumulated in fp32 in tensor memory; the dropped
// Alo Blo^T term and the TF32 reading of lo leave a relative error near 2^-21 per product, the
// order of fp32 rounding itself.  The tensor core's own accumulation error grows with the
// number of k steps summed into one accumulator, so K is cut into partial sums of 128 that
// the epilogue adds in fp32 registers (round to nearest): the error then stays near that of
// a K = 128 product whatever K is.  B (the weights) is split once on the host side
// (ssla_split_tf32); A is split in shared memory as it arrives.
//
// Persistent, warp-specialised CTA of 14 warps on a 128 x bn output tile per item (items walk n
// fastest, so the CTAs resident together share A row panels in L2).  K of one partial sum
// (<= 128, the pixel-event projections) with N > 128: N split evenly into tiles of at most 256
// columns, 2 stages; otherwise bn = 128 (or N rounded up to 16 when smaller), 3 stages:
//   warp 0      TMA: A (128 x 32 fp32) and the two B tiles per 32-wide k block, into a
//               2- or 3-stage ring (swizzle 128B, zero fill past the matrix edges);
//   warps 2-5   split: each thread rounds one 128-byte row of the A tile to TF32 in place and
//               writes the remainder to the stage's lo tile;
//   warp 1      MMA: one thread issues 3 x 4 tcgen05.mma.kind::tf32 (M = 128, N = bn, K = 8)
//               per k block; four k blocks form a partial sum in one of two TMEM
//               accumulators (double-buffered) and commit stage / accumulator barriers;
//   warps 6-13  epilogue: 32x32b TMEM loads (warp w reads lanes 32 (w % 4) ..) of every
//               partial sum, added in registers (the accumulator released at once), then each
//               warp's 32 x 32 blocks staged in shared memory and written by TMA stores.
// Every wait is bounded; on a timeout the CTA records an error flag and all roles stop.
#include "common.cuh"
#include "tc_util.cuh"
#include "tma_map.cuh"

namespace ssla {
namespace gemm {
namespace {

using namespace ssla::tc;

constexpr int BM = 128, BN = 128, BK = 32;
constexpr int TILE = BM * BK * 4;  // 16 KB A tile
// stage: A (hi in place) | A lo | B hi | B lo, B tiles of BNT rows
__host__ __device__ constexpr int stage_bytes(int bnt) { return 2 * TILE + 2 * bnt * BK * 4; }
constexpr int KB_PARTIAL = 4;  // k blocks (K = 128) per tensor-core partial sum, then fp32 adds
constexpr int NT = 448;       // 14 warps
constexpr int EPI_WARPS = 8;  // warps 6..13
constexpr int STAGING = 32 * 32 * 4;  // per epilogue warp: 32 rows x 32 fp32, 128-byte swizzle
constexpr uint32_t kWaitIters = 1u << 24;
constexpr size_t smem_bytes(int bnt, int st) { return (size_t)st * stage_bytes(bnt) + EPI_WARPS * STAGING + 1024; }

__device__ __forceinline__ uint64_t desc_sw128(const void* tile) {
  return smem_desc(smem_u32(tile), 1024u, 1024u) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

template <int ST>
struct Bars {
  uint64_t full[ST], split[ST], empty[ST], accf[2], acce[2], rd;  // rd: split threads' packed-row reads done
  uint32_t tbase;
  volatile int abort;  // read in every role's loop condition
};

template <class BarsT>
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, BarsT& S, int* err) {
  if (mbar_wait(bar, parity, kWaitIters)) return true;
  if (!S.abort) {
    S.abort = 1;
    atomicExch(err, 1);
  }
  return false;
}

// MULTI: K spans more than one partial sum (the epilogue adds partial sums in registers);
// without it the accumulator is read once, 32 columns at a time, straight into the stores.
// BNT: the largest N tile (B tile rows, TMEM columns per accumulator); ST: pipeline stages.
template <bool MULTI, int BNT, int ST>
__global__ void __launch_bounds__(NT, 1) gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap ma,
                                                             const __grid_constant__ CUtensorMap mbh,
                                                             const __grid_constant__ CUtensorMap mbl,
                                                             const __grid_constant__ CUtensorMap mc, int use_tma_store,
                                                             int M, int N, int K, int bn, int a_cols,
                                                             float* __restrict__ C,
                                                             int64_t ldc, int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  constexpr int STAGES = ST, STAGE_BYTES = stage_bytes(BNT), BTILE = BNT * BK * 4;
  __shared__ Bars<ST> S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int mtiles = (M + BM - 1) / BM, ntiles = (N + bn - 1) / bn, kblocks = (K + BK - 1) / BK;
  const int items = mtiles * ntiles;
  if (warp == 1) tmem_alloc(&S.tbase, 2 * BNT);
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.split[s], 128);
      mbar_init(&S.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&S.accf[a], 1);
      mbar_init(&S.acce[a], 32 * EPI_WARPS);
    }
    mbar_init(&S.rd, 128);
    S.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tensormap(&ma);
    prefetch_tensormap(&mbh);
    prefetch_tensormap(&mbl);
    if (use_tma_store) prefetch_tensormap(&mc);
  }
  __syncthreads();
  fence_after();
  const uint32_t tb = S.tbase;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      for (int i = blockIdx.x; i < items && !S.abort; i += gridDim.x) {
        const int m0 = (i / ntiles) * BM, n0 = (i % ntiles) * bn;
        for (int k = 0; k < kblocks; ++k, ++it) {
          const int s = it % STAGES;
          const uint32_t use = it / STAGES;
          if (use > 0 && !wait_or_abort(&S.empty[s], (use - 1) & 1, S, err)) break;
          unsigned char* st = smem + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&S.full[s], (a_cols ? BM * a_cols * 4 : TILE) + 2 * BTILE);
          tma_load_2d(st, &ma, k * BK, m0, &S.full[s]);
          tma_load_2d(st + 2 * TILE, &mbh, k * BK, n0, &S.full[s]);
          tma_load_2d(st + 2 * TILE + BTILE, &mbl, k * BK, n0, &S.full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32(BM, bn);
      uint32_t it = 0, t = 0;  // t counts partial sums (accumulator uses)
      bool ok = true;
      for (int i = blockIdx.x; ok && i < items && !S.abort; i += gridDim.x) {
        for (int k = 0; k < kblocks; ++k, ++it) {
          const int kp = k % KB_PARTIAL;  // position inside the current partial sum
          const uint32_t a = t & 1;
          if (kp == 0) {
            const uint32_t u = t >> 1;
            if (u > 0 && !wait_or_abort(&S.acce[a], (u - 1) & 1, S, err)) {
              ok = false;
              break;
            }
            fence_after();
          }
          const uint32_t d = tb + a * BNT;
          const int s = it % STAGES;
          if (!wait_or_abort(&S.split[s], (it / STAGES) & 1, S, err)) {
            ok = false;
            break;
          }
          fence_after();
          unsigned char* st = smem + s * STAGE_BYTES;
          const uint64_t ah = desc_sw128(st), al = desc_sw128(st + TILE);
          const uint64_t bh = desc_sw128(st + 2 * TILE), bl = desc_sw128(st + 2 * TILE + BTILE);
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) {  // K = 8 per MMA: 32 bytes along the swizzled row
            const uint64_t o = 2u * kk;
            mma_tf32(d, ah + o, bl + o, idesc, (kp > 0 || kk > 0) ? 1u : 0u);
            mma_tf32(d, al + o, bh + o, idesc, 1u);
            mma_tf32(d, ah + o, bh + o, idesc, 1u);
          }
          commit(&S.empty[s]);
          if (kp == KB_PARTIAL - 1 || k == kblocks - 1) {
            commit(&S.accf[a]);
            ++t;
          }
        }
      }
    }
  } else if (warp < 6) {
    // split: thread r (0..127) owns row r of the A tile (128 bytes: 8 16-byte pieces; the
    // swizzle permutes pieces within the row, and hi / lo share the layout)
    const int r = tid - 64;
    uint32_t it = 0, rounds = 0;
    for (int i = blockIdx.x; i < items && !S.abort; i += gridDim.x) {
      bool ok = true;
      for (int k = 0; k < kblocks; ++k, ++it) {
        const int s = it % STAGES;
        if (!wait_or_abort(&S.full[s], (it / STAGES) & 1, S, err)) {
          ok = false;
          break;
        }
        float4* hi = reinterpret_cast<float4*>(smem + s * STAGE_BYTES + r * 128);
        float4* lo = reinterpret_cast<float4*>(smem + s * STAGE_BYTES + TILE + r * 128);
        if (a_cols) {
          // compact A (K < 32 columns, rows packed at K * 4 bytes): read this row's pieces, wait
          // until all 128 rows are read (the swizzled rows overwrite the packed data), then write
          // logical piece j of row r at piece position j ^ (r % 8), zeros past K
          const float4* src = reinterpret_cast<const float4*>(smem + s * STAGE_BYTES + r * a_cols * 4);
          float4 x[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) x[j] = 4 * j < a_cols ? src[j] : make_float4(0.f, 0.f, 0.f, 0.f);
          mbar_arrive(&S.rd);  // a bounded barrier over the 128 split threads
          if (!wait_or_abort(&S.rd, (rounds++) & 1, S, err)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int q = j ^ (r & 7);
            const float4 h = make_float4(tf32_rna(x[j].x), tf32_rna(x[j].y), tf32_rna(x[j].z), tf32_rna(x[j].w));
            hi[q] = h;
            lo[q] = make_float4(x[j].x - h.x, x[j].y - h.y, x[j].z - h.z, x[j].w - h.w);
          }
          fence_proxy_async();
          mbar_arrive(&S.split[s]);
          continue;
        }
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const int j = (jj + r) & 7;  // rotate the piece order by row: 8 rows hit 8 bank groups
          const float4 x = hi[j];
          const float4 h = make_float4(tf32_rna(x.x), tf32_rna(x.y), tf32_rna(x.z), tf32_rna(x.w));
          hi[j] = h;
          lo[j] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
        }
        fence_proxy_async();
        mbar_arrive(&S.split[s]);
      }
      if (!ok) break;
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (rows of the tile); warps 6-9
    // (group 0) take columns 0-63, warps 10-13 (group 1) columns 64-127.  Both 32-column
    // chunks of a partial sum are read and added before the accumulator is released; with the TMA
    // store each warp then stages a 32 x 32 block at a time in shared memory (128-byte
    // swizzle, conflict-free row writes) and one lane stores it, clipped at the matrix edges;
    // otherwise rows are stored directly.
    const int ew = warp - 6, sub = warp & 3, grp = ew >> 2;
    unsigned char* stg = smem + STAGES * STAGE_BYTES + ew * STAGING;
    const int r = sub * 32 + lane;  // tile row of this thread
    const bool vec = (ldc % 4) == 0 && (reinterpret_cast<uintptr_t>(C) % 16) == 0;
    const int partials = MULTI ? (kblocks + KB_PARTIAL - 1) / KB_PARTIAL : 1;
    const int nc = bn - grp * 64 >= 64 ? 2 : (bn - grp * 64 > 0 ? (bn - grp * 64 + 31) / 32 : 0);  // uniform
    uint32_t t = 0;
    bool ok = true;
    for (int i = blockIdx.x; ok && i < items && !S.abort; i += gridDim.x) {
      const int m0 = (i / ntiles) * BM, n0 = (i % ntiles) * bn;
      if constexpr (!MULTI) {
        // one partial sum: 32-column chunks q = grp, grp + 2, ... straight from TMEM to the
        // stores; the accumulator is released after the last chunk
        const uint32_t a = t & 1;
        if (!wait_or_abort(&S.accf[a], (t >> 1) & 1, S, err)) break;
        fence_after();
        const int nch = (bn + 31) / 32;
        for (int q = grp; q < nch; q += 2) {
          float w[32];
          tmem_ld32x32b_x32(tb + ((uint32_t)(sub * 32) << 16) + a * BNT + q * 32, w);
          const int col0 = n0 + q * 32;
          if (use_tma_store) {
            if (lane == 0) bulk_wait_read_all();  // the previous store has read the staging block
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<float4*>(stg + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                  make_float4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0 && m0 + sub * 32 < M && col0 < N) {
              tma_store_2d(&mc, stg, col0, m0 + sub * 32);
              bulk_commit_group();
            }
          } else {
            const int row = m0 + r;
            float* crow = C + (int64_t)row * ldc;
            if (row < M && col0 < N) {
              if (vec && col0 + 32 <= N) {
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  *reinterpret_cast<float4*>(crow + col0 + 4 * j) =
                      make_float4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
              } else {
                for (int j = 0; j < 32; ++j)
                  if (col0 + j < N) crow[col0 + j] = w[j];
              }
            }
          }
        }
        fence_before();
        mbar_arrive(&S.acce[a]);
        ++t;
        continue;
      }
      float v[2][32];
      for (int p = 0; p < partials; ++p, ++t) {
        const uint32_t a = t & 1;
        if (!wait_or_abort(&S.accf[a], (t >> 1) & 1, S, err)) {
          ok = false;
          break;
        }
        fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          if (c < nc) {
            float w[32];
            tmem_ld32x32b_x32(tb + ((uint32_t)(sub * 32) << 16) + a * BNT + grp * 64 + c * 32, w);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[c][j] = (MULTI && p) ? v[c][j] + w[j] : w[j];
          }
        }
        fence_before();
        mbar_arrive(&S.acce[a]);  // the accumulator is free for the next partial sum
      }
      if (!ok) break;
      if (use_tma_store) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          if (c >= nc) break;
          if (lane == 0) bulk_wait_read_all();  // the previous store has read the staging block
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(stg + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                make_float4(v[c][4 * j], v[c][4 * j + 1], v[c][4 * j + 2], v[c][4 * j + 3]);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0 && m0 + sub * 32 < M && n0 + grp * 64 + c * 32 < N) {
            tma_store_2d(&mc, stg, n0 + grp * 64 + c * 32, m0 + sub * 32);
            bulk_commit_group();
          }
        }
      } else {
        const int row = m0 + r;
        float* crow = C + (int64_t)row * ldc;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int col0 = n0 + grp * 64 + c * 32;
          if (c < nc && row < M && col0 < N) {
            if (vec && col0 + 32 <= N) {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                *reinterpret_cast<float4*>(crow + col0 + 4 * j) =
                    make_float4(v[c][4 * j], v[c][4 * j + 1], v[c][4 * j + 2], v[c][4 * j + 3]);
            } else {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < N) crow[col0 + j] = v[c][j];
            }
          }
        }
      }
    }
    if (use_tma_store && lane == 0) bulk_wait_all();
  }
  __syncthreads();
  fence_after();
  if (warp == 1) tmem_dealloc(tb, 2 * BNT);
}

__global__ void split_tf32_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ hi,
                                  float* __restrict__ lo) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i], h = tf32_rna(v);
    hi[i] = h;
    lo[i] = v - h;
  }
}

// box_cols = BK: 128-byte swizzled k blocks; box_cols < BK: whole rows of a narrow matrix,
// packed (no swizzle), rearranged by the split warps.
int make_map(CUtensorMap* m, const float* base, int64_t rows, int64_t cols, int64_t ld, int box_rows = BM,
             int box_cols = BK) {
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  return tma::encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box,
                     box_cols == BK ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, "ssla_gemm_f32_tc");
}

}  // namespace
}  // namespace gemm
}  // namespace ssla

using namespace ssla;

extern "C" int ssla_split_tf32(const float* x, int64_t n, float* hi, float* lo, ssla_stream_t stream) {
  SSLA_CHECK_ARG(n >= 0, "ssla_split_tf32: bad size");
  if (n == 0) return SSLA_OK;
  SSLA_CHECK_ARG(x && hi && lo, "ssla_split_tf32: null pointer");
  const int64_t blocks = (n + 255) / 256;
  gemm::split_tf32_kernel<<<(unsigned)(blocks < 148 * 8 ? blocks : 148 * 8), 256, 0, (cudaStream_t)stream>>>(x, n, hi,
                                                                                                            lo);
  SSLA_CHECK_LAUNCH("ssla_split_tf32");
  return SSLA_OK;
}

extern "C" int ssla_gemm_f32_tc(const float* A, int64_t M, int64_t K, int64_t lda, const float* B_hi,
                                const float* B_lo, int64_t N, int64_t ldb, float* C, int64_t ldc, int* err,
                                ssla_stream_t stream) {
  SSLA_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "ssla_gemm_f32_tc: bad sizes");
  if (M == 0 || N == 0) return SSLA_OK;
  SSLA_CHECK_ARG(K > 0 && A && B_hi && B_lo && C && err, "ssla_gemm_f32_tc: null pointer or K = 0");
  SSLA_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "ssla_gemm_f32_tc: sizes exceed 2^31");
  SSLA_CHECK_ARG(lda >= K && ldb >= K && ldc >= N, "ssla_gemm_f32_tc: leading dimensions smaller than the rows");
  SSLA_CHECK_ARG(lda % 4 == 0 && ldb % 4 == 0 && reinterpret_cast<uintptr_t>(A) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(B_hi) % 16 == 0 && reinterpret_cast<uintptr_t>(B_lo) % 16 == 0,
                 "ssla_gemm_f32_tc: A and B need 16-byte aligned rows (lda, ldb multiples of 4)");
  // kernel shape: K beyond one partial sum -> 128-column tiles, 3 stages (partial sums held in
  // registers); otherwise N above 128 -> up to 256-column tiles (N split evenly), 2 stages
  const bool multi = K > (int64_t)gemm::KB_PARTIAL * gemm::BK;
  const bool wide = !multi && N > gemm::BN;
  int bn;
  if (wide) {
    const int64_t nt = (N + 255) / 256;
    bn = (int)(((N + nt - 1) / nt + 31) / 32 * 32);  // whole 32-column epilogue chunks: none spills into the next tile
  } else {
    bn = N >= gemm::BN ? gemm::BN : (int)((N + 15) / 16 * 16);
  }
  CUtensorMap ma, mbh, mbl, mc;
  int rc;
  const int brows = wide ? 256 : gemm::BN;
  // A narrower than one k block (the first layers' 12 / 24 features): whole packed rows per
  // copy instead of 32-column boxes that read mostly outside the matrix
  const int a_cols = K < gemm::BK ? (int)K : 0;
  // B rows padded to exactly one k block (ldb == 32 with K < 32, the layout the projection
  // weights are prepared in) are read whole: their extra columns meet the zero columns of A and
  // must only be finite.  Any other ldb reads K columns and lets TMA fill the rest with zeros.
  const int64_t bcols = (K < gemm::BK && ldb == gemm::BK) ? gemm::BK : K;
  if ((rc = gemm::make_map(&ma, A, M, K, lda, gemm::BM, a_cols ? a_cols : gemm::BK)) || (rc = gemm::make_map(&mbh, B_hi, N, bcols, ldb, brows)) ||
      (rc = gemm::make_map(&mbl, B_lo, N, bcols, ldb, brows)))
    return rc;
  // output through TMA stores (32 x 32 boxes) when its rows are 16-byte aligned
  const int use_tma_store = (ldc % 4 == 0 && reinterpret_cast<uintptr_t>(C) % 16 == 0) ? 1 : 0;
  memset(&mc, 0, sizeof(mc));
  if (use_tma_store && (rc = gemm::make_map(&mc, C, M, N, ldc, 32))) return rc;
  auto kern = multi ? gemm::gemm_tf32x3_kernel<true, 128, 3>
                    : (wide ? gemm::gemm_tf32x3_kernel<false, 256, 2> : gemm::gemm_tf32x3_kernel<false, 128, 3>);
  const size_t smem = multi || !wide ? gemm::smem_bytes(128, 3) : gemm::smem_bytes(256, 2);
  const int variant = multi ? 0 : (wide ? 1 : 2);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    set_error("ssla_gemm_f32_tc: device query failed");
    return SSLA_ERR_CUDA;
  }
  // the shared-memory opt-in is a per-device function attribute: set once per (device, variant)
  static bool ready[64][3] = {};
  if (dev >= 64 || !ready[dev][variant]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
      set_error("ssla_gemm_f32_tc: cannot reserve %zu bytes of shared memory", smem);
      return SSLA_ERR_CUDA;
    }
    if (dev < 64) ready[dev][variant] = true;
  }
  const int64_t items = ((M + gemm::BM - 1) / gemm::BM) * ((N + bn - 1) / bn);
  const unsigned grid = (unsigned)(items < sms ? items : sms);
  kern<<<grid, gemm::NT, smem, (cudaStream_t)stream>>>(ma, mbh, mbl, mc, use_tma_store, (int)M, (int)N, (int)K, bn, a_cols,
                                                      C, ldc, err);
  SSLA_CHECK_LAUNCH("ssla_gemm_f32_tc");
  return SSLA_OK;
}
