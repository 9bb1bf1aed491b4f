/*
 * ssla_b200 — C ABI of the B200 (sm_100a) kernels behind SSLA's gated-linear-attention
 * hot path.  Every entry point takes plain device pointers, element counts and a CUDA
 * stream, enqueues its kernels on that stream without synchronising, and returns an
 * int status (SSLA_OK or a negative code; ssla_last_error() gives the message).
 *
 * Layouts follow the reference operators: packed variable-length sequences
 * [T_total, H, D] with int64 cu_seqlens[N+1] (ops/gla/chunk.py:1131-1150,
 * ops/common/scan.py:148-158).  All tensors are dense row-major (contiguous).
 * The reference is pure Python/Triton; each declaration names the reference
 * function whose kernels it replaces (path within the haohq19/ssla project).
 */
#ifndef SSLA_B200_H_
#define SSLA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ssla_stream_t; /* == cudaStream_t */

/* status codes */
#define SSLA_OK 0
#define SSLA_ERR_INVALID_ARG -1
#define SSLA_ERR_CUDA -2
#define SSLA_ERR_WORKSPACE -3
#define SSLA_ERR_UNSUPPORTED -4

/* element type codes */
#define SSLA_F32 0
#define SSLA_BF16 1
#define SSLA_F16 2

/* ------------------------------------------------------------------ library */
int ssla_abi_version(void);
/* Message of the last failing call on this host thread ("" if none). */
const char* ssla_last_error(void);

/* ------------------------------------------------------------------ scan
 * h_t = g_t * h_{t-1} + u_t per channel, h_{-1} = 0, over each sequence of u,g [T,C].
 * Replaces ops/common/scan.py:11-43 (sequential_scan_fwd) and SequentialScan.forward
 * (ops/common/scan.py:92-114).  fp32 arithmetic, one rounding per multiply and add.
 */
int ssla_scan_fwd(const void* u, int dtype_u, const void* g, int dtype_g, void* h, int dtype_h,
                  const int64_t* cu_seqlens, int64_t n_seqs, int64_t T, int64_t C,
                  ssla_stream_t stream);
/* Reverse pass: du = dh, dg = dh * h_{t-1}, dh_{t-1} = dh_t * g_t (+ do_{t-1}).
 * Replaces ops/common/scan.py:46-86 (sequential_scan_bwd) and SequentialScan.backward
 * (ops/common/scan.py:116-137). */
int ssla_scan_bwd(const void* dout, int dtype_do, const void* g, int dtype_g, const void* h,
                  int dtype_h, void* du, int dtype_du, void* dg, int dtype_dg,
                  const int64_t* cu_seqlens, int64_t n_seqs, int64_t T, int64_t C,
                  ssla_stream_t stream);

/* ------------------------------------------------------------------ scalar GLA
 * Per-channel scalar state: S_t = exp(g_t) S_{t-1} + k_t v_t, o_t = scale q_t S_t.
 * q,k,v,g,o [T,H]; h0/ht [N,H] fp32 (nullable).  Replaces chunk_gla_scalar
 * (ops/gla/chunk_scalar.py:1044-1092) with the recurrence of
 * ops/gla/naive_scalar.py:7-66. */
int ssla_gla_scalar_fwd(const void* q, const void* k, const void* v, const void* g, int dtype,
                        int dtype_g, const int64_t* cu_seqlens, int64_t n_seqs, int64_t T,
                        int64_t H, float scale, const float* h0, void* o, float* ht,
                        ssla_stream_t stream);
/* dq,dk,dv in `dtype`, dg fp32 [T,H], dh0 fp32 [N,H] (nullable), dht nullable.
 * Replaces ChunkGLAScalarFunction.backward (ops/gla/chunk_scalar.py:1025-1041). */
int ssla_gla_scalar_bwd(const void* q, const void* k, const void* v, const void* g, int dtype,
                        int dtype_g, const int64_t* cu_seqlens, int64_t n_seqs, int64_t T,
                        int64_t H, float scale, const float* h0, const void* dout,
                        const float* dht, void* dq, void* dk, void* dv, float* dg, float* dh0,
                        ssla_stream_t stream);

/* ------------------------------------------------------------------ recurrent GLA
 * Token-by-token GLA with a [K,V] fp32 state per (sequence, head):
 *   S_t = diag(exp(g_t)) S_{t-1} + k_t v_t^T,   o_t = (scale q_t)^T S_t.
 * q,k,g [T,H,K], v,o [T,H,V] (o in `dtype`); h0/ht [N,H,K,V] fp32, each nullable.
 * Semantics of naive_gla_recurrent (ops/gla/naive.py:50-111); exposed as
 * fused_recurrent_gla with chunk_gla's signature (ops/gla/chunk.py:1120-1129). */
int ssla_recurrent_gla_fwd(const void* q, const void* k, const void* v, const void* g, int dtype,
                           int dtype_g, const int64_t* cu_seqlens, int64_t n_seqs, int64_t T,
                           int64_t H, int64_t K, int64_t V, float scale, const float* h0,
                           void* o, float* ht, ssla_stream_t stream);

/* ------------------------------------------------------------------ chunked GLA
 * chunk_gla forward / backward (ops/gla/chunk.py:906-1053, ops/common/chunk_h.py:242-347).
 * Layout: q,k,g [T,H,K]; v,o,do [T,H,V]; h0,ht,dht,dh0 [N,H,K,V] fp32 (nullable).
 * `states` is a caller-allocated device buffer of ssla_chunk_gla_states_bytes() that the
 * forward fills (the call's chunk table, which 64-token chunks the exact kernels handle, and
 * the state at every chunk start: fp32, plus the 16-bit scaled copy the tensor-core kernels
 * read for 16-bit inputs with K = V = 64) and the backward reads; it replaces the reference's
 * cached chunk indices (ops/utils/index.py:69-86) and saved h (ops/gla/chunk.py:933).
 * `workspace` is caller-allocated device scratch of ssla_chunk_gla_workspace_bytes() (the
 * forward needs only a prefix of it).  dq,dk,dv are written in `dtype`; dg in fp32 (the
 * reference returns dg in fp32, ops/gla/chunk.py:1116).  K, V <= 64. */
int64_t ssla_chunk_gla_max_chunks(int64_t n_seqs, int64_t T);
size_t ssla_chunk_gla_states_bytes(int64_t n_seqs, int64_t T, int64_t H, int64_t K, int64_t V,
                                   int dtype, int dtype_g);
size_t ssla_chunk_gla_workspace_bytes(int64_t n_seqs, int64_t T, int64_t H, int64_t K,
                                      int64_t V, int dtype, int dtype_g);
int ssla_chunk_gla_fwd(const void* q, const void* k, const void* v, const void* g, int dtype,
                       int dtype_g, const int64_t* cu_seqlens, int64_t n_seqs, int64_t T,
                       int64_t H, int64_t K, int64_t V, float scale, const float* h0, void* o,
                       float* ht, void* states, size_t states_bytes, void* workspace,
                       size_t workspace_bytes, ssla_stream_t stream);
int ssla_chunk_gla_bwd(const void* q, const void* k, const void* v, const void* g, int dtype,
                       int dtype_g, const int64_t* cu_seqlens, int64_t n_seqs, int64_t T,
                       int64_t H, int64_t K, int64_t V, float scale, const void* states,
                       size_t states_bytes, const void* dout, const float* dht, void* dq,
                       void* dk, void* dv, float* dg, float* dh0, void* workspace,
                       size_t workspace_bytes, ssla_stream_t stream);

/* chunk_gla forward that allocates nothing: no counterpart in the reference.  For callers
 * that cannot call cudaMalloc (a runtime that owns every allocation and hands the library
 * only input/output buffers, a pool that has claimed all device memory).  Same arguments
 * and results as ssla_chunk_gla_fwd minus `states` and `workspace`: the intermediates live
 * in a fixed 64 MiB scratch array built into the library (held on every GPU that loads it
 * until exit); shapes needing more return SSLA_ERR_WORKSPACE.  The first call on each device
 * looks up the array's device address (make it before any stream capture).  All calls on a
 * device share the array, so calls that overlap on the GPU race: serialise them. */
int ssla_chunk_gla_fwd_noalloc(const void* q, const void* k, const void* v, const void* g,
                               int dtype, int dtype_g, const int64_t* cu_seqlens, int64_t n_seqs,
                               int64_t T, int64_t H, int64_t K, int64_t V, float scale,
                               const float* h0, void* o, float* ht, ssla_stream_t stream);

/* ------------------------------------------------------------------ pixel grouping
 * group_events (utils/farsecnn_utils.py:130-174, utils/async_utils.py:10-84) followed, with
 * keep_first, by the hot-pixel truncation of model_mos.py:173-209: events [B,Nmax,C] fp32 rows
 * <x, y, t, features...> with lengths [B] are grouped by (sample, pixel) in ascending id order,
 * events of a group in input order, the last max_per_px of each group kept, then the first
 * keep_first of those (pass INT64_MAX for no truncation).  Two calls with one host read
 * between: _count fills the workspace and writes totals[3] = {events, groups G, kept K} (int32,
 * device); _emit writes batch_id,h,w,lengths [G] int64 and time [K] int64, features [K,C-3]
 * fp32 (with dt_col >= 0 that feature column becomes the pixel delay of model_mos.py:190-200).
 * Requires B*H*W and B*Nmax below 2^31. */
size_t ssla_group_events_workspace_bytes(int64_t B, int64_t Nmax, int64_t H, int64_t W);
int ssla_group_events_count(const float* events, int64_t B, int64_t Nmax, int64_t C, const int64_t* lengths,
                            int64_t H, int64_t W, int64_t max_per_px, int64_t keep_first, void* workspace,
                            size_t workspace_bytes, int* totals, ssla_stream_t stream);
int ssla_group_events_emit(const float* events, int64_t B, int64_t Nmax, int64_t C, int64_t H, int64_t W,
                           int64_t max_per_px, int64_t keep_first, const void* workspace, int64_t G, int64_t K,
                           int dt_col, int64_t* batch_id, int64_t* h, int64_t* w, int64_t* lengths, int64_t* time,
                           float* features, ssla_stream_t stream);

/* ------------------------------------------------------------------ segments
 * Reductions of rows of src [R,C] into out [S,C] by a row->segment index [R] (int64).
 * Semantics of torch_scatter.scatter_max / scatter_mean / scatter_sum (dim=0) as called
 * by layers/sparse_pooling.py:33: max with argmax (smallest row index among ties,
 * R for empty segments, value 0 for empty segments); sum accumulated in fp32 in
 * ascending row order; mean = sum / max(count,1).  Deterministic, no atomics on data.
 *
 * Sorted path: `index` non-decreasing; `seg_offsets` [S+1] int64 is produced by
 * ssla_segment_offsets_sorted.  Unsorted path: ssla_segment_csr builds a CSR
 * (offsets + rows in ascending order per segment) from any index. */
int ssla_segment_offsets_sorted(const int64_t* index, int64_t R, int64_t S, int64_t* seg_offsets,
                                ssla_stream_t stream);
size_t ssla_segment_csr_workspace_bytes(int64_t R, int64_t S);
int ssla_segment_csr(const int64_t* index, int64_t R, int64_t S, int64_t* seg_offsets,
                     int64_t* rows, void* workspace, size_t workspace_bytes,
                     ssla_stream_t stream);
/* op: 0 = sum, 1 = mean, 2 = max.  rows == NULL means identity (sorted input).
 * arg (int64 [S,C]) is written for max when non-NULL. */
#define SSLA_REDUCE_SUM 0
#define SSLA_REDUCE_MEAN 1
#define SSLA_REDUCE_MAX 2
int ssla_segment_reduce(const void* src, int dtype, const int64_t* seg_offsets, const int64_t* rows,
                        int64_t R, int64_t S, int64_t C, int op, void* out, int64_t* arg,
                        ssla_stream_t stream);
/* out[r,:] = src[index[r],:]  (row gather; inverse of pooling, layers/sparse_pooling.py) */
int ssla_gather_rows(const void* src, int dtype, const int64_t* index, int64_t R, int64_t C,
                     void* out, ssla_stream_t stream);
/* Sparse pooling in one pass (layers/sparse_pooling.py:33 with pool_func = scatter_max and
 * scatter_mean, followed by the gather back pooled[index]): from an arbitrary row->segment
 * index, out_max [S,C] (+ arg [S,C], first maximal row, R for empty segments), out_mean [S,C]
 * and back [R,C] = out_max[index[r]], all with the semantics of ssla_segment_reduce above
 * (same results bit for bit).  Every output is optional (NULL); back needs out_max.
 * seg_offsets [S+1] (optional) receives the segment offsets of the counting sort.  Rows whose
 * index lies outside [0, S) are ignored and their back row is left untouched.  The one-pass
 * kernel handles C * element size a power-of-two multiple of 16 bytes up to 512 bytes with
 * 16-byte aligned buffers; other shapes run the CSR + reductions + gather sequence. */
size_t ssla_scatter_pool_workspace_bytes(int64_t R, int64_t S);
int ssla_scatter_pool(const void* src, int dtype, const int64_t* index, int64_t R, int64_t S, int64_t C,
                      void* out_max, int64_t* arg, void* out_mean, void* back, int64_t* seg_offsets,
                      void* workspace, size_t workspace_bytes, ssla_stream_t stream);
/* out[d,:] = sum over p with index[p]==d of src[p,:], fp32 sum in ascending p; zero rows
 * for unused d.  Deterministic replacement of utils/async_utils.py:243-264
 * (zeros(E,C).index_add_(0, idx, src)). */
size_t ssla_index_add_rows_workspace_bytes(int64_t P, int64_t D);
int ssla_index_add_rows(const void* src, int dtype, const int64_t* index, int64_t P, int64_t D,
                        int64_t C, void* out, void* workspace, size_t workspace_bytes,
                        ssla_stream_t stream);

/* ---------------------------------------------------------------- MoS layer (inference)
 * Fused per-patch work of MosAttention.forward (layers/mos_attention.py:97-136) for fp32:
 * for every patch sequence (cu_seqlens, events in time order) and patch event t,
 *   [q | v | g] = y[key[t], 0:3C];  h = sigmoid(g) * h + v;  z[dst[t], :] = q * h
 * y rows hold 3C floats (the q/v/g projections of the scattered event); C % 4 == 0. */
int ssla_mos_patch_scan_fwd(const float* y, const int64_t* key, const int64_t* dst,
                            const int64_t* cu_seqlens, int64_t n_seqs, int64_t C, float* z,
                            ssla_stream_t stream);
/* The same with the row indices formed from the routing's (src, pos) pair of each patch event:
 * key = src * P + pos (src when P == 1), dst = src * Pg + pos, or dst = t (the patch event's
 * own row) when Pg == 0; pos may be NULL when P == 1 and Pg <= 1 (pos = 0). */
int ssla_mos_patch_scan_routed_fwd(const float* y, const int64_t* src, const int64_t* pos, int64_t P, int64_t Pg,
                                   const int64_t* cu_seqlens, int64_t n_seqs, int64_t C, float* z,
                                   ssla_stream_t stream);
/* The same with the projection done in the kernel: [q | v | g] = w[pos[t]] @ x[src[t]], with
 * w [P, 3C, I] fp32 (the q/v/g projections folded into the per-position scatter weights) and
 * x [*, I] the layer input rows.  w must fit in shared memory
 * (ssla_mos_patch_scan_proj_smem_bytes(P, C, I) <= 200 KiB). */
size_t ssla_mos_patch_scan_proj_smem_bytes(int64_t P, int64_t C, int64_t I);
int ssla_mos_patch_scan_proj_fwd(const float* x, int64_t I, const float* w, int64_t P,
                                 const int64_t* src, const int64_t* pos, const int64_t* dst,
                                 const int64_t* cu_seqlens, int64_t n_seqs, int64_t C, float* z,
                                 ssla_stream_t stream);
/* out[M, N] (row stride ldo) = A[M, K] (row stride lda) @ B[K, N] (contiguous), fp32, for
 * skinny shapes (B must fit in 96 KiB of shared memory: ssla_rows_matmul_smem_bytes). */
size_t ssla_rows_matmul_smem_bytes(int64_t K, int64_t N);
int ssla_rows_matmul_f32(const float* A, int64_t M, int64_t K, int64_t lda, const float* B, int64_t N,
                         float* out, int64_t ldo, ssla_stream_t stream);
/* out = LayerNorm(x + r) * w + b over rows of C channels (r may be NULL); 1 <= C <= 1024.  Replaces the residual add + nn.LayerNorm closing MosAttention
 * and LinearAttention (layers/mos_attention.py:144, layers/linear_attention.py:100). */
int ssla_layernorm_residual_fwd(const float* x, const float* r, const float* w, const float* b,
                                int64_t rows, int64_t C, float eps, float* out, ssla_stream_t stream);

/* ---------------------------------------------------------------- event routing
 * Pixel groups -> receptive fields with each field's events in time order: the GPU form of
 * scatter_group_events_to_patch / gather_receptive_fields (utils/async_utils.py:125-240,
 * utils/farsecnn_utils.py:177-265).  Geometry: frame H x W, window kh x kw, stride sh x sw,
 * leading padding pt / pl, output oh x ow fields per sample, B samples.
 *   ssla_route_pixel_map:  map[(b*H + y)*W + x] = group id (map pre-filled with -1); groups
 *                          outside the frame are skipped and counted in *bad.
 *   ssla_route_groups_time_sorted: *bad = 1 if some group's times decrease.
 *   ssla_route_field_lengths: flen[b*oh*ow + f] = events in field f of sample b.
 *   ssla_route_compact_fields: the non-empty fields of flen [nf] in ascending order:
 *                    field_ids, lengths and event offsets field_off (each sized for nf, field_off
 *                    for nf + 1; the first F entries written, field_off[F] = total), and
 *                    stats[4] = {flags[0], flags[1], F, total events} (flags may be NULL: 0).
 *   ssla_route_fill: for the non-empty fields field_ids[F] (ascending) with output offsets
 *                    field_off[F+1]: src (event index), pos (window position) and time of every
 *                    routed event, ordered by (time, pos, event) within each field.
 * kh * kw <= 32. */
int ssla_route_pixel_map(const int64_t* batch_id, const int64_t* h, const int64_t* w, int64_t G,
                         int64_t B, int64_t H, int64_t W, int* map, int* bad, ssla_stream_t stream);
int ssla_route_groups_time_sorted(const int64_t* gstart, const int64_t* glen, const int64_t* gtime,
                                  int64_t G, int* bad, ssla_stream_t stream);
int ssla_route_field_lengths(const int* map, const int64_t* glen, int64_t B, int64_t H, int64_t W,
                             int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t pt, int64_t pl,
                             int64_t oh, int64_t ow, int64_t* flen, ssla_stream_t stream);
size_t ssla_route_compact_fields_workspace_bytes(int64_t nf);
int ssla_route_compact_fields(const int64_t* flen, int64_t nf, const int* flags, int64_t* field_ids,
                              int64_t* lengths, int64_t* field_off, int64_t* stats, void* workspace,
                              size_t workspace_bytes, ssla_stream_t stream);
int ssla_route_fill(const int* map, const int64_t* gstart, const int64_t* glen, const int64_t* gtime,
                    int64_t B, int64_t H, int64_t W, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                    int64_t pt, int64_t pl, int64_t oh, int64_t ow, const int64_t* field_ids,
                    const int64_t* field_off, int64_t F, int64_t* src, int64_t* pos, int64_t* time,
                    ssla_stream_t stream);

/* ---------------------------------------------------------------- detection post-processing
 * Batched greedy NMS (MosModel.postprocess_with_nms, model_mos.py:232-299; torchvision nms on
 * class-offset boxes, model_mos.py:20-29): for each of B images, the candidates (score >= conf
 * when filtering) sorted by descending score (ascending index among equal scores), a box is
 * kept unless an earlier kept box has IoU > iou_thr with it; at most max_det kept.
 * boxes [B, N, 4] fp32 xyxy (class offsets applied), scores [B, N]; keep [B, max_det] anchor
 * indices in score order, count [B].  N <= 4096. */
size_t ssla_batched_nms_workspace_bytes(int64_t B);
int ssla_batched_nms(const float* boxes, const float* scores, int64_t B, int64_t N, int filtering,
                     float conf, float iou_thr, int64_t max_det, int64_t* keep, int64_t* count,
                     void* workspace, size_t workspace_bytes, ssla_stream_t stream);

/* ---------------------------------------------------------------- event-stream input
 * Prophesee .dat (Event2D) payloads resident in device memory: `words` holds events as pairs of
 * 32-bit words (t, packed x | y << 14 | p << 28; utils/io/dat_events_tools.py:14, :40-44);
 * recording b of a batch starts at event rec_start[b] and has rec_count[b] events.
 * ssla_dat_window_ranges replaces PSEELoader.seek_time(t_end - window) followed by
 * load_delta_t(window + 1) (utils/io/psee_loader.py:109-219, as called by
 * dataset/gen1.py:190-193): range [B, 2] gets each sample's [begin, end) event range (relative
 * to rec_start), lengths [B] its size.  term_criterion is seek_time's bisection stop (100000).
 * ssla_dat_decode_windows replaces the Gen1 collation (model_base.py:82-117): out [B, Nmax, 4]
 * fp32 rows <x, y, t, 2p - 1>, rows past a sample's length (0, 0, 0, -1).  words 8-byte and
 * out 16-byte aligned. */
int ssla_dat_window_ranges(const uint32_t* words, const int64_t* rec_start, const int64_t* rec_count,
                           const int64_t* t_end, int64_t B, int64_t window, int64_t term_criterion,
                           int64_t* range, int64_t* lengths, ssla_stream_t stream);
int ssla_dat_decode_windows(const uint32_t* words, const int64_t* rec_start, const int64_t* range,
                            int64_t B, int64_t Nmax, float* out, ssla_stream_t stream);

/* ---------------------------------------------------------------- fp32 GEMM on tensor cores
 * C[M, N] = A[M, K] * B[N, K]^T in fp32 by split TF32 (A B^T ~ Ahi Bhi^T + Ahi Blo^T + Alo Bhi^T,
 * hi = TF32 rounding, lo = remainder; relative error near 2^-21 per product), for the MoS
 * layers' per-position projections (layers/mos_attention.py:148-167, fp32 F.linear there).
 * B is given pre-split (ssla_split_tf32 of the fp32 weights, same [N, ldb] layout).  A, B_hi,
 * B_lo 16-byte aligned with lda, ldb multiples of 4; *err (device int) is set to 1 if a
 * pipeline wait timed out.  With K < 32 and ldb == 32, B rows are read whole (faster copies):
 * the padding columns K..31 must be finite (zero, as ssla_b200's weight preparation writes);
 * any other ldb reads only K columns. */
int ssla_split_tf32(const float* x, int64_t n, float* hi, float* lo, ssla_stream_t stream);
int ssla_gemm_f32_tc(const float* A, int64_t M, int64_t K, int64_t lda, const float* B_hi, const float* B_lo,
                     int64_t N, int64_t ldb, float* C, int64_t ldc, int* err, ssla_stream_t stream);

/* Number of bounded shared-memory barrier waits in the tensor-core chunk kernels that gave up
 * since the last reset (synchronous device read; 0 in a healthy run).  A CTA whose wait gave
 * up writes NaN into the outputs of the items it still had, so such results are visible
 * without this read; a nonzero count says why. */
int ssla_chunk_gla_tc_timeouts(int reset, unsigned* count);

#ifdef __cplusplus
}
#endif

#endif /* SSLA_B200_H_ */
