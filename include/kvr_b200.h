/*
 * kvr_b200.h — C ABI of the B200-native compressed-KV hot path.
 *
 * Plain pointers and sizes only: every pointer named "device" is a CUDA
 * device pointer on the current device, every call is asynchronous on the
 * given stream (NULL = legacy default stream) and returns KVR_OK or a KVR_E*
 * code; kvr_last_error() then holds a one-line message for the calling host
 * thread.  No entry point allocates device memory: callers own all buffers,
 * including the workspaces whose sizes the *_workspace_bytes() helpers report.
 * Workspaces must be zero-filled once before their first use; every
 * successful call leaves them zero-filled again (their counters self-reset).
 * A call that returned KVR_ETIMEOUT may leave them dirty: zero them again.
 *
 * Reference interfaces replaced (paths inside Misaka477/RINA-1bit-KV):
 *   modules/kvr_cuda.cu:53-77 / kvr_cuda.py:20-26     -> kvr_compute_scores
 *   modules/kvr_retrieval.py:95-122  (calibrate)       -> kvr_absmax_scales
 *   modules/kvr_retrieval.py:162-207 (append/batch)    -> kvr_int4w_encode_k, kvr_int4w_encode_vres
 *   modules/kvr_retrieval.py:265-289 (all scores)      -> kvr_int4w_token_scores
 *   modules/kvr_retrieval.py:291-315 (chunk scores)    -> kvr_int4w_chunk_scores
 *   modules/kvr_retrieval.py:370-392 (top-k)           -> kvr_topk_rows
 *   modules/kvr_retrieval.py:394-412 (gather, V recon) -> kvr_int4w_gather, kvr_int4w_vpredict(_prepare),
 *                                                         kvr_int4w_vres_add
 *   modules/kvr_retrieval.py:248-263, 332-367 (attractor branch) -> kvr_int4w_attractor_select
 *   modules/kvr_window.py:19-41      (ring append)     -> kvr_window_write
 *   modules/kvr_generator.py:78-98   (RoPE + store update of a decode step) -> kvr_decode_store_update,
 *                                                         kvr_sd1_decode_step_update (fused with the step)
 *   modules/kvr_window.py:43-69, kvr_hook.py:274-282,
 *   modules/kvr_triton.py:42-104     (attention)       -> kvr_decode_attn
 *   (no reference counterpart: the 1-bit sd1 codec)    -> kvr_sd1_*, kvr_transform, kvr_lse_merge
 */
#ifndef KVR_B200_H
#define KVR_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KVR_API __attribute__((visibility("default")))
#else
#define KVR_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *kvr_stream_t; /* same type as cudaStream_t */

enum kvr_status {
  KVR_OK = 0,
  KVR_EINVAL = 1,   /* bad argument (shape, dtype, alignment, null pointer) */
  KVR_ECUDA = 2,    /* a CUDA runtime call or kernel launch failed */
  KVR_ENOTSUP = 3,  /* valid but unsupported configuration (e.g. head_dim != 128) */
  KVR_ETIMEOUT = 4  /* a bounded device-side wait gave up (see kvr_sd1_* notes) */
};

enum kvr_dtype { KVR_F32 = 0, KVR_F16 = 1, KVR_BF16 = 2 };
enum kvr_transform_kind { KVR_HADAMARD = 0, KVR_DCT = 1 };

/* One-line description of the last failure on this host thread ("" if none). */
KVR_API const char *kvr_last_error(void);
/* ABI version: (major << 16) | minor. */
KVR_API int kvr_abi_version(void);

/* ---------------------------------------------------------------- int4w ----
 * The reference-faithful codec: int4 K_pre codes with a per-(head, channel)
 * absmax scale, V predicted from K through W plus an int2 per-head residual.
 * Layouts follow modules/kvr_retrieval.py: K (n, n_kv, d), packed K
 * (n, n_kv, d/2) uint8, packed residual (n, n_kv, d/4) uint8.
 */

/* calibrate()'s k_scales = clamp(max_t |x[t, c]|, min=clamp_min) over n rows of
 * `cols` columns (kvr_retrieval.py:99).  x is (n, cols) with row stride `cols`. */
KVR_API int kvr_absmax_scales(const void *x, int dtype, int64_t n, int64_t cols, float clamp_min,
                      float *out /* device (cols) */, kvr_stream_t stream);

/* kq = clamp(rint(k / (2*s/16)), -8, 7), packed two per byte, even element in
 * the high nibble (kvr_retrieval.py:69-72, 167-171, 190-193).  k is
 * (n, n_kv, d) with token stride `tok_stride` elements. */
KVR_API int kvr_int4w_encode_k(const void *k, int dtype, int64_t n, int n_kv, int d, int64_t tok_stride,
                       const float *k_scales /* (n_kv, d) */, uint8_t *k_packed /* (n, n_kv, d/2) */,
                       kvr_stream_t stream);

/* vrq = clamp(rint((v - v_pred) / (2*vr/4)), -2, 1), packed four per byte,
 * element 0 in bits 7-6 (kvr_retrieval.py:80-83, 173-180, 196-203).
 * v (n, n_kv, d) of `dtype`; v_pred (n, n_kv, d) fp32 contiguous. */
KVR_API int kvr_int4w_encode_vres(const void *v, int dtype, const float *v_pred, int64_t n, int n_kv, int d,
                          const float *vr_scales /* (n_kv) */, uint8_t *vr_packed /* (n, n_kv, d/4) */,
                          kvr_stream_t stream);

/* Drop-in for the reference's native score kernel (kvr_cuda.cu:9-49, 53-77):
 * interleaved-pair RoPE from (n_stored, d/2) cos/sin tables, dot with the
 * pre-averaged q, divided by sqrt(d).  scores (n_stored, n_kv) fp32,
 * bit-identical to the reference kernel (same per-element rounding order).
 * d in {64, 128, 256}; every pointer 16-byte aligned. */
KVR_API int kvr_compute_scores(const float *q_avg /* (n_kv, d) */, const uint8_t *k_pack, const float *k_scales,
                       const float *cos_tbl, const float *sin_tbl, int n_kv, int d, int64_t n_stored,
                       float *scores, kvr_stream_t stream);

/* compute_all_scores (kvr_retrieval.py:265-289): cosine between the GQA-group
 * mean of the post-RoPE query q (n_q, d) fp32 and the rotate_half-RoPE'd
 * dequantised K of every stored token (position = token index); NaN -> -inf.
 * cos/sin are (max_pos, d) rows with row stride `rope_stride`; if
 * `rope_halves_equal` is nonzero the kernel reads only the first d/2 columns
 * (valid for HF tables, whose halves are duplicated).  Output is HEAD-MAJOR:
 * scores[h * score_stride + t]. */
KVR_API int kvr_int4w_token_scores(const float *q, int n_q, const uint8_t *k_packed, const float *k_scales,
                           const float *cos_tbl, const float *sin_tbl, int64_t rope_stride,
                           int rope_halves_equal, int n_kv, int d, int64_t n_stored, float *scores,
                           int64_t score_stride, kvr_stream_t stream);

/* compute_chunk_scores (kvr_retrieval.py:291-315): cosine against the mean of
 * each full chunk of `chunk` RoPE'd tokens (the partial tail is dropped).
 * Output head-major scores[h * score_stride + c], c < n_stored / chunk. */
KVR_API int kvr_int4w_chunk_scores(const float *q, int n_q, const uint8_t *k_packed, const float *k_scales,
                           const float *cos_tbl, const float *sin_tbl, int64_t rope_stride,
                           int rope_halves_equal, int n_kv, int d, int64_t n_stored, int chunk,
                           float *scores, int64_t score_stride, kvr_stream_t stream);

/* Per-row top-k (kvr_retrieval.py:379, 391-392) over `rows` rows of `n`
 * contiguous fp32 scores (row r at scores + r * row_stride).  Entries with
 * index in [ex_start, ex_end) and NaN count as -inf, -0.0 equals +0.0.
 * Order: score descending, then index ascending (deterministic in place of
 * torch.topk's unspecified tie order).  k must be <= n and <= 4096.
 * Writes idx[r * out_row_stride + j * out_elem_stride] (int64) and, if vals is
 * not NULL, the scores at the same offsets. */
KVR_API int kvr_topk_rows(const float *scores, int rows, int64_t n, int64_t row_stride, int k,
                  int64_t ex_start, int64_t ex_end, int64_t *idx, float *vals,
                  int64_t out_row_stride, int64_t out_elem_stride, kvr_stream_t stream);

/* compute_all_scores + exclusion + torch.topk of the token branch
 * (kvr_retrieval.py:265-289, 389-392) in one call: the cosine scores of
 * kvr_int4w_token_scores, a per-head histogram of them, the rows split around
 * the bin of the k-th largest score by many CTAs, and the exact top k (score desc, index asc; excluded tokens and NaN
 * as -inf) per head.  idx (k, n_kv) int64, rows sorted by score.  The
 * workspace (kvr_int4w_token_topk_workspace_bytes) must be zero-filled once;
 * the call leaves it ready for the next one.  n_kv <= 8, d = 128, k <= 4096. */
KVR_API size_t kvr_int4w_token_topk_workspace_bytes(int n_kv, int64_t n_stored, int k);
KVR_API int kvr_int4w_token_topk(const float *q, int n_q, const uint8_t *k_packed, const float *k_scales,
                                 const float *cos_tbl, const float *sin_tbl, int64_t rope_stride, int rope_halves_equal,
                                 int n_kv, int d, int64_t n_stored, int k, int64_t ex_start, int64_t ex_end,
                                 int64_t *idx, void *workspace, size_t workspace_bytes, kvr_stream_t stream);

/* Gather for V reconstruction and K re-rotation (kvr_retrieval.py:394-412).
 * top (k, n_kv) int64 token indices.  Writes
 *   ret_k (k, n_kv, d) fp32 : RoPE(deq K[top[i,h], h]) at position top[i,h];
 *   x     (n_kv, k, n_kv*d) fp32 : deq K_pre of ALL heads of token top[i,h]
 *                                  minus K_mean (input of a library V-predict
 *                                  GEMM; NULL skips it, k_mean may then be NULL).
 * count (optional, device int32): only rows i < *count are written. */
KVR_API int kvr_int4w_gather(const uint8_t *k_packed, const float *k_scales, const int64_t *top, int k, int n_kv,
                     int d, const float *cos_tbl, const float *sin_tbl, int64_t rope_stride,
                     const float *k_mean /* (n_kv*d) */, float *ret_k, float *x, const int32_t *count,
                     kvr_stream_t stream);

/* V reconstruction of the selected tokens on the tensor cores
 * (kvr_retrieval.py:131-134, 394-402): ret_v[i, h, :] = fp16(W[h] . (deq K[t] -
 * K_mean) + V_mean[h] + int2 residual[t, h] * (2*vr_scales[h]/4)),
 * t = top[i, h], contracting over all n_kv*d channels of token t straight from
 * its packed int4 codes.  w3/unscale/bias come from kvr_int4w_vpredict_prepare
 * (once per calibration): W' = W * diag(step) split into fp16 hi + lo parts
 * with a power-of-two scale per output row (fp32-level accuracy), stored in
 * the kernel's tensor-core operand layout (opaque to callers).
 * count (optional, device int32): only rows i < *count are written.  d = 128,
 * n_kv <= 8; k_packed, w3, vr_packed and ret_v 16-byte aligned. */
KVR_API size_t kvr_int4w_vpredict_weights_bytes(int n_kv, int d);
KVR_API int kvr_int4w_vpredict_prepare(const float *W /* (n_kv*d, n_kv*d) */, const float *k_mean,
                                       const float *v_mean, const float *k_scales, int n_kv, int d, void *w3,
                                       float *unscale /* (n_kv*d) */, float *bias /* (n_kv*d) */,
                                       kvr_stream_t stream);
KVR_API int kvr_int4w_vpredict(const uint8_t *k_packed, const int64_t *top, const int32_t *count, int k, int n_kv,
                               int d, const void *w3, const float *unscale, const float *bias,
                               const uint8_t *vr_packed, const float *vr_scales, uint16_t *ret_v /* fp16 */,
                               kvr_stream_t stream);
/* Synchronises `stream`, then reads and clears the V-predict kernel's error
 * word: KVR_ETIMEOUT if a bounded device-side wait gave up since the last call. */
KVR_API int kvr_int4w_vpredict_status(kvr_stream_t stream);

/* Attractor branch of retrieve_topk (kvr_retrieval.py:248-263, 332-367)
 * with no host sync: head-0 group-mean query vs the centroids (n_attractors,
 * d), the top_a basins, the top 16 tokens of each basin by head-0 cosine of
 * the re-rotated dequantised K (a basin's tokens: the t < n_labelled with
 * labels[t] == basin), the ascending union minus [ex_start, ex_end).  Writes
 * top (top_a*16, n_kv) int64 (the same token in every column; rows past the
 * count repeat a valid token) and count (device int32).  Ties: score desc,
 * then index asc.  Full-row (max_pos, d) rope tables; d = 128. */
KVR_API size_t kvr_int4w_attractor_workspace_bytes(int64_t n_labelled, int top_a);
KVR_API int kvr_int4w_attractor_select(const float *q, int n_q, int n_kv, const uint8_t *k_packed,
                                       const float *k_scales, const float *cos_tbl, const float *sin_tbl,
                                       int64_t rope_stride, const float *centroids, int n_attractors,
                                       const int32_t *labels, int64_t n_labelled, int top_a, int64_t ex_start,
                                       int64_t ex_end, int64_t *top, int32_t *count, void *workspace,
                                       size_t workspace_bytes, kvr_stream_t stream);

/* Basins of tokens appended after the clustering (no reference counterpart:
 * the reference never labels appended tokens): labels[t] for t in [t0, t1)
 * = nearest centroid (argmin ||c||^2 - 2 x.c, lowest index on ties) of the
 * token's head-0 K dequantised from its int4 codes. */
KVR_API int kvr_int4w_assign_basins(const uint8_t *k_packed, const float *k_scales, int n_kv, int64_t t0, int64_t t1,
                                    const float *centroids, int k, int32_t *labels, kvr_stream_t stream);

/* ret_v[i, h, :] = fp16(v_base[h, i, :] + unpack2(vr_packed[top[i,h], h]) * (2*vr[h]/4))
 * with v_base (n_kv, k, d) fp32 (= x @ W_h^T + V_mean_h) (kvr_retrieval.py:399-402). */
KVR_API int kvr_int4w_vres_add(const float *v_base, const uint8_t *vr_packed, const float *vr_scales,
                       const int64_t *top, int k, int n_kv, int d, uint16_t *ret_v /* fp16 */,
                       kvr_stream_t stream);

/* --------------------------------------------------------------- window ----
 * Ring write of post-RoPE K and V (kvr_window.py:19-41): token i of the n
 * new ones goes to slot (pos + i) % cap, converted to fp16.  Only the last
 * min(n, cap) tokens are written (earlier ones would be overwritten). */
KVR_API int kvr_window_write(const void *k, const void *v, int dtype, int64_t n, int n_kv, int d,
                     uint16_t *ring_k, uint16_t *ring_v, int64_t cap, int64_t pos, kvr_stream_t stream);

/* ------------------------------------------------------------ attention ----
 * Exact decode attention softmax(q k^T / scale) v per Q head (GQA kvh = hq / g)
 * over the concatenation of two K/V segments (segment 1 may be empty), without
 * materialising the concatenation (kvr_window.py:43-69, kvr_hook.py:274-282,
 * kvr_triton.py:42-79).  Segment s is K/V of shape (n_s, n_kv, d) with token
 * stride tok_stride_s elements and dtypes kdt_s / vdt_s.  scale <= 0 means
 * sqrt(d).  Split over the tokens across CTAs, merged by log-sum-exp. */
KVR_API size_t kvr_decode_attn_workspace_bytes(int n_q, int n_kv, int d, int64_t n_tok_total);
KVR_API int kvr_decode_attn(const void *q, int q_dtype, int n_q, int n_kv, int d,
                    const void *k0, const void *v0, int kdt0, int vdt0, int64_t n0, int64_t tok_stride0,
                    const void *k1, const void *v1, int kdt1, int vdt1, int64_t n1, int64_t tok_stride1,
                    float scale, void *out, int out_dtype, void *workspace, size_t workspace_bytes,
                    kvr_stream_t stream);
/* kvr_decode_attn whose segment 1 holds *n1_count rows (a device-side
 * count, at most n1): for a retrieved set whose size is only known on the
 * device (the attractor branch), with no host round trip. */
KVR_API int kvr_decode_attn_counted(const void *q, int q_dtype, int n_q, int n_kv, int d, const void *k0,
                                    const void *v0, int kdt0, int vdt0, int64_t n0, int64_t tok_stride0,
                                    const void *k1, const void *v1, int kdt1, int vdt1, int64_t n1,
                                    int64_t tok_stride1, const int32_t *n1_count, float scale, void *out,
                                    int out_dtype, void *workspace, size_t workspace_bytes, kvr_stream_t stream);

/* One decode step's store update for a layer, fused (kvr_generator.py:78-98,
 * kvr_hook.py:136-148, kvr_window.py:19-25): q_out = RoPE(q) and, when
 * write_kv, window slot `slot` <- (fp16(RoPE(k)), fp16(v)), all at position
 * `pos` with the rotate_half convention and every elementwise op rounded to
 * `dtype` as the eager reference does.  If tail_k/tail_v are given, the slot's
 * old K/V rows (post-RoPE fp16, the evicted token) are first copied to row
 * tail_row of the 1-bit store's pending tail.  q, k, v: (n_q|n_kv, d) of
 * dtype; tables (max_pos, d) fp32 with row stride rope_stride; d = 128. */
KVR_API int kvr_decode_store_update(const void *q, const void *k, const void *v, int dtype, int n_q, int n_kv,
                                    int d, const float *cos_tbl, const float *sin_tbl, int64_t rope_stride,
                                    int64_t pos, void *q_out, uint16_t *win_k, uint16_t *win_v, int64_t win_cap,
                                    int64_t slot, uint16_t *tail_k, uint16_t *tail_v, int64_t tail_row,
                                    int write_kv, kvr_stream_t stream);

/* ------------------------------------------------------------------ sd1 ----
 * 1-bit codec (no reference counterpart).  head_dim d = 128, tile t in
 * {32, 64, 128}.  Store of one layer, per (batch b, kv head h, tile i):
 *   kbits[((b*n_kv + h)*nt_cap + i)*t*4 + j*4 + w]  uint32 (token j, channels 32w..32w+31)
 *   kscale[((b*n_kv + h)*nt_cap + i)*d + c]          fp16
 * and vbits / vscale alike.  Inputs K, V are (B, n, n_kv, d)-like with
 * explicit element strides for batch and token (head stride = d).
 */

/* Orthonormal transform of `rows` vectors of d = 128 fp32 (y may alias x). */
KVR_API int kvr_transform(const float *x, float *y, int64_t rows, int kind, int inverse, kvr_stream_t stream);

/* Encode n_tiles full tiles per (b, h) starting at store tile `tile0`.
 * If cos_tbl != NULL, K is pre-RoPE and is rotated (rotate_half, HF (max_pos, d)
 * rows of stride rope_stride) at positions pos0 + token index. */
KVR_API int kvr_sd1_encode(const void *k, const void *v, int dtype, int batch, int n_kv, int64_t n_tiles,
                   int tile, int64_t batch_stride, int64_t tok_stride, const float *cos_tbl,
                   const float *sin_tbl, int64_t rope_stride, int64_t pos0, int kind, uint32_t *kbits,
                   uint16_t *kscale, uint32_t *vbits, uint16_t *vscale, int64_t nt_cap, int64_t tile0,
                   kvr_stream_t stream);

/* Tile selection scores (B, n_kv, n_tiles) fp32 for q (B, n_q, d) of q_dtype. */
KVR_API int kvr_sd1_tile_scores(const void *q, int q_dtype, int batch, int n_q, int n_kv, const uint32_t *kbits,
                        const uint16_t *kscale, int64_t nt_cap, int64_t n_tiles, int tile, int kind,
                        float *scores, kvr_stream_t stream);

/* Decode selected tiles to post-RoPE K (fp32) and V (fp16) vectors:
 * sel (B, n_kv, k) int64 tile indices (entries < 0 are skipped, rows left 0);
 * out_k / out_v (B, k*t, n_kv, d). */
KVR_API int kvr_sd1_decode_tiles(const uint32_t *kbits, const uint16_t *kscale, const uint32_t *vbits,
                         const uint16_t *vscale, int64_t nt_cap, int batch, int n_kv, int tile, int kind,
                         const int64_t *sel, int k, float *out_k, uint16_t *out_v, kvr_stream_t stream);

/* Selection for one decode step of one layer: score every full tile
 * (kvr_sd1_tile_scores) and keep the top k_sel tiles per (b, h) by (score
 * desc, tile asc), tiles in [ex_t0, ex_t1) excluded.  Writes
 *   sel        (B, n_kv, k_sel) int32 tile indices + tile_base (-1 past n_tiles),
 *   sel_scores (B, n_kv, k_sel) fp32 (may be NULL),
 *   qprime     (B, n_q, d) fp32: the transformed per-head query kvr_sd1_attend needs.
 * One launch (the last CTA of each (b, h) selects). */
KVR_API size_t kvr_sd1_select_workspace_bytes(int batch, int n_kv, int64_t n_tiles);
KVR_API int kvr_sd1_select(const void *q, int q_dtype, int batch, int n_q, int n_kv, const uint32_t *kbits,
                   const uint16_t *kscale, int64_t nt_cap, int64_t n_tiles, int tile, int kind, int k_sel,
                   int64_t ex_t0, int64_t ex_t1, int64_t tile_base, int32_t *sel, float *sel_scores,
                   float *qprime, void *workspace, size_t workspace_bytes, kvr_stream_t stream);

/* Attention over window + pending tail + the selected tiles (sel entries are
 * store tile indices; negative entries are skipped), exact log-sum-exp merge.
 * Window: ring (B, win_cap, n_kv, d) fp16 with n_win valid slots; tail:
 * (B, t, n_kv, d) fp16 with n_tail valid tokens.  q (B, n_q, d) of q_dtype,
 * qprime from kvr_sd1_select.  Writes out (B, n_q, d) of out_dtype, or, if
 * partial_out != NULL, the unnormalised partial rows (B, n_q, d + 2) =
 * [m, l, o] for kvr_lse_merge instead.  Selected tiles are staged into shared
 * memory by bulk asynchronous copies; their waits are bounded and report
 * KVR_ETIMEOUT. */
KVR_API size_t kvr_sd1_attend_workspace_bytes(int batch, int n_q, int n_kv, int tile, int k_sel, int64_t n_win,
                                      int64_t n_tail);
KVR_API int kvr_sd1_attend(const void *q, int q_dtype, const float *qprime, int batch, int n_q, int n_kv,
                   const uint16_t *win_k, const uint16_t *win_v, int64_t win_cap, int64_t n_win,
                   const uint16_t *tail_k, const uint16_t *tail_v, int64_t n_tail, const uint32_t *kbits,
                   const uint16_t *kscale, const uint32_t *vbits, const uint16_t *vscale, int64_t nt_cap,
                   int tile, int kind, const int32_t *sel, int k_sel, float scale, void *out, int out_dtype,
                   float *partial_out, void *workspace, size_t workspace_bytes, kvr_stream_t stream);

/* One sd1 decode step: tile selection + attention over window, tail and the
 * selected tiles (sel/qprime live in the workspace; sel_out may be NULL).
 * Few rows (batch * n_kv <= 16): one kernel, a thread-block cluster per row
 * (see kvr_set_sd1_step_path); otherwise kvr_sd1_select followed by
 * kvr_sd1_attend on one stream. */
/* Which kernels kvr_sd1_decode_step runs (no reference counterpart; a
 * tuning and test switch, process-wide): 0 (default) = one kernel per step,
 * a thread-block cluster per (b, h) row, wherever batch * n_kv <= 16 and the
 * shapes fit its limits (k_sel <= 32, at most 96 window + tail rows and 1024
 * tiles per CTA of the cluster); otherwise, and with 1, the selection kernel
 * followed by the attention kernel.  Both give the same selection; outputs
 * agree to fp32 rounding (the partials are merged in a different order).
 * 2 = the one-kernel path with 8-CTA clusters only (its fallback where
 * 16-CTA clusters cannot be placed).  Returns the previous value.  The initial value comes from the environment
 * variable KVR_SD1_STEP ("split" = 1). */
KVR_API int kvr_set_sd1_step_path(int path);
KVR_API size_t kvr_sd1_workspace_bytes(int batch, int n_q, int n_kv, int64_t n_tiles, int tile, int k_sel,
                               int64_t n_win, int64_t n_tail);
KVR_API int kvr_sd1_decode_step(const void *q, int q_dtype, int batch, int n_q, int n_kv,
                        const uint16_t *win_k, const uint16_t *win_v, int64_t win_cap, int64_t n_win,
                        const uint16_t *tail_k, const uint16_t *tail_v, int64_t n_tail,
                        const uint32_t *kbits, const uint16_t *kscale, const uint32_t *vbits,
                        const uint16_t *vscale, int64_t nt_cap, int64_t n_tiles, int tile, int kind,
                        int k_sel, int64_t ex_t0, int64_t ex_t1, float scale, void *out, int out_dtype,
                        int32_t *sel_out, void *workspace, size_t workspace_bytes, kvr_stream_t stream);

/* One batch-1 decode step of a layer with its store update fused in
 * (modules/kvr_generator.py:78-98 + kvr_hook.py:136-148 + the retrieval and
 * attention of kvr_hook.py:274-282, with the 1-bit codec): q, k, v are the
 * new token's PRE-RoPE rows ((n_q | n_kv, 128) of dtype); RoPE at `pos` as
 * in kvr_decode_store_update; q_out receives the rotated q.  The new K (fp16,
 * rotated) and V land in window slot `slot`, which must be one of the n_win
 * rows attended (n_win counts the new row).  With `evict`, the slot's old row
 * first moves to tail row n_tail - 1 (n_tail counts it; at most `tile`).
 * Then the step runs as kvr_sd1_decode_step over window, tail and store.  One
 * cluster kernel where kvr_sd1_decode_step would run one; otherwise
 * kvr_decode_store_update followed by kvr_sd1_decode_step (same results).
 * Workspace: kvr_sd1_workspace_bytes(1, n_q, n_kv, n_tiles, tile, k_sel,
 * n_win, n_tail). */
KVR_API int kvr_sd1_decode_step_update(const void *q, const void *k, const void *v, int dtype, int n_q, int n_kv,
                               const float *cos_tbl, const float *sin_tbl, int64_t rope_stride, int64_t pos,
                               void *q_out, uint16_t *win_k, uint16_t *win_v, int64_t win_cap, int64_t n_win,
                               int64_t slot, uint16_t *tail_k, uint16_t *tail_v, int64_t n_tail, int evict,
                               const uint32_t *kbits, const uint16_t *kscale, const uint32_t *vbits,
                               const uint16_t *vscale, int64_t nt_cap, int64_t n_tiles, int tile, int kind,
                               int k_sel, int64_t ex_t0, int64_t ex_t1, float scale, void *out, int out_dtype,
                               int32_t *sel_out, void *workspace, size_t workspace_bytes, kvr_stream_t stream);

/* Prefill-sized tile scoring on the tensor cores (tcgen05, kind::f16):
 * q (nq, n_q, d) post-RoPE queries of a prefill block (batch 1); for every
 * query and KV head, the score of each stored tile is the max over its tokens
 * of q'.k_hat with q' = fp16(T(group mean of q)) and k_hat = s (2 bit - 1)
 * (fp32 accumulation).  scores (nq, n_kv, n_tiles) fp32.  tile must be 64.
 * No reference counterpart (north_star: tensor cores for prefill Q.K^T). */
KVR_API size_t kvr_sd1_prefill_workspace_bytes(int64_t nq, int n_kv);
KVR_API int kvr_sd1_prefill_scores(const void *q, int q_dtype, int64_t nq, int n_q, int n_kv, const uint32_t *kbits,
                                   const uint16_t *kscale, int64_t nt_cap, int64_t n_tiles, int tile, int kind,
                                   float *scores, void *workspace, size_t workspace_bytes, kvr_stream_t stream);

/* k-means on the device for the int4w attractor branch (replaces the host
 * MiniBatchKMeans of modules/kvr_retrieval.py:234-246; the reference's basins
 * are then used by retrieve_topk, :332-367).  x (n, d) fp32, d = 128,
 * 1 <= k <= 256, n >= k.  Deterministic Lloyd iterations: centroid j starts at
 * point floor(j n / k); `iters` updates; labels (n) int32 from a final
 * assignment (lowest index on ties); centroids (k, d) fp32. */
KVR_API size_t kvr_kmeans_workspace_bytes(int64_t n, int k);
KVR_API int kvr_kmeans(const float *x, int64_t n, int d, int k, int iters, float *centroids, int32_t *labels,
                       void *workspace, size_t workspace_bytes, kvr_stream_t stream);

/* Partial-attention merge for a sequence split across P sources:
 * partials (P, n_q, d + 2) fp32 rows = [m, l, o_0 .. o_{d-1}] with o
 * unnormalised (sum_j e^{s_j - m} v_j); out (n_q, d) = sum_p e^{m_p-M} o_p / sum_p e^{m_p-M} l_p. */
KVR_API int kvr_lse_merge(const float *partials, int P, int n_q, int d, void *out, int out_dtype,
                  kvr_stream_t stream);

/* Global top-k of a sequence split (no reference counterpart: the reference
 * has no multi-GPU code; the selection rule is its top-k,
 * modules/kvr_retrieval.py:389-392, with the tie rule score descending then
 * index ascending).  scores/idx (n_ranks, rows, k_local): every rank's local
 * candidates (global tile indices, -1 = none) as gathered by an all-gather.
 * Writes global_sel (rows, k_sel) (optional) and local_sel (rows, k_sel): the
 * selected tiles in [tile_base, tile_base + n_local) as local indices, -1
 * elsewhere and past the number of candidates.  At most 4096 candidates per
 * row. */
KVR_API int kvr_merge_candidates(const float *scores, const int32_t *idx, int n_ranks, int rows, int k_local,
                                 int k_sel, int64_t tile_base, int64_t n_local, int32_t *global_sel,
                                 int32_t *local_sel, kvr_stream_t stream);

/* ----------------------------------------------- sequence split over NVLink ----
 * No reference counterpart (the reference has no multi-GPU code).  In place of
 * the NCCL all-gathers of a sequence split, each rank keeps one exchange
 * buffer in its own HBM and maps the other ranks' buffers (CUDA IPC): an
 * exchange is one kernel per rank that writes its data into every rank's
 * buffer with plain stores over NVLink, raises release flags, waits
 * (bounded; a timeout sets the buffer's error word, see
 * kvr_workspace_status) for every rank's flags and merges locally.  bufs[r]
 * is rank r's buffer as mapped in this process (bufs[rank] = its own).  All
 * ranks must issue the same sequence of exchanges.  At most 8 ranks. */
KVR_API size_t kvr_peer_buffer_bytes(void);
KVR_API size_t kvr_peer_handle_bytes(void);
KVR_API int kvr_peer_alloc(void **buf);            /* cudaMalloc + zero fill (set-up, not per step) */
KVR_API int kvr_peer_free(void *buf);
KVR_API int kvr_peer_handle(void *buf, void *handle_out);
KVR_API int kvr_peer_open(const void *handle, void **buf);
KVR_API int kvr_peer_close(void *buf);
/* Candidate exchange + global top-k (same semantics as kvr_merge_candidates):
 * scores/idx (rows, k_local) of this rank; rows <= 64, k_local <= 64. */
KVR_API int kvr_peer_merge_candidates(void *const *bufs, int n_ranks, int rank, const float *scores,
                                      const int32_t *idx, int rows, int k_local, int k_sel, int64_t tile_base,
                                      int64_t n_local, int32_t *global_sel, int32_t *local_sel,
                                      kvr_stream_t stream);
/* Partial-row exchange + log-sum-exp merge (same arithmetic as kvr_lse_merge):
 * partials (n_rows, d + 2) of this rank -> out (n_rows, d); n_rows <= 512. */
KVR_API int kvr_peer_lse_merge(void *const *bufs, int n_ranks, int rank, const float *partials, int n_rows, int d,
                               void *out, int out_dtype, kvr_stream_t stream);

/* Allocation-free variant of kvr_decode_attn (no counterpart in the
 * reference).  For callers that cannot allocate device memory — a plugin
 * inside a host that owns the GPU heap, or a path where cudaMalloc would
 * stall or is forbidden — it takes no workspace: its scratch is a fixed
 * 2 MiB device array inside the library (kvr_decode_attn_noalloc_max_scratch_bytes),
 * held on every GPU that loads the library until the process exits.  A call
 * whose scratch need (kvr_decode_attn_workspace_bytes) exceeds it returns
 * KVR_EINVAL.  It calls no cudaMalloc/cudaFree.  The first call on each device
 * looks up the array's device address with that device current; make that
 * first call before any stream capture.  All calls share the one array:
 * calls that overlap on the GPU (other streams, other host threads) race and
 * must be serialised by the caller.  The array's address is kept per device
 * ordinal for the life of the process: after cudaDeviceReset, or from a
 * different CUDA context on the same device, that address is stale and this
 * entry point must not be called again.  Arguments as kvr_decode_attn. */
KVR_API size_t kvr_decode_attn_noalloc_max_scratch_bytes(void);
KVR_API int kvr_decode_attn_noalloc(const void *q, int q_dtype, int n_q, int n_kv, int d,
                                    const void *k0, const void *v0, int kdt0, int vdt0, int64_t n0,
                                    int64_t tok_stride0, const void *k1, const void *v1, int kdt1, int vdt1,
                                    int64_t n1, int64_t tok_stride1, float scale, void *out, int out_dtype,
                                    kvr_stream_t stream);

/* Synchronises `stream`, then reads and clears the error word every workspace
 * starts with: KVR_ETIMEOUT if a bounded device-side wait of an earlier call
 * using this workspace gave up, else KVR_OK. */
KVR_API int kvr_workspace_status(const void *workspace, kvr_stream_t stream);

/* Test of the failure path above (no reference counterpart): one kernel
 * whose mbarrier can never complete runs the kernels' bounded wait with
 * spin_limit (<= 65536) polls, gives up, sets the workspace's error word and
 * returns — no copy in flight, no fault; kvr_workspace_status then reports
 * KVR_ETIMEOUT and the context stays usable. */
KVR_API int kvr_selftest_bounded_wait(void *workspace, uint32_t spin_limit, kvr_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* KVR_B200_H */
