/*
 * jakal_b200.h — C ABI of the B200-native (sm_100a) Jakal-Net operator hot path.
 *
 * Every entry point takes raw device pointers, sizes, dtype codes and a CUDA stream,
 * launches asynchronously on that stream and returns an int status (JK_OK == 0, negative
 * codes below). No entry point allocates device memory except where stated; callers own
 * every buffer. Inputs are read-only and C-contiguous; outputs are fully overwritten.
 *
 * Reference interfaces (Ahnd6474/Jakal-Net, paths relative to that project) that each
 * entry point replaces are cited beside the declaration.
 */
#ifndef JAKAL_B200_H_
#define JAKAL_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (jk_status_string gives the text) ---------------------------------- */
#define JK_OK 0
#define JK_ERR_BAD_SHAPE (-1)          /* sizes inconsistent or out of the supported range */
#define JK_ERR_BAD_DTYPE (-2)          /* dtype code unknown or not supported by this op  */
#define JK_ERR_UNSUPPORTED_KIND (-3)   /* compress / scorer kind not implemented          */
#define JK_ERR_UNSUPPORTED_DEVICE (-4) /* no sm_100 device, or pointer not on the device  */
#define JK_ERR_LAUNCH (-5)             /* CUDA launch / runtime error                     */
#define JK_ERR_DEVICE_TIMEOUT (-6)     /* a bounded device-side wait gave up              */
#define JK_ERR_BAD_ARG (-7)            /* null pointer, negative k, bad window, ...       */
#define JK_ERR_ALIGNMENT (-8)          /* pointer not 16-byte aligned where required      */

/* ---- dtype codes --------------------------------------------------------------------- */
#define JK_F32 0
#define JK_BF16 1
#define JK_F16 2
/* Projection planes only: f32 projections (rank <= 32) stored as three bf16 planes
 * [h | m | l | 0] of 32 columns each (rp = 128), see jk_split3_bf16; the score tiles then
 * sum the six cross products, which reproduces an f32 dot product. */
#define JK_BF16X3 3

/* ---- edge / route compressors --------------------------------------------------------- */
#define JK_SOFTSIGN 0              /* s / (1 + |s|)                       propagation.py:85   */
#define JK_SIGNED_ABS_SOFTMAX 1    /* sign(s) * softmax(|s|)              propagation.py:74-82 */
#define JK_SIGNED_ENTMAX15 2       /* sign(s) * entmax15(|s|)             kernels.py:155-236  */
#define JK_SOFTMAX 3               /* softmax(s)  (routes)                transition.py:187-194 */

/* ---- multi-head scorers (MultiHeadPairwise / MultiHeadRoute, modules.py:259-302) ------ */
#define JK_HEADS_MAX 0              /* max_h s_h                       modules.py:291-298   */
#define JK_HEADS_SMOOTHMAX 1        /* logsumexp_h s_h - log H         modules.py:276-280   */
#define JK_HEADS_SIGNED_SMOOTHMAX 2 /* sum_h s_h * softmax_h(|s_h|)    modules.py:281-284   */

/* Multi-head scorer for the *_mh entry points. The projection rows hold `heads` blocks of
 * 16 * kph columns (head h at columns [16 kph h, 16 kph (h + 1)), zero padded up to rp);
 * the score of head h is the f32 dot of its blocks plus head_bias[h], and the heads are
 * combined per pair by `combine` before selection / compression. Replaces the
 * multihead_{max,smoothmax,signed_smoothmax}_low_rank_bilinear pairwise kinds and the
 * multihead_max_low_rank_bilinear_route (kernel_common.py:151-178;
 * jakal_net_native.cpp:724-776; jakal_net_native_cuda.cu:881-1027, 1186-1350). */
typedef struct jk_heads {
  int heads;              /* 2..4 (top-k kernels), 2 (window / dense kernels)        */
  int kph;                /* 16-column K steps per head; heads * 16 * kph <= rp       */
  int combine;            /* JK_HEADS_*                                              */
  const float* head_bias; /* device, `heads` floats added before combining, or NULL  */
} jk_heads_t;

typedef struct CUstream_st* jk_stream_t; /* == cudaStream_t; NULL = legacy default stream */

/* Human-readable text for a status code. */
const char* jk_status_string(int status);

/* Library / device probe. Returns JK_OK when the current device is sm_100 and the
 * kernels can launch; otherwise JK_ERR_UNSUPPORTED_DEVICE. Replaces the loader probes
 * native_backend.py:98-178 (supported_devices) / jakal_net_native.cpp:5914-5931. */
int jk_device_check(void);

/* Synchronises `stream`, then reads and clears the library's device-side error word
 * (set by a kernel whose bounded wait gave up). *device_status receives JK_OK or
 * JK_ERR_DEVICE_TIMEOUT. */
int jk_device_status(jk_stream_t stream, int* device_status);

/* Padded projection width the fused kernels expect for a score rank `rank`
 * (rank rounded up to a multiple of 64). */
int64_t jk_padded_rank(int64_t rank);

/*
 * Low-rank projection prologue (tcgen05 GEMM):
 *   out[r, c] = round(x[r, :] . w[c, :])                         c <  rank
 *   then, if core != NULL:  out = round(out * core[c])
 *   then, if temperature != 1: out = round(out / temperature)
 *   out[r, c] = 0 for rank <= c < out_stride (padding)
 * x [rows, dim], w [rank, dim], core [rank], out [rows, out_stride]; all in `dtype`
 * (JK_BF16 or JK_F16); round() = round-to-nearest into dtype, matching a torch.matmul in
 * the input dtype followed by the elementwise ops in that dtype.
 * Requirements: dim % 8 == 0, rank <= 128, out_stride == jk_padded_rank(rank).
 * Replaces the projection steps of jakal_net_native.cpp:6236-6239 (propagation) and
 * :6977-6986 (pairwise-route transition); native_backend.py:4445-4458.
 */
int jk_lowrank_project(const void* x, int64_t rows, int64_t dim, const void* w, int64_t rank,
                       const void* core, float temperature, int dtype, void* out,
                       int64_t out_stride, jk_stream_t stream);

/* The target and source projections of a propagation in one pass over x (rank <= 64,
 * bf16 / f16): out = round(x . w^T) and out2 = round(round(x . w2^T) * core) [/ T], each
 * [rows, 64]; one N = 128 GEMM against w and w2 stacked. Replaces the two matmuls of
 * jakal_net_native.cpp:6236-6239 (same rounding points as jk_lowrank_project). */
int jk_lowrank_project_pair(const void* x, int64_t rows, int64_t dim, const void* w, const void* w2,
                            int64_t rank, const void* core, float temperature, int dtype, void* out,
                            void* out2, jk_stream_t stream);

/*
 * Fused per-row top-k aggregate (tcgen05 score GEMM + streaming top-k + gather):
 *   score[b,t,s] = row_proj[b,t,:] . col_proj[b,s,:]              (f32 accumulation)
 *   visible(t,s) = s < n_cols and (window < 0 or t - window <= s <= t)
 *   sel(t)       = the min(k, #visible) visible s with the largest score, ties to the
 *                  lower s
 *   e[t,s]       = compress(score + score_bias) over sel(t)        (compress = JK_*)
 *   w[t,s]       = e[t,s] * (col_sender ? col_sender[b,s] : 1)
 *   out_state[b,t]  = sum_{s in sel(t)} w[t,s] * col_state[b,s]
 *   out_val[b,t,:]  = sum_{s in sel(t)} w[t,s] * col_val[b,s,:]
 * score_bias is added to every score; when bias_dev != NULL the f32 it points to (device
 * memory) is added as well, so a bias tensor needs no host synchronisation.
 * Shapes: row_proj [B, n_rows, rp], col_proj [B, n_cols, rp] (rp = jk_padded_rank, dtype
 * proj_dtype = JK_BF16 | JK_F16 | JK_BF16X3); col_state and col_sender [B, n_cols] in state_dtype;
 * col_val [B, n_cols, dim] in val_dtype; out_state [B, n_rows], out_val [B, n_rows, dim] in
 * out_dtype. Optional out_scores f32 [B, n_rows, k] (score + bias, sorted descending,
 * -inf in empty slots) and out_index int64 [B, n_rows, k] (-1 in empty slots).
 * 1 <= k <= 64. rp <= 128.
 * Replaces low_rank_propagation_topk_forward_cuda (jakal_net_native_cuda.cu:2545-2660,
 * kernel :1029-1183) as called from propagation_topk (jakal_net_native.cpp:6355-6389);
 * the window > 0 form is the window-intersect-top-k operator built from
 * kernel_common.py:433-456 + propagation.py:67-88.
 */
int jk_propagation_topk_forward(const void* row_proj, const void* col_proj, int64_t batch,
                                int64_t n_rows, int64_t n_cols, int64_t rp, int proj_dtype,
                                const void* col_state, const void* col_sender, int state_dtype,
                                const void* col_val, int64_t dim, int val_dtype, int64_t k,
                                int64_t window, float score_bias, const float* bias_dev,
                                int compress, void* out_state, void* out_val, int out_dtype,
                                float* out_scores, int64_t* out_index, jk_stream_t stream);

/*
 * Fused window / dense propagation without top-k (flash-style: tcgen05 score tile -> exact
 * f32 edges -> bf16 hi + lo edge tiles -> tcgen05 value GEMM, TMEM accumulator):
 *   visible(t,s) = s < n_cols and (window < 0 or t - window <= s <= t)
 *   e[t,s]       = compress over the visible s of row t of (score + score_bias (+ *bias_dev))
 *                  compress = JK_SOFTSIGN | JK_SIGNED_ABS_SOFTMAX | JK_SIGNED_ENTMAX15
 *   out_state[b,t] = sum_s e * col_state[b,s],  out_val[b,t,:] = sum_s e * col_val[b,s,:]
 * row_proj [B,n_rows,rp], col_proj [B,n_cols,rp] (JK_BF16 | JK_F16 | JK_BF16X3); col_val
 * [B,n_cols,dim] in the projections' 16-bit type (bf16 for JK_BF16X3), dim % 64 == 0; for
 * f32 values pass the bf16 hi plane as col_val and the lo plane as col_val_lo (see
 * jk_split2_bf16), else col_val_lo = NULL. col_state in state_dtype; outputs in out_dtype.
 * Replaces propagation_window / propagation_dense / propagation_query_dense
 * (jakal_net_native.cpp:6190-6303, 5962-6076, 6078-6188) and the CUDA kernels
 * jakal_net_native_cuda.cu:1579-1750, 2023-2109, 1388-1576.
 */
int jk_propagation_window_forward(const void* row_proj, const void* col_proj, int64_t batch,
                                  int64_t n_rows, int64_t n_cols, int64_t rp, int proj_dtype,
                                  const void* col_state, int state_dtype, const void* col_val,
                                  const void* col_val_lo, int64_t dim, int64_t window,
                                  float score_bias, const float* bias_dev, int compress,
                                  void* out_state, void* out_val, int out_dtype,
                                  jk_stream_t stream);

/* Dense pairwise transition (Transition.forward with a dense route, transition.py:238-254):
 * every source routes to every destination, routes compressed over the destinations of
 * the source (JK_SOFTMAX | JK_SIGNED_ABS_SOFTMAX | JK_SIGNED_ENTMAX15), times the source's
 * sender strength, accumulated into the destinations:
 *   out_state[d] = sum_s r[s,d] * sender[s] * src_state[s],
 *   out_val[d]   = sum_s r[s,d] * sender[s] * src_val[s].
 * src_proj [B, n_src, rp] (route source projection divided by the temperature) and
 * dst_proj [B, n_dst, rp]; logits = src_proj . dst_proj + score_bias (+ *bias_dev).
 * stats: caller scratch of batch * n_src * 3 floats (per-source max, sender / normaliser,
 * entmax threshold). dim % 64 == 0; f32 values as bf16 hi (src_val) + lo (src_val_lo)
 * planes, like jk_propagation_window_forward.
 * Replaces transition_pairwise_dense (jakal_net_native.cpp:6705-6914; native_backend.py
 * :5801-5822). */
int jk_transition_pairwise_dense_forward(const void* src_proj, const void* dst_proj, int64_t batch,
                                         int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                         const void* src_state, const void* sender, int state_dtype,
                                         const void* src_val, const void* src_val_lo, int64_t dim,
                                         float score_bias, const float* bias_dev, int compress,
                                         float* stats, void* out_state, void* out_val, int out_dtype,
                                         jk_stream_t stream);

/* Row block of a propagation / per-query top-k (row-sharded multi-GPU): the arguments of
 * jk_propagation_topk_forward over the FULL tensors, computing only the rows
 * [row_begin, row_begin + row_count) (row_begin a multiple of 128; row_count a multiple of
 * 128 unless the block runs to the last row); the other output rows are not written.
 * Nothing in the reference corresponds (its kernels run on one GPU); this is the per-rank
 * step of the query-row-block partition, whose outputs an all-gather then assembles. */
int jk_propagation_topk_rows_forward(const void* row_proj, const void* col_proj, int64_t batch,
                                     int64_t n_rows, int64_t row_begin, int64_t row_count,
                                     int64_t n_cols, int64_t rp, int proj_dtype, const void* col_state,
                                     const void* col_sender, int state_dtype, const void* col_val,
                                     int64_t dim, int val_dtype, int64_t k, int64_t window,
                                     float score_bias, const float* bias_dev, int compress,
                                     void* out_state, void* out_val, int out_dtype, float* out_scores,
                                     int64_t* out_index, jk_stream_t stream);

/* Multi-head variants: the entry point of the same name without _mh, with the scorer
 * `heads` (jk_heads_t above; 16-bit projections only, not JK_BF16X3). */
int jk_propagation_topk_forward_mh(const void* row_proj, const void* col_proj, int64_t batch,
                                   int64_t n_rows, int64_t n_cols, int64_t rp, int proj_dtype,
                                   const void* col_state, const void* col_sender, int state_dtype,
                                   const void* col_val, int64_t dim, int val_dtype, int64_t k,
                                   int64_t window, float score_bias, const float* bias_dev,
                                   int compress, void* out_state, void* out_val, int out_dtype,
                                   float* out_scores, int64_t* out_index, const jk_heads_t* heads,
                                   jk_stream_t stream);
int jk_transition_query_topk_forward_mh(const void* query_proj, const void* source_proj, int64_t batch,
                                        int64_t n_query, int64_t n_source, int64_t rp, int proj_dtype,
                                        const void* source_state, const void* source_sender,
                                        int state_dtype, const void* source_val, int64_t dim,
                                        int val_dtype, int64_t k, float score_bias,
                                        const float* bias_dev, int compress, void* out_state,
                                        void* out_val, int out_dtype, float* out_scores,
                                        int64_t* out_index, const jk_heads_t* heads, jk_stream_t stream);
int jk_transition_pairwise_topk_forward_mh(const void* src_proj, const void* dst_proj, int64_t batch,
                                           int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                           const void* src_state, const void* src_sender, int state_dtype,
                                           const void* src_val, int64_t dim, int val_dtype, int64_t k,
                                           float score_bias, const float* bias_dev, int compress,
                                           float* accum, void* out_state, void* out_val, int out_dtype,
                                           const jk_heads_t* heads, jk_stream_t stream);
int jk_propagation_window_forward_mh(const void* row_proj, const void* col_proj, int64_t batch,
                                     int64_t n_rows, int64_t n_cols, int64_t rp, int proj_dtype,
                                     const void* col_state, int state_dtype, const void* col_val,
                                     const void* col_val_lo, int64_t dim, int64_t window,
                                     float score_bias, const float* bias_dev, int compress,
                                     void* out_state, void* out_val, int out_dtype,
                                     const jk_heads_t* heads, jk_stream_t stream);
int jk_transition_pairwise_dense_forward_mh(const void* src_proj, const void* dst_proj, int64_t batch,
                                            int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                            const void* src_state, const void* sender, int state_dtype,
                                            const void* src_val, const void* src_val_lo, int64_t dim,
                                            float score_bias, const float* bias_dev, int compress,
                                            float* stats, void* out_state, void* out_val, int out_dtype,
                                            const jk_heads_t* heads, jk_stream_t stream);

/* f32 -> three bf16 planes [h|m|l|0] of 32 columns (rank <= 32), out [rows, 128] bf16, for
 * JK_BF16X3 projections. Replaces nothing: the reference computes these dots in f32. */
int jk_split3_bf16(const float* x, int64_t rows, int64_t rank, void* out, jk_stream_t stream);

/* f32 -> bf16 hi plane + bf16 lo plane (x - hi), n elements each, for f32 values. */
int jk_split2_bf16(const float* x, int64_t n, void* hi, void* lo, jk_stream_t stream);

/* f32 x [batch, rows, cols] (plus, when extra_col is not NULL, extra_col [batch, rows] as
 * column cols) -> bf16 out [batch, nblk * rows, out_cols]: block k (rows [k * rows,
 * (k + 1) * rows) of every batch item) holds the hi plane bf16(x) when bit k of plane_bits is
 * 0, the lo plane bf16(x - hi) when it is 1; columns past the data are zero. Stacking the
 * route matrix as (hi, hi, lo) and the values as (hi, lo, hi) makes one GEMM over the stacked
 * dimension sum the three products of an f32-accurate split GEMM. nblk <= 4. Replaces
 * nothing in the reference (its scatter adds f32 routes into f32 accumulators). */
int jk_split_stack_bf16(const float* x, const float* extra_col, int64_t batch, int64_t rows, int64_t cols,
                        int64_t out_cols, int nblk, unsigned plane_bits, void* out, jk_stream_t stream);

/*
 * Per-query ("query top-k") transition: identical contract to
 * jk_propagation_topk_forward with rows = query slots (row_proj = target-side route
 * projection of query_val), columns = source nodes (col_proj = core-weighted,
 * temperature-scaled source projection), compress = JK_SOFTMAX and
 * col_sender = sender strength softplus(src.state); window must be -1.
 * Replaces transition_query_topk (jakal_net_native.cpp:7089-7246) and
 * query_topk_reduce_cuda (jakal_net_native_cuda.cu:2335-2417).
 */
int jk_transition_query_topk_forward(const void* query_proj, const void* source_proj,
                                     int64_t batch, int64_t n_query, int64_t n_source,
                                     int64_t rp, int proj_dtype, const void* source_state,
                                     const void* source_sender, int state_dtype,
                                     const void* source_val, int64_t dim, int val_dtype,
                                     int64_t k, float score_bias, const float* bias_dev,
                                     int compress, void* out_state, void* out_val,
                                     int out_dtype, float* out_scores, int64_t* out_index,
                                     jk_stream_t stream);

/*
 * Per-source sparse transition (SparseTransition):
 *   logit[b,i,j] = src_proj[b,i,:] . dst_proj[b,j,:] + score_bias (+ *bias_dev)
 *                  (src_proj already core-weighted and temperature-scaled)
 *   sel(i)       = top-k destinations j of source i, ties to the lower j
 *   r[i,j]       = compress(logit) over sel(i)        (JK_SOFTMAX / SIGNED_ABS / ENTMAX15)
 *   out_state[b,j] = sum_i r[i,j] * src_sender[b,i] * src_state[b,i]
 *   out_val[b,j,:] = sum_i r[i,j] * src_sender[b,i] * src_val[b,i,:]
 * src_state / src_sender in state_dtype, src_val in val_dtype. `accum` is caller-provided
 * f32 scratch of B*n_dst*(dim+1) elements, 16-byte aligned (zeroed by the call); outputs
 * are written in out_dtype. 1 <= k <= 64.
 * Replaces low_rank_pairwise_topk_forward_cuda (jakal_net_native_cuda.cu:2420-2542,
 * kernel :740-878) as called from transition_pairwise_topk
 * (jakal_net_native.cpp:6958-7007).
 */
int jk_transition_pairwise_topk_forward(const void* src_proj, const void* dst_proj,
                                        int64_t batch, int64_t n_src, int64_t n_dst,
                                        int64_t rp, int proj_dtype, const void* src_state,
                                        const void* src_sender, int state_dtype,
                                        const void* src_val, int64_t dim, int val_dtype,
                                        int64_t k, float score_bias, const float* bias_dev,
                                        int compress, float* accum, void* out_state,
                                        void* out_val, int out_dtype, jk_stream_t stream);

/*
 * Routes form of the per-source sparse transition (deterministic, no atomics):
 *   routes[b, s, d] = compress(logit[b, s, :] over sel(s))[d] * (src_sender ? src_sender[b, s] : 1)
 * for the k selected destinations d of every source s (selection, bias and compressors as
 * jk_transition_pairwise_topk_forward); every other entry is left untouched, so the caller
 * zeroes routes (f32 [B, n_src, n_dst]) first. The aggregate
 *   out_state[b, d] = sum_s routes[b, s, d] * src_state[b, s],
 *   out_val[b, d, :] = sum_s routes[b, s, d] * src_val[b, s, :]
 * is then a plain GEMM (routes^T x values), with no atomics and a fixed summation order.
 * Optional out_scores f32 / out_index int64 [B, n_src, k]: every source's selection (logit +
 * bias, in descending order, -inf / -1 in empty slots) -- what the backward of the route
 * scores needs (native_backend.py:4459-4491).
 * Same sizes and limits as jk_transition_pairwise_topk_forward (1 <= k <= 64, rp <= 128).
 * Replaces the scatter of low_rank_pairwise_topk_forward_cuda (jakal_net_native_cuda.cu:
 * 740-878, atomicAdd at :862-873) and of the blocked path jakal_net_native.cpp:6916-7087.
 */
int jk_transition_pairwise_topk_routes(const void* src_proj, const void* dst_proj, int64_t batch,
                                       int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                       const void* src_sender, int state_dtype, int64_t k,
                                       float score_bias, const float* bias_dev, int compress,
                                       float* routes, float* out_scores, int64_t* out_index,
                                       jk_stream_t stream);

/* Multi-head (jk_heads_t) variant of jk_transition_pairwise_topk_routes. */
int jk_transition_pairwise_topk_routes_mh(const void* src_proj, const void* dst_proj, int64_t batch,
                                          int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                          const void* src_sender, int state_dtype, int64_t k,
                                          float score_bias, const float* bias_dev, int compress,
                                          float* routes, float* out_scores, int64_t* out_index,
                                          const jk_heads_t* heads, jk_stream_t stream);

/*
 * Select-aggregate over materialised f32 score rows (any k, any score rank):
 *   scores [B, row_count, n_cols] holds score[b, t, s] for the rows t in
 *   [row_begin, row_begin + row_count) of an n_rows-row operator (e.g. a plain GEMM of the
 *   projections). Visibility, selection (ties to the lower column), score_bias / bias_dev,
 *   compressors and sender weighting are those of jk_propagation_topk_forward, with no limit
 *   on k or on the rank that produced the scores.
 *   scatter == 0 (gather): out_state [B, n_rows] / out_val [B, n_rows, dim] (out_dtype) get
 *     rows row_begin..; state / sender [B, n_cols], val [B, n_cols, dim] are per column.
 *   scatter == 1 (per-source transition): rows are sources; state / sender [B, n_rows],
 *     val [B, n_rows, dim]; acc_state [B, n_cols] and acc_val [B, n_cols, dim] (f32, zeroed
 *     by the caller) receive sum_t w[t, s] * state[t] and sum_t w[t, s] * val[t, :].
 *   sel_score f32 / sel_index int64 [B, row_count, k] (caller scratch, also a result): the
 *   selected scores (bias included) and columns in ascending column order, -inf / -1 pad.
 * One CTA per row: an exact 4-pass radix select over order-preserving keys, block prefix
 * sums for the survivors, block reductions for the compressor, then the gather or the
 * scatter. Replaces the blocked top-k paths that take any k:
 * jakal_net_native.cpp:6390-6447 (propagation_topk), :6916-7087 (transition_pairwise_topk)
 * and :7089-7246 (transition_query_topk), the path the reference takes when its CUDA kernels
 * refuse k > 64 (jakal_net_native_cuda.cu:2432-2434, 2557-2559).
 */
int jk_select_aggregate_forward(const float* scores, int64_t batch, int64_t n_rows, int64_t n_cols,
                                int64_t row_begin, int64_t row_count, const void* state,
                                const void* sender, int state_dtype, const void* val, int64_t dim,
                                int val_dtype, int64_t k, int64_t window, float score_bias,
                                const float* bias_dev, int compress, int scatter, void* out_state,
                                void* out_val, int out_dtype, float* acc_state, float* acc_val,
                                float* sel_score, int64_t* sel_index, jk_stream_t stream);

/* ---- backward (training) kernels --------------------------------------------------
 * The row-wise pieces of the top-k operators' backward, behind the reference's autograd
 * Functions (native_backend.py:4408-4601 uses softmax_backward_cuda and the reduce
 * backward; the kernels replaced are jakal_net_native_cuda.cu:2112-2320). `dtype` applies to
 * every tensor argument of a call (JK_F32, JK_BF16, JK_F16); accumulation is f32.
 */

/* grad_scores[r, j] = routes[r, j] * (grad_routes[r, j] - sum_j' routes[r, j'] grad_routes[r, j'])
 * for rows x n row-major tensors (the softmax backward; jakal_net_native.cpp:408-416). */
int jk_softmax_backward(const void* routes, const void* grad_routes, void* grad_scores, int64_t rows,
                        int64_t n, int dtype, jk_stream_t stream);

/* grad_scores[i] = grad_edges[i] / (1 + |scores[i]|)^2 over n elements (softsign backward;
 * jakal_net_native.cpp:398-406). */
int jk_softsign_backward(const void* scores, const void* grad_edges, void* grad_scores, int64_t n,
                         int dtype, jk_stream_t stream);

/* Gather half of the backward of a top-k reduce (out[b, q] = sum_e edges[b, q, e] *
 * x[b, indices[b, q, e]]; jakal_net_native.cpp:152-166):
 *   grad_edges[b, q, e] = grad_state[b, q] * state[b, idx] + grad_val[b, q, :] . val[b, idx, :]
 * indices int64 [B, n_rows, k] (-1: no edge, gradient 0), state [B, n_src], val
 * [B, n_src, dim], grad_state [B, n_rows], grad_val [B, n_rows, dim] in dtype; grad_edges
 * [B, n_rows, k] in out_dtype. The scatter half (the gradients of state and val) is a GEMM of
 * the dense edge matrix (jk_topk_to_dense). */
int jk_topk_reduce_backward_edges(const int64_t* indices, const void* state, const void* val,
                                  const void* grad_state, const void* grad_val, void* grad_edges,
                                  int64_t batch, int64_t n_rows, int64_t n_src, int64_t k, int64_t dim,
                                  int dtype, int out_dtype, jk_stream_t stream);

/* dense[r, indices[r, e]] += w[r, e] for rows x k selections (f32 w, int64 indices, -1 and
 * zero weights skipped); dense f32 [rows, n_cols] zeroed by the caller. A selection names
 * each column once; padded window index lists may repeat a placeholder column with weight 0,
 * which adds nothing. Turns the scatters of the backward into GEMMs with a fixed summation
 * order. */
int jk_topk_to_dense(const float* w, const int64_t* indices, float* dense, int64_t rows, int64_t k,
                     int64_t n_cols, jk_stream_t stream);

/* Failure-path test entry (no reference counterpart): jk_propagation_window_forward
 * (softsign, no bias) with a producer warp that issues no load and no MMA, so every consumer
 * wait runs into its bound (about 2 s): the kernel sets the device error word, releases its
 * TMEM and returns; jk_device_status then reports JK_ERR_DEVICE_TIMEOUT and the context stays
 * usable. Outputs are zeros. For tests of that path only. */
int jk_debug_window_stalled_producer(const void* row_proj, const void* col_proj, int64_t batch,
                                     int64_t n_rows, int64_t n_cols, int64_t rp, int proj_dtype,
                                     const void* col_state, int state_dtype, const void* col_val,
                                     int64_t dim, int64_t window, void* out_state, void* out_val,
                                     int out_dtype, jk_stream_t stream);

/*
 * Allocation-free per-source sparse transition. No counterpart in the reference: it exists
 * for callers that cannot allocate device memory at call time -- plain-C / FFI hosts with no
 * device allocator of their own, and latency-critical loops that must not call cudaMalloc /
 * cudaFree because those can synchronise the device. Same contract as
 * jk_transition_pairwise_topk_forward without the `accum` argument: the f32 scratch is a
 * fixed 16 MiB device array inside the library (held on every GPU that loads it until exit),
 * so B * n_dst * (dim + 1) must not exceed jk_transition_pairwise_topk_noalloc_capacity()
 * floats, else JK_ERR_BAD_SHAPE. Every call looks up the array's address on the current
 * device (so it stays valid after a device reset or from another context); the first call
 * on a device also loads the library's module there, so make it before any stream capture. Calls share the array: calls that overlap on the GPU
 * race; serialise them on one stream. The scratch is zeroed on the stream by every call.
 */
int jk_transition_pairwise_topk_forward_noalloc(const void* src_proj, const void* dst_proj,
                                                int64_t batch, int64_t n_src, int64_t n_dst,
                                                int64_t rp, int proj_dtype, const void* src_state,
                                                const void* src_sender, int state_dtype,
                                                const void* src_val, int64_t dim, int val_dtype,
                                                int64_t k, float score_bias, const float* bias_dev,
                                                int compress, void* out_state, void* out_val,
                                                int out_dtype, jk_stream_t stream);

/* Scratch capacity (in f32 elements) of the allocation-free entry point above. */
int64_t jk_transition_pairwise_topk_noalloc_capacity(void);

#ifdef __cplusplus
}
#endif

#endif /* JAKAL_B200_H_ */
