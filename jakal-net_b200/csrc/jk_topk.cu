// Fused low-rank score -> top-k -> edge compress -> aggregate: host entry points. The kernel
// itself (and its design notes) is in jk_topk_kernel.cuh; its launchers are instantiated
// per value type in jk_topk_vt_bf16.cu, jk_topk_vt_f16.cu and jk_topk_vt_f32.cu.
#include "jk_topk_kernel.cuh"

namespace jk {
namespace topk {

JK_TOPK_EXTERN(float)
JK_TOPK_EXTERN(__nv_bfloat16)
JK_TOPK_EXTERN(__half)

// Converts the f32 destination accumulators of the scatter mode into the outputs.
__global__ void finalize_scatter(const float* acc_state, const float* acc_val, int64_t n_state, int64_t n_val,
                                 void* out_state, void* out_val, int out_dtype) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t j = i; j < n_val; j += stride) st_elem(out_val, j, out_dtype, acc_val[j]);
  for (int64_t j = i; j < n_state; j += stride) st_elem(out_state, j, out_dtype, acc_state[j]);
}

template <int KATOMS, int MODE>
int launch_k(const CUtensorMap& tr, const CUtensorMap& tc, const CUtensorMap& tv, const CUtensorMap& to,
             const Params& p, int64_t batch,
             uint32_t idesc, cudaStream_t st) {
  switch (p.val_dtype) {
    case JK_F32: return launch_vt<KATOMS, MODE, float>(tr, tc, tv, to, p, batch, idesc, st);
    case JK_BF16: return launch_vt<KATOMS, MODE, __nv_bfloat16>(tr, tc, tv, to, p, batch, idesc, st);
    default: return launch_vt<KATOMS, MODE, __half>(tr, tc, tv, to, p, batch, idesc, st);
  }
}

template <int MODE>
int launch(const void* row_proj, const void* col_proj, int64_t batch, int64_t n_rows, int64_t n_cols, int64_t rp,
           int proj_dtype, Params& p, cudaStream_t st) {
  CUtensorMap tr, tc, tv, to;
  const bool bf16 = proj_dtype != JK_F16;
  p.split3 = proj_dtype == JK_BF16X3 ? 1 : 0;
  int status = make_tmap_3d_16bit(&tr, row_proj, rp, n_rows, batch, 64, kRows, bf16);
  if (status != JK_OK) return status;
  status = make_tmap_3d_16bit(&tc, col_proj, rp, n_cols, batch, 64, kCols, bf16);
  if (status != JK_OK) return status;
  tv = tc;  // placeholder when the slab path is off
  p.slab_ok = 0;
  if (MODE == kGather && p.val_dtype != JK_F32 && p.dim % 64 == 0 && aligned16(p.col_val)) {
    if (make_tmap_3d_16bit(&tv, p.col_val, p.dim, n_cols, batch, 64, kEK, p.val_dtype == JK_BF16, true) == JK_OK)
      p.slab_ok = 1;
  }
  to = tc;  // placeholder when the outputs are not stored by TMA
  p.tma_out = 0;
  if (MODE == kGather && p.slab_ok && p.out_dtype != JK_F32 && aligned16(p.out_val)) {
    if (make_tmap_3d_16bit(&to, p.out_val, p.dim, n_rows, batch, 64, kRows, p.out_dtype == JK_BF16, true) == JK_OK)
      p.tma_out = 1;
  }
  const uint32_t idesc = idesc_f16(kRows, kCols, bf16 ? 1u : 0u);
  if (rp == 64) return launch_k<1, MODE>(tr, tc, tv, to, p, batch, idesc, st);
  return launch_k<2, MODE>(tr, tc, tv, to, p, batch, idesc, st);
}

int validate_common(const void* row_proj, const void* col_proj, int64_t batch, int64_t n_rows, int64_t n_cols,
                    int64_t rp, int proj_dtype, const void* state, int state_dtype, const void* val, int64_t dim,
                    int val_dtype, int64_t k, int compress, int out_dtype) {
  if (row_proj == nullptr || col_proj == nullptr || state == nullptr || val == nullptr) return JK_ERR_BAD_ARG;
  if (proj_dtype != JK_BF16 && proj_dtype != JK_F16 && proj_dtype != JK_BF16X3) return JK_ERR_BAD_DTYPE;
  if (proj_dtype == JK_BF16X3 && rp != 128) return JK_ERR_BAD_SHAPE;
  if (val_dtype < JK_F32 || val_dtype > JK_F16 || out_dtype < JK_F32 || out_dtype > JK_F16 || state_dtype < JK_F32 ||
      state_dtype > JK_F16)
    return JK_ERR_BAD_DTYPE;
  if (compress < JK_SOFTSIGN || compress > JK_SOFTMAX) return JK_ERR_UNSUPPORTED_KIND;
  if (k < 1 || k > 64) return JK_ERR_BAD_ARG;
  if (batch <= 0 || n_rows <= 0 || n_cols <= 0 || dim <= 0) return JK_ERR_BAD_SHAPE;
  if (batch > 65535 || n_rows > (int64_t(1) << 30) || n_cols > (int64_t(1) << 30)) return JK_ERR_BAD_SHAPE;
  if (rp != 64 && rp != 128) return JK_ERR_BAD_SHAPE;
  if (!aligned16(row_proj) || !aligned16(col_proj)) return JK_ERR_ALIGNMENT;
  if (dim % 8 == 0 && !aligned16(val)) return JK_ERR_ALIGNMENT;
  return JK_OK;
}

}  // namespace topk
}  // namespace jk

namespace jk {
namespace topk {

int gather_forward(const void* row_proj, const void* col_proj, int64_t batch, int64_t n_rows, int64_t n_cols,
                   int64_t rp, int proj_dtype, const void* col_state, const void* col_sender, int state_dtype,
                   const void* col_val, int64_t dim, int val_dtype, int64_t k, int64_t window, float score_bias,
                   const float* bias_dev, int compress, void* out_state, void* out_val, int out_dtype,
                   float* out_scores, int64_t* out_index, const jk_heads_t* heads, int64_t row_begin,
                   int64_t row_count, jk_stream_t stream) {
  int st = validate_common(row_proj, col_proj, batch, n_rows, n_cols, rp, proj_dtype, col_state, state_dtype, col_val,
                           dim, val_dtype, k, compress, out_dtype);
  if (st != JK_OK) return st;
  // Row block [row_begin, row_begin + row_count): kRows-aligned start, and a whole number
  // of kRows tiles unless it runs to the last row.
  if (row_begin < 0 || row_count <= 0 || row_begin + row_count > n_rows || row_begin % kRows != 0 ||
      (row_count % kRows != 0 && row_begin + row_count != n_rows))
    return JK_ERR_BAD_ARG;
  if (st != JK_OK) return st;
  if (out_state == nullptr || out_val == nullptr) return JK_ERR_BAD_ARG;
  if (dim % 8 == 0 && !aligned16(out_val)) return JK_ERR_ALIGNMENT;
  if (window < -1) return JK_ERR_BAD_ARG;
  Heads hd;
  st = read_heads(heads, rp, proj_dtype, 4, hd);
  if (st != JK_OK) return st;
  st = check_device();
  if (st != JK_OK) return st;
  Params p{};
  p.n_rows = n_rows;
  p.n_cols = n_cols;
  p.rp = rp;
  p.dim = dim;
  p.k = static_cast<int>(k);
  p.window = window;
  p.row_begin = row_begin;
  p.row_count = row_count;
  p.bias = score_bias;
  p.bias_dev = bias_dev;
  p.compress = compress;
  p.state_dtype = state_dtype;
  p.val_dtype = val_dtype;
  p.out_dtype = out_dtype;
  p.col_state = col_state;
  p.col_val = col_val;
  p.col_sender = col_sender;
  p.out_state = out_state;
  p.out_val = out_val;
  p.out_scores = out_scores;
  p.out_index = out_index;
  p.heads = hd.heads;
  p.kph = hd.kph;
  p.combine = hd.combine;
  p.head_bias = hd.bias;
  return launch<kGather>(row_proj, col_proj, batch, n_rows, n_cols, rp, proj_dtype, p,
                         reinterpret_cast<cudaStream_t>(stream));
}

int routes_forward(const void* src_proj, const void* dst_proj, int64_t batch, int64_t n_src, int64_t n_dst,
                   int64_t rp, int proj_dtype, const void* src_sender, int state_dtype, int64_t k, float score_bias,
                   const float* bias_dev, int compress, float* routes, float* out_scores, int64_t* out_index,
                   const jk_heads_t* heads, jk_stream_t stream) {
  // the value / state arguments of the shared checks are not read in the routes form
  int st = validate_common(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, routes, JK_F32, routes, 1, JK_F32,
                           k, compress, JK_F32);
  if (st != JK_OK) return st;
  if (routes == nullptr) return JK_ERR_BAD_ARG;
  if (src_sender != nullptr && (state_dtype < JK_F32 || state_dtype > JK_F16)) return JK_ERR_BAD_DTYPE;
  Heads hd;
  st = read_heads(heads, rp, proj_dtype, 4, hd);
  if (st != JK_OK) return st;
  st = check_device();
  if (st != JK_OK) return st;
  Params p{};
  p.n_rows = n_src;
  p.row_count = n_src;
  p.n_cols = n_dst;
  p.rp = rp;
  p.dim = 1;
  p.k = static_cast<int>(k);
  p.window = -1;
  p.bias = score_bias;
  p.bias_dev = bias_dev;
  p.compress = compress;
  p.state_dtype = state_dtype;
  p.val_dtype = JK_F32;
  p.out_dtype = JK_F32;
  p.col_state = routes;
  p.col_val = routes;
  p.col_sender = src_sender;
  p.routes = routes;
  p.out_scores = out_scores;
  p.out_index = out_index;
  p.heads = hd.heads;
  p.kph = hd.kph;
  p.combine = hd.combine;
  p.head_bias = hd.bias;
  return launch<kScatter>(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, p,
                          reinterpret_cast<cudaStream_t>(stream));
}

int scatter_forward(const void* src_proj, const void* dst_proj, int64_t batch, int64_t n_src, int64_t n_dst,
                    int64_t rp, int proj_dtype, const void* src_state, const void* src_sender, int state_dtype,
                    const void* src_val, int64_t dim, int val_dtype, int64_t k, float score_bias,
                    const float* bias_dev, int compress, float* accum, void* out_state, void* out_val, int out_dtype,
                    const jk_heads_t* heads, jk_stream_t stream) {
  int st = validate_common(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, src_state, state_dtype, src_val,
                           dim, val_dtype, k, compress, out_dtype);
  if (st != JK_OK) return st;
  if (accum == nullptr || out_state == nullptr || out_val == nullptr) return JK_ERR_BAD_ARG;
  if (!aligned16(accum)) return JK_ERR_ALIGNMENT;
  Heads hd;
  st = read_heads(heads, rp, proj_dtype, 4, hd);
  if (st != JK_OK) return st;
  st = check_device();
  if (st != JK_OK) return st;
  auto cs = reinterpret_cast<cudaStream_t>(stream);
  const int64_t n_state = batch * n_dst;
  const int64_t n_val = batch * n_dst * dim;
  // Value accumulators first (16-byte aligned for the vector atomics), then state.
  float* acc_val = accum;
  float* acc_state = accum + n_val;
  if (cudaMemsetAsync(accum, 0, sizeof(float) * (n_state + n_val), cs) != cudaSuccess) return launch_status();
  Params p{};
  p.n_rows = n_src;
  p.row_count = n_src;
  p.n_cols = n_dst;
  p.rp = rp;
  p.dim = dim;
  p.k = static_cast<int>(k);
  p.window = -1;
  p.bias = score_bias;
  p.bias_dev = bias_dev;
  p.compress = compress;
  p.state_dtype = state_dtype;
  p.val_dtype = val_dtype;
  p.out_dtype = out_dtype;
  p.col_state = src_state;
  p.col_val = src_val;
  p.col_sender = src_sender;
  p.acc_state = acc_state;
  p.acc_val = acc_val;
  p.heads = hd.heads;
  p.kph = hd.kph;
  p.combine = hd.combine;
  p.head_bias = hd.bias;
  st = launch<kScatter>(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, p, cs);
  if (st != JK_OK) return st;
  const int64_t work = n_val > n_state ? n_val : n_state;
  int blocks = static_cast<int>((work + 255) / 256);
  if (blocks > 4 * 148 * 8) blocks = 4 * 148 * 8;
  if (blocks < 1) blocks = 1;
  finalize_scatter<<<blocks, 256, 0, cs>>>(acc_state, acc_val, n_state, n_val, out_state, out_val, out_dtype);
  return launch_status();
}

}  // namespace topk
}  // namespace jk

extern "C" int jk_propagation_topk_forward(const void* row_proj, const void* col_proj, int64_t batch, int64_t n_rows,
                                           int64_t n_cols, int64_t rp, int proj_dtype, const void* col_state,
                                           const void* col_sender, int state_dtype, const void* col_val, int64_t dim,
                                           int val_dtype, int64_t k, int64_t window, float score_bias,
                                           const float* bias_dev, int compress, void* out_state, void* out_val,
                                           int out_dtype, float* out_scores, int64_t* out_index, jk_stream_t stream) {
  return jk::topk::gather_forward(row_proj, col_proj, batch, n_rows, n_cols, rp, proj_dtype, col_state, col_sender,
                                  state_dtype, col_val, dim, val_dtype, k, window, score_bias, bias_dev, compress,
                                  out_state, out_val, out_dtype, out_scores, out_index, nullptr, 0, n_rows, stream);
}

extern "C" int jk_propagation_topk_forward_mh(const void* row_proj, const void* col_proj, int64_t batch,
                                              int64_t n_rows, int64_t n_cols, int64_t rp, int proj_dtype,
                                              const void* col_state, const void* col_sender, int state_dtype,
                                              const void* col_val, int64_t dim, int val_dtype, int64_t k,
                                              int64_t window, float score_bias, const float* bias_dev, int compress,
                                              void* out_state, void* out_val, int out_dtype, float* out_scores,
                                              int64_t* out_index, const jk_heads_t* heads, jk_stream_t stream) {
  if (heads == nullptr) return JK_ERR_BAD_ARG;
  return jk::topk::gather_forward(row_proj, col_proj, batch, n_rows, n_cols, rp, proj_dtype, col_state, col_sender,
                                  state_dtype, col_val, dim, val_dtype, k, window, score_bias, bias_dev, compress,
                                  out_state, out_val, out_dtype, out_scores, out_index, heads, 0, n_rows, stream);
}

extern "C" int jk_propagation_topk_rows_forward(const void* row_proj, const void* col_proj, int64_t batch,
                                                int64_t n_rows, int64_t row_begin, int64_t row_count, int64_t n_cols,
                                                int64_t rp, int proj_dtype, const void* col_state,
                                                const void* col_sender, int state_dtype, const void* col_val,
                                                int64_t dim, int val_dtype, int64_t k, int64_t window,
                                                float score_bias, const float* bias_dev, int compress, void* out_state,
                                                void* out_val, int out_dtype, float* out_scores, int64_t* out_index,
                                                jk_stream_t stream) {
  return jk::topk::gather_forward(row_proj, col_proj, batch, n_rows, n_cols, rp, proj_dtype, col_state, col_sender,
                                  state_dtype, col_val, dim, val_dtype, k, window, score_bias, bias_dev, compress,
                                  out_state, out_val, out_dtype, out_scores, out_index, nullptr, row_begin, row_count,
                                  stream);
}

extern "C" int jk_transition_query_topk_forward(const void* query_proj, const void* source_proj, int64_t batch,
                                                int64_t n_query, int64_t n_source, int64_t rp, int proj_dtype,
                                                const void* source_state, const void* source_sender, int state_dtype,
                                                const void* source_val, int64_t dim, int val_dtype, int64_t k,
                                                float score_bias, const float* bias_dev, int compress,
                                                void* out_state, void* out_val, int out_dtype, float* out_scores,
                                                int64_t* out_index, jk_stream_t stream) {
  return jk::topk::gather_forward(query_proj, source_proj, batch, n_query, n_source, rp, proj_dtype, source_state,
                                  source_sender, state_dtype, source_val, dim, val_dtype, k, -1, score_bias, bias_dev,
                                  compress, out_state, out_val, out_dtype, out_scores, out_index, nullptr, 0, n_query, stream);
}

extern "C" int jk_transition_query_topk_forward_mh(const void* query_proj, const void* source_proj, int64_t batch,
                                                   int64_t n_query, int64_t n_source, int64_t rp, int proj_dtype,
                                                   const void* source_state, const void* source_sender,
                                                   int state_dtype, const void* source_val, int64_t dim,
                                                   int val_dtype, int64_t k, float score_bias, const float* bias_dev,
                                                   int compress, void* out_state, void* out_val, int out_dtype,
                                                   float* out_scores, int64_t* out_index, const jk_heads_t* heads,
                                                   jk_stream_t stream) {
  if (heads == nullptr) return JK_ERR_BAD_ARG;
  return jk::topk::gather_forward(query_proj, source_proj, batch, n_query, n_source, rp, proj_dtype, source_state,
                                  source_sender, state_dtype, source_val, dim, val_dtype, k, -1, score_bias, bias_dev,
                                  compress, out_state, out_val, out_dtype, out_scores, out_index, heads, 0, n_query, stream);
}

extern "C" int jk_transition_pairwise_topk_forward(const void* src_proj, const void* dst_proj, int64_t batch,
                                                   int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                                   const void* src_state, const void* src_sender, int state_dtype,
                                                   const void* src_val, int64_t dim, int val_dtype, int64_t k,
                                                   float score_bias, const float* bias_dev, int compress,
                                                   float* accum, void* out_state, void* out_val, int out_dtype,
                                                   jk_stream_t stream) {
  return jk::topk::scatter_forward(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, src_state, src_sender,
                                   state_dtype, src_val, dim, val_dtype, k, score_bias, bias_dev, compress, accum,
                                   out_state, out_val, out_dtype, nullptr, stream);
}

extern "C" int jk_transition_pairwise_topk_forward_mh(const void* src_proj, const void* dst_proj, int64_t batch,
                                                      int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                                      const void* src_state, const void* src_sender, int state_dtype,
                                                      const void* src_val, int64_t dim, int val_dtype, int64_t k,
                                                      float score_bias, const float* bias_dev, int compress,
                                                      float* accum, void* out_state, void* out_val, int out_dtype,
                                                      const jk_heads_t* heads, jk_stream_t stream) {
  if (heads == nullptr) return JK_ERR_BAD_ARG;
  return jk::topk::scatter_forward(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, src_state, src_sender,
                                   state_dtype, src_val, dim, val_dtype, k, score_bias, bias_dev, compress, accum,
                                   out_state, out_val, out_dtype, heads, stream);
}



extern "C" int jk_transition_pairwise_topk_routes(const void* src_proj, const void* dst_proj, int64_t batch,
                                                  int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                                  const void* src_sender, int state_dtype, int64_t k,
                                                  float score_bias, const float* bias_dev, int compress,
                                                  float* routes, float* out_scores, int64_t* out_index,
                                                  jk_stream_t stream) {
  return jk::topk::routes_forward(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, src_sender, state_dtype, k,
                                  score_bias, bias_dev, compress, routes, out_scores, out_index, nullptr, stream);
}

extern "C" int jk_transition_pairwise_topk_routes_mh(const void* src_proj, const void* dst_proj, int64_t batch,
                                                     int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                                     const void* src_sender, int state_dtype, int64_t k,
                                                     float score_bias, const float* bias_dev, int compress,
                                                     float* routes, float* out_scores, int64_t* out_index,
                                                     const jk_heads_t* heads, jk_stream_t stream) {
  if (heads == nullptr) return JK_ERR_BAD_ARG;
  return jk::topk::routes_forward(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, src_sender, state_dtype, k,
                                  score_bias, bias_dev, compress, routes, out_scores, out_index, heads, stream);
}

namespace jk {
JK_ERROR_READER(read_error_topk)
}  // namespace jk
