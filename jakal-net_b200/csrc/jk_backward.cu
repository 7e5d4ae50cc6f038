// Backward kernels of the top-k operators (the training side of the hot path).
//
// The reference trains its per-source sparse transition through an autograd Function whose
// backward calls, from the native module, the compressor backwards and the gradient of the
// low-rank route scores (native_backend.py:4408-4601; the CUDA kernels it replaces are
// native/jakal_net_native_cuda.cu:2112-2320). The row-wise pieces live here:
//   * softmax backward        g_s = r * (g_r - sum(r * g_r))       (per row of routes)
//   * softsign backward       g_s = g_e / (1 + |s|)^2              (elementwise)
//   * top-k reduce backward   g_e[q, e] = g_state[q] * state[idx] + g_val[q, :] . val[idx, :]
//                             (the gather half of the reduce's backward; the scatter half
//                             is a GEMM of the dense edge matrix, see jk_topk_to_dense)
//   * top-k to dense          dense[r, idx[r, e]] += w[r, e]  (k non-zeros per row; the dense
//                             matrix turns every scatter of the backward into a GEMM with a
//                             fixed summation order)
// One warp per row for the row-wise kernels; f32 accumulation throughout.
#include "jk_host.h"
#include "jk_sm100.cuh"

namespace jk {
namespace bwd {

constexpr int kWarpsPerBlock = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void softmax_backward_kernel(const void* routes, const void* grad, void* out, int64_t rows, int64_t n,
                                        int dtype) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t base = row * n;
  float dot = 0.f;
  for (int64_t j = lane; j < n; j += 32) dot = fmaf(ld_elem(routes, base + j, dtype), ld_elem(grad, base + j, dtype), dot);
  dot = warp_sum(dot);
  for (int64_t j = lane; j < n; j += 32) {
    const float r = ld_elem(routes, base + j, dtype);
    st_elem(out, base + j, dtype, r * (ld_elem(grad, base + j, dtype) - dot));
  }
}

__global__ void softsign_backward_kernel(const void* scores, const void* grad, void* out, int64_t n, int dtype) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float d = 1.f + fabsf(ld_elem(scores, i, dtype));
    st_elem(out, i, dtype, ld_elem(grad, i, dtype) / (d * d));
  }
}

// grad_edges[b, q, e] = grad_state[b, q] * state[b, idx] + sum_d grad_val[b, q, d] * val[b, idx, d]
// (idx = indices[b, q, e]; idx < 0: 0). One warp per (b, q) row, lanes over d.
__global__ void topk_reduce_backward_kernel(const int64_t* indices, const void* state, const void* val,
                                            const void* grad_state, const void* grad_val, void* grad_edges,
                                            int64_t rows, int64_t n_rows_per_batch, int64_t n_src, int64_t k,
                                            int64_t dim, int dtype, int out_dtype) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t b = row / n_rows_per_batch;
  const float gs = ld_elem(grad_state, row, dtype);
  for (int64_t e = 0; e < k; ++e) {
    const int64_t j = indices[row * k + e];
    float acc = 0.f;
    if (j >= 0) {
      const int64_t src = b * n_src + j;
      for (int64_t d = lane; d < dim; d += 32)
        acc = fmaf(ld_elem(grad_val, row * dim + d, dtype), ld_elem(val, src * dim + d, dtype), acc);
      acc = warp_sum(acc);
      acc = fmaf(gs, ld_elem(state, src, dtype), acc);
    }
    if (lane == 0) st_elem(grad_edges, row * k + e, out_dtype, acc);
  }
}

// dense[row, indices[row, e]] += w[row, e] for every e with indices >= 0 (dense zeroed by
// the caller). A selection names each column once, but a window's padded index lists repeat a
// placeholder column with zero weight: adding keeps those entries exact (adding zero to the
// one real weight changes nothing, whatever the order).
__global__ void topk_to_dense_kernel(const float* w, const int64_t* indices, float* dense, int64_t rows, int64_t k,
                                     int64_t n_cols) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < rows * k; i += stride) {
    const int64_t j = indices[i];
    const float v = w[i];
    if (j >= 0 && j < n_cols && v != 0.f) atomicAdd(dense + (i / k) * n_cols + j, v);
  }
}

inline unsigned grid_for(int64_t work, int per_block) {
  int64_t g = (work + per_block - 1) / per_block;
  if (g > 148 * 64) g = 148 * 64;
  return static_cast<unsigned>(g < 1 ? 1 : g);
}

}  // namespace bwd
}  // namespace jk

extern "C" int jk_softmax_backward(const void* routes, const void* grad_routes, void* grad_scores, int64_t rows,
                                   int64_t n, int dtype, jk_stream_t stream) {
  using namespace jk;
  if (routes == nullptr || grad_routes == nullptr || grad_scores == nullptr) return JK_ERR_BAD_ARG;
  if (dtype < JK_F32 || dtype > JK_F16) return JK_ERR_BAD_DTYPE;
  if (rows < 0 || n < 0) return JK_ERR_BAD_SHAPE;
  if (rows == 0 || n == 0) return JK_OK;
  int st = check_device();
  if (st != JK_OK) return st;
  const unsigned grid = static_cast<unsigned>((rows + bwd::kWarpsPerBlock - 1) / bwd::kWarpsPerBlock);
  bwd::softmax_backward_kernel<<<grid, bwd::kWarpsPerBlock * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      routes, grad_routes, grad_scores, rows, n, dtype);
  return launch_status();
}

extern "C" int jk_softsign_backward(const void* scores, const void* grad_edges, void* grad_scores, int64_t n,
                                    int dtype, jk_stream_t stream) {
  using namespace jk;
  if (scores == nullptr || grad_edges == nullptr || grad_scores == nullptr) return JK_ERR_BAD_ARG;
  if (dtype < JK_F32 || dtype > JK_F16) return JK_ERR_BAD_DTYPE;
  if (n < 0) return JK_ERR_BAD_SHAPE;
  if (n == 0) return JK_OK;
  int st = check_device();
  if (st != JK_OK) return st;
  bwd::softsign_backward_kernel<<<bwd::grid_for(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      scores, grad_edges, grad_scores, n, dtype);
  return launch_status();
}

extern "C" int jk_topk_reduce_backward_edges(const int64_t* indices, const void* state, const void* val,
                                             const void* grad_state, const void* grad_val, void* grad_edges,
                                             int64_t batch, int64_t n_rows, int64_t n_src, int64_t k, int64_t dim,
                                             int dtype, int out_dtype, jk_stream_t stream) {
  using namespace jk;
  if (indices == nullptr || state == nullptr || val == nullptr || grad_state == nullptr || grad_val == nullptr ||
      grad_edges == nullptr)
    return JK_ERR_BAD_ARG;
  if (dtype < JK_F32 || dtype > JK_F16 || out_dtype < JK_F32 || out_dtype > JK_F16) return JK_ERR_BAD_DTYPE;
  if (batch < 0 || n_rows < 0 || n_src < 0 || k < 0 || dim < 0) return JK_ERR_BAD_SHAPE;
  const int64_t rows = batch * n_rows;
  if (rows == 0 || k == 0) return JK_OK;
  int st = check_device();
  if (st != JK_OK) return st;
  const unsigned grid = static_cast<unsigned>((rows + bwd::kWarpsPerBlock - 1) / bwd::kWarpsPerBlock);
  bwd::topk_reduce_backward_kernel<<<grid, bwd::kWarpsPerBlock * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      indices, state, val, grad_state, grad_val, grad_edges, rows, n_rows, n_src, k, dim, dtype, out_dtype);
  return launch_status();
}

extern "C" int jk_topk_to_dense(const float* w, const int64_t* indices, float* dense, int64_t rows, int64_t k,
                                int64_t n_cols, jk_stream_t stream) {
  using namespace jk;
  if (w == nullptr || indices == nullptr || dense == nullptr) return JK_ERR_BAD_ARG;
  if (rows < 0 || k < 0 || n_cols <= 0) return JK_ERR_BAD_SHAPE;
  if (rows == 0 || k == 0) return JK_OK;
  int st = check_device();
  if (st != JK_OK) return st;
  bwd::topk_to_dense_kernel<<<bwd::grid_for(rows * k, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      w, indices, dense, rows, k, n_cols);
  return launch_status();
}
