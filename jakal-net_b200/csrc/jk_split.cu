// Splits f32 operands into bf16 planes so that the bf16 tcgen05 kernels reproduce f32
// arithmetic:
//   * projections (rank <= 32): x = h + m + l with h = bf16(x), m = bf16(x - h),
//     l = bf16(x - h - m); written as one padded row [h(32) | m(32) | l(32) | 0(32)]
//     (JK_BF16X3, rp = 128). The fused kernels form a score from the six products
//     hh + hm + mh + hl + lh + mm, which leaves an error of order 2^-24 relative -- the
//     accuracy of an f32 dot product;
//   * values: v = hi + lo, hi = bf16(v), lo = bf16(v - hi) (about 16 significant bits; the
//     window kernel multiplies both planes, the edge planes carry the rest).
#include "jk_host.h"
#include "jk_sm100.cuh"

namespace jk {
namespace split {

__global__ void split3_kernel(const float* __restrict__ x, int64_t rows, int rank, __nv_bfloat16* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // (row, col < 32)
  if (i >= rows * 32) return;
  const int64_t row = i >> 5;
  const int c = static_cast<int>(i & 31);
  const float v = c < rank ? x[row * rank + c] : 0.f;
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  const float r1 = v - __bfloat162float(h);
  const __nv_bfloat16 m = __float2bfloat16_rn(r1);
  const __nv_bfloat16 l = __float2bfloat16_rn(r1 - __bfloat162float(m));
  __nv_bfloat16* o = out + row * 128;
  o[c] = h;
  o[32 + c] = m;
  o[64 + c] = l;
  o[96 + c] = __float2bfloat16_rn(0.f);
}

__global__ void split2_kernel(const float* __restrict__ x, int64_t n, __nv_bfloat16* __restrict__ hi,
                              __nv_bfloat16* __restrict__ lo) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = x[i];
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[i] = h;
    lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
  }
}

// out[b, i * rows + r, c] = plane (bits >> i) & 1 (0 = hi, 1 = lo) of v, where v = x[b, r, c]
// for c < cols, extra[b, r] at c == cols (when given), 0 beyond.
__global__ void split_stack_kernel(const float* __restrict__ x, const float* __restrict__ extra, int64_t batch,
                                   int64_t rows, int64_t cols, int64_t out_cols, int nblk, unsigned bits,
                                   __nv_bfloat16* __restrict__ out) {
  // one (batch item, row) per block iteration, the threads across its columns (coalesced)
  for (int64_t br = blockIdx.x; br < batch * rows; br += gridDim.x) {
    const int64_t b = br / rows, r = br - b * rows;
    const float* xr = x + br * cols;
    const float ex = (extra != nullptr) ? extra[br] : 0.f;
    for (int64_t c = threadIdx.x; c < out_cols; c += blockDim.x) {
      const float v = c < cols ? xr[c] : (c == cols ? ex : 0.f);
      const __nv_bfloat16 h = __float2bfloat16_rn(v);
      const __nv_bfloat16 l = __float2bfloat16_rn(v - __bfloat162float(h));
      for (int k = 0; k < nblk; ++k)
        out[((b * nblk + k) * rows + r) * out_cols + c] = ((bits >> k) & 1u) ? l : h;
    }
  }
}

}  // namespace split
}  // namespace jk

extern "C" int jk_split3_bf16(const float* x, int64_t rows, int64_t rank, void* out, jk_stream_t stream) {
  using namespace jk;
  if (x == nullptr || out == nullptr) return JK_ERR_BAD_ARG;
  if (rows <= 0 || rank <= 0 || rank > 32) return JK_ERR_BAD_SHAPE;
  if (!aligned16(out)) return JK_ERR_ALIGNMENT;
  int st = check_device();
  if (st != JK_OK) return st;
  const int64_t work = rows * 32;
  split::split3_kernel<<<static_cast<unsigned>((work + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, rows, static_cast<int>(rank), reinterpret_cast<__nv_bfloat16*>(out));
  return launch_status();
}

extern "C" int jk_split2_bf16(const float* x, int64_t n, void* hi, void* lo, jk_stream_t stream) {
  using namespace jk;
  if (x == nullptr || hi == nullptr || lo == nullptr) return JK_ERR_BAD_ARG;
  if (n <= 0) return JK_ERR_BAD_SHAPE;
  int st = check_device();
  if (st != JK_OK) return st;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  split::split2_kernel<<<static_cast<unsigned>(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, n, reinterpret_cast<__nv_bfloat16*>(hi), reinterpret_cast<__nv_bfloat16*>(lo));
  return launch_status();
}

extern "C" int jk_split_stack_bf16(const float* x, const float* extra_col, int64_t batch, int64_t rows,
                                   int64_t cols, int64_t out_cols, int nblk, unsigned plane_bits, void* out,
                                   jk_stream_t stream) {
  using namespace jk;
  if (x == nullptr || out == nullptr) return JK_ERR_BAD_ARG;
  if (batch <= 0 || rows <= 0 || cols <= 0 || nblk < 1 || nblk > 4) return JK_ERR_BAD_SHAPE;
  if (out_cols < cols + (extra_col != nullptr ? 1 : 0)) return JK_ERR_BAD_SHAPE;
  int st = check_device();
  if (st != JK_OK) return st;
  int64_t blocks = batch * rows;
  if (blocks > 148 * 64) blocks = 148 * 64;
  const int threads = out_cols >= 256 ? 256 : (out_cols >= 128 ? 128 : 64);
  split::split_stack_kernel<<<static_cast<unsigned>(blocks), threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, extra_col, batch, rows, cols, out_cols, nblk, plane_bits, reinterpret_cast<__nv_bfloat16*>(out));
  return launch_status();
}
