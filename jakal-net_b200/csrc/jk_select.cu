// Select-aggregate over materialised score rows: the any-k / any-rank form of the fused
// top-k kernel (jk_topk.cu).
//
// The fused kernel keeps scores on chip and needs k <= 64, a padded projection rank <= 128
// and 16-bit (or three-plane f32, rank <= 32) projections. Everything else the reference
// accepts -- k up to the row length, any score rank, f32 projections of any rank, diagonal
// scorers wider than 128 -- goes through this kernel: the caller materialises a block of f32
// score rows (a plain GEMM of the projections), and one CTA per row then
//   1. finds the k-th largest visible score exactly, by a 4-pass radix select (8 bits per
//      pass) over order-preserving 32-bit keys, histogrammed in shared memory;
//   2. compacts the survivors in ascending column order (block prefix sums), keeping the
//      lowest columns among keys equal to the threshold (tie order: higher score first,
//      then lower column);
//   3. forms the row statistics of the edge / route compressor with block reductions
//      (softmax max and sum, signed-abs max and sum, the signed_entmax15 threshold by the
//      same fixed-point iteration as the fused kernel);
//   4. aggregates: gather (propagation / per-query transition: out[t] = sum_e w_e v[col_e])
//      or scatter (per-source transition: acc[col_e] += w_e v[t], f32 atomics).
// Reference behaviour it reproduces: the blocked top-k paths that take any k,
// native/jakal_net_native.cpp:6390-6447 (propagation), :6916-7087 (per-source transition)
// and :7089-7246 (per-query transition), with the edges of propagation.py:67-88 and the
// routes of transition.py:53-76.
#include "jk_host.h"
#include "jk_sm100.cuh"

#include <cfloat>

namespace jk {
namespace sel {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kAcc = 8;  // value columns per thread per dim chunk (chunk = 2048 columns)

struct Params {
  const float* scores;  // [B, row_count, n_cols], rows row_begin .. row_begin + row_count
  int64_t n_rows, n_cols, row_begin, row_count;
  int64_t k, window;
  float bias;
  const float* bias_dev;
  int compress;
  int scatter;
  const void* state;
  const void* sender;
  int state_dtype;
  const void* val;
  int64_t dim;
  int val_dtype;
  void* out_state;  // gather: [B, n_rows] / [B, n_rows, dim] in out_dtype
  void* out_val;
  int out_dtype;
  float* acc_state;  // scatter: f32 [B, n_cols] / [B, n_cols, dim]
  float* acc_val;
  float* sel_score;     // [B, row_count, k]: score + bias, ascending column order, -inf pad
  int64_t* sel_index;   // [B, row_count, k]: column, -1 pad
};

// Order-preserving key: a larger key is a larger score (NaN above +inf, as torch.topk).
__device__ __forceinline__ uint32_t order_key(float s) {
  const uint32_t u = __float_as_uint(s);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float sgnf(float x) { return x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f); }

struct SumOp {
  __device__ float operator()(float a, float b) const { return a + b; }
};
struct MaxOp {
  __device__ float operator()(float a, float b) const { return fmaxf(a, b); }
};

// Reduction over the block; every thread gets the result. `red` holds kWarps floats.
template <typename Op>
__device__ float block_reduce(float v, Op op, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();  // the previous reduction's readers are done with red
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < kWarps; ++i) r = op(r, red[i]);
  return r;
}

// Exclusive prefix sum of one int per thread over the block; *total gets the sum.
__device__ int block_scan(int x, int* wsum, int* total) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  int inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (l >= o) inc += y;
  }
  __syncthreads();
  if (l == 31) wsum[w] = inc;
  __syncthreads();
  int off = 0, tot = 0;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) {
    off += i < w ? wsum[i] : 0;
    tot += wsum[i];
  }
  *total = tot;
  return off + inc - x;
}

// Row statistics of a compressor; edge(x) turns a selected score (bias included) into its
// edge / route weight.
struct Stats {
  int compress;
  float m, inv, zmax, tau;
  __device__ __forceinline__ float edge(float x) const {
    if (compress == JK_SOFTSIGN) return x / (1.f + fabsf(x));
    if (compress == JK_SOFTMAX) return expf(x - m) * inv;
    if (compress == JK_SIGNED_ABS_SOFTMAX) return sgnf(x) * expf(fabsf(x) - m) * inv;
    const float pz = fmaxf((fabsf(x) - zmax) * 0.5f - tau, 0.f);
    return sgnf(x) * pz * pz * inv;
  }
};

__device__ Stats row_stats(const float* sc, int64_t n, int compress, float* red) {
  Stats st{compress, 0.f, 0.f, 0.f, 0.f};
  if (compress == JK_SOFTSIGN || n <= 0) return st;
  const int tid = threadIdx.x;
  if (compress == JK_SOFTMAX) {
    float m = -INFINITY;
    for (int64_t e = tid; e < n; e += kThreads) m = fmaxf(m, sc[e]);
    m = block_reduce(m, MaxOp{}, red);
    float z = 0.f;
    for (int64_t e = tid; e < n; e += kThreads) z += expf(sc[e] - m);
    z = block_reduce(z, SumOp{}, red);
    st.m = m;
    st.inv = 1.f / z;
  } else if (compress == JK_SIGNED_ABS_SOFTMAX) {
    float m = 0.f;
    for (int64_t e = tid; e < n; e += kThreads) m = fmaxf(m, fabsf(sc[e]));
    m = block_reduce(m, MaxOp{}, red);
    float z = 0.f;
    for (int64_t e = tid; e < n; e += kThreads) z += expf(fabsf(sc[e]) - m);
    z = block_reduce(z, SumOp{}, red);
    st.m = m;
    st.inv = 1.f / z;
  } else {
    // sign(s) * entmax15(|s|) (kernels.py:155-236): z = (|s| - max|s|) / 2; tau solves
    // sum_{z > tau} (z - tau)^2 = 1, found as in the fused kernel by the fixed-point
    // iteration over the support with tau = mean - sqrt(max(0, (1 - rho (msq - mean^2)) / rho)).
    float zmax = 0.f;
    for (int64_t e = tid; e < n; e += kThreads) zmax = fmaxf(zmax, fabsf(sc[e]));
    zmax = block_reduce(zmax, MaxOp{}, red);
    float tau = -INFINITY;
    for (int64_t iter = 0; iter <= n; ++iter) {
      float sum = 0.f, sum_sq = 0.f, rho = 0.f;
      for (int64_t e = tid; e < n; e += kThreads) {
        const float z = (fabsf(sc[e]) - zmax) * 0.5f;
        if (z > tau || iter == 0) {
          sum += z;
          sum_sq += z * z;
          rho += 1.f;
        }
      }
      sum = block_reduce(sum, SumOp{}, red);
      sum_sq = block_reduce(sum_sq, SumOp{}, red);
      rho = block_reduce(rho, SumOp{}, red);
      const float mean = sum / rho;
      const float mean_sq = sum_sq / rho;
      const float delta = fmaxf((1.f - rho * (mean_sq - mean * mean)) / rho, 0.f);
      const float next = mean - sqrtf(delta);
      if (iter > 0 && next == tau) break;
      tau = next;
    }
    float zs = 0.f;
    for (int64_t e = tid; e < n; e += kThreads) {
      const float pz = fmaxf((fabsf(sc[e]) - zmax) * 0.5f - tau, 0.f);
      zs += pz * pz;
    }
    zs = block_reduce(zs, SumOp{}, red);
    st.zmax = zmax;
    st.tau = tau;
    st.inv = zs > 0.f ? 1.f / fmaxf(zs, FLT_EPSILON) : 0.f;
  }
  return st;
}

__global__ void __launch_bounds__(kThreads) select_kernel(const Params p) {
  __shared__ int hist[256];
  __shared__ float red[kWarps];
  __shared__ int wsum[kWarps];
  __shared__ uint32_t s_prefix;
  __shared__ long long s_remaining;
  __shared__ float s_w[kThreads];
  __shared__ long long s_j[kThreads];

  const int tid = threadIdx.x;
  const int64_t r = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int64_t t = p.row_begin + r;  // global row
  const float* srow = p.scores + (b * p.row_count + r) * p.n_cols;
  int64_t lo = 0, hi = p.n_cols;  // visible columns [lo, hi)
  if (p.window >= 0) {
    lo = t - p.window > 0 ? t - p.window : 0;
    hi = t + 1 < p.n_cols ? t + 1 : p.n_cols;
    if (hi < lo) hi = lo;
  }
  const int64_t n_vis = hi - lo;
  const int64_t kk = p.k < n_vis ? p.k : n_vis;
  const float bias = p.bias + (p.bias_dev != nullptr ? *p.bias_dev : 0.f);
  float* osc = p.sel_score + (b * p.row_count + r) * p.k;
  int64_t* oix = p.sel_index + (b * p.row_count + r) * p.k;
  for (int64_t e = kk + tid; e < p.k; e += kThreads) {
    osc[e] = -INFINITY;
    oix[e] = -1;
  }

  // 1. threshold key: the kk-th largest visible key, and how many keys equal to it to keep
  const bool take_all = kk == n_vis;
  uint32_t thr = 0;
  int64_t need_eq = 0;
  if (!take_all) {
    uint32_t prefix = 0, mask = 0;
    int64_t remaining = kk;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += kThreads) hist[i] = 0;
      __syncthreads();
      for (int64_t j = lo + tid; j < hi; j += kThreads) {
        const uint32_t key = order_key(srow[j]);
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1);
      }
      __syncthreads();
      if (tid == 0) {
        int64_t above = 0;
        int bin = 255;
        for (; bin > 0; --bin) {
          if (above + hist[bin] >= remaining) break;
          above += hist[bin];
        }
        s_prefix = prefix | (static_cast<uint32_t>(bin) << shift);
        s_remaining = remaining - above;
      }
      __syncthreads();
      prefix = s_prefix;
      remaining = s_remaining;
      mask |= 255u << shift;
    }
    thr = prefix;
    need_eq = remaining;
  }

  // 2. survivors in ascending column order
  int64_t taken = 0, eq_seen = 0;
  for (int64_t base = lo; base < hi && taken < kk; base += kThreads) {
    const int64_t j = base + tid;
    const bool in = j < hi;
    const float s = in ? srow[j] : 0.f;
    const uint32_t key = in ? order_key(s) : 0u;
    const bool gt = in && (take_all || key > thr);
    const bool eq = in && !take_all && key == thr;
    int eq_tot = 0, tk_tot = 0;
    const int eq_rank = block_scan(eq ? 1 : 0, wsum, &eq_tot);
    const bool take = gt || (eq && eq_seen + eq_rank < need_eq);
    const int pos = block_scan(take ? 1 : 0, wsum, &tk_tot);
    if (take) {
      osc[taken + pos] = s + bias;
      oix[taken + pos] = j;
    }
    eq_seen += eq_tot;
    taken += tk_tot;
  }
  __syncthreads();  // the survivors written above are read by every thread below

  // 3. compressor statistics over the kk survivors
  const Stats st = row_stats(osc, kk, p.compress, red);

  // 4. aggregate
  const int64_t D = p.dim;
  if (!p.scatter) {
    float st_part = 0.f;
    const int64_t row_out = b * p.n_rows + t;
    for (int64_t d0 = 0; d0 < D; d0 += int64_t(kThreads) * kAcc) {
      float acc[kAcc];
#pragma unroll
      for (int a = 0; a < kAcc; ++a) acc[a] = 0.f;
      for (int64_t e0 = 0; e0 < kk; e0 += kThreads) {
        __syncthreads();  // the previous chunk's readers are done with s_w / s_j
        const int64_t e = e0 + tid;
        if (e < kk) {
          const int64_t col = b * p.n_cols + oix[e];
          float w = st.edge(osc[e]);
          if (p.sender != nullptr) w *= ld_elem(p.sender, col, p.state_dtype);
          s_w[tid] = w;
          s_j[tid] = col;
          if (d0 == 0) st_part = fmaf(w, ld_elem(p.state, col, p.state_dtype), st_part);
        }
        __syncthreads();
        const int n = kk - e0 < kThreads ? static_cast<int>(kk - e0) : kThreads;
        for (int u = 0; u < n; ++u) {
          const float w = s_w[u];
          const int64_t vrow = s_j[u] * D;
#pragma unroll
          for (int a = 0; a < kAcc; ++a) {
            const int64_t d = d0 + a * kThreads + tid;
            if (d < D) acc[a] = fmaf(w, ld_elem(p.val, vrow + d, p.val_dtype), acc[a]);
          }
        }
      }
#pragma unroll
      for (int a = 0; a < kAcc; ++a) {
        const int64_t d = d0 + a * kThreads + tid;
        if (d < D) st_elem(p.out_val, row_out * D + d, p.out_dtype, acc[a]);
      }
    }
    const float total = block_reduce(st_part, SumOp{}, red);
    if (tid == 0) st_elem(p.out_state, row_out, p.out_dtype, total);
  } else {
    const int64_t src = b * p.n_rows + t;
    const float sender = p.sender != nullptr ? ld_elem(p.sender, src, p.state_dtype) : 1.f;
    const float sstate = ld_elem(p.state, src, p.state_dtype);
    for (int64_t d0 = 0; d0 < D; d0 += int64_t(kThreads) * kAcc) {
      float v[kAcc];
#pragma unroll
      for (int a = 0; a < kAcc; ++a) {
        const int64_t d = d0 + a * kThreads + tid;
        v[a] = d < D ? ld_elem(p.val, src * D + d, p.val_dtype) : 0.f;
      }
      for (int64_t e0 = 0; e0 < kk; e0 += kThreads) {
        __syncthreads();
        const int64_t e = e0 + tid;
        if (e < kk) {
          const int64_t dst = b * p.n_cols + oix[e];
          const float w = st.edge(osc[e]) * sender;
          s_w[tid] = w;
          s_j[tid] = dst;
          if (d0 == 0) atomicAdd(p.acc_state + dst, w * sstate);
        }
        __syncthreads();
        const int n = kk - e0 < kThreads ? static_cast<int>(kk - e0) : kThreads;
        for (int u = 0; u < n; ++u) {
          const float w = s_w[u];
          float* arow = p.acc_val + s_j[u] * D;
#pragma unroll
          for (int a = 0; a < kAcc; ++a) {
            const int64_t d = d0 + a * kThreads + tid;
            if (d < D) atomicAdd(arow + d, w * v[a]);
          }
        }
      }
    }
  }
}

}  // namespace sel
}  // namespace jk

extern "C" int jk_select_aggregate_forward(const float* scores, int64_t batch, int64_t n_rows, int64_t n_cols,
                                           int64_t row_begin, int64_t row_count, const void* state,
                                           const void* sender, int state_dtype, const void* val, int64_t dim,
                                           int val_dtype, int64_t k, int64_t window, float score_bias,
                                           const float* bias_dev, int compress, int scatter, void* out_state,
                                           void* out_val, int out_dtype, float* acc_state, float* acc_val,
                                           float* sel_score, int64_t* sel_index, jk_stream_t stream) {
  using namespace jk;
  if (scores == nullptr || state == nullptr || val == nullptr || sel_score == nullptr || sel_index == nullptr)
    return JK_ERR_BAD_ARG;
  if (scatter ? (acc_state == nullptr || acc_val == nullptr) : (out_state == nullptr || out_val == nullptr))
    return JK_ERR_BAD_ARG;
  if (state_dtype < JK_F32 || state_dtype > JK_F16 || val_dtype < JK_F32 || val_dtype > JK_F16 ||
      (!scatter && (out_dtype < JK_F32 || out_dtype > JK_F16)))
    return JK_ERR_BAD_DTYPE;
  if (compress < JK_SOFTSIGN || compress > JK_SOFTMAX) return JK_ERR_UNSUPPORTED_KIND;
  if (batch <= 0 || batch > 65535 || n_rows <= 0 || n_cols <= 0 || dim <= 0) return JK_ERR_BAD_SHAPE;
  if (n_cols > (int64_t(1) << 31) - 1 || row_count <= 0 || row_count > (int64_t(1) << 31) - 1 || row_begin < 0 ||
      row_begin + row_count > n_rows)
    return JK_ERR_BAD_SHAPE;
  if (k < 1 || window < -1) return JK_ERR_BAD_ARG;
  int st = check_device();
  if (st != JK_OK) return st;
  sel::Params p{};
  p.scores = scores;
  p.n_rows = n_rows;
  p.n_cols = n_cols;
  p.row_begin = row_begin;
  p.row_count = row_count;
  p.k = k;
  p.window = window;
  p.bias = score_bias;
  p.bias_dev = bias_dev;
  p.compress = compress;
  p.scatter = scatter ? 1 : 0;
  p.state = state;
  p.sender = sender;
  p.state_dtype = state_dtype;
  p.val = val;
  p.dim = dim;
  p.val_dtype = val_dtype;
  p.out_state = out_state;
  p.out_val = out_val;
  p.out_dtype = out_dtype;
  p.acc_state = acc_state;
  p.acc_val = acc_val;
  p.sel_score = sel_score;
  p.sel_index = sel_index;
  const dim3 grid(static_cast<unsigned>(row_count), static_cast<unsigned>(batch));
  sel::select_kernel<<<grid, sel::kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return launch_status();
}
