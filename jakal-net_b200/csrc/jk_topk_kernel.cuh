// Shared by the fused top-k units (jk_topk.cu and the per-value-type instantiation units
// jk_topk_vt_*.cu, compiled in parallel): the kernel template and its launcher.
#pragma once

// Fused low-rank score -> top-k -> edge compress -> aggregate kernel.
//
// Covers three reference operators that share one structure ("every row picks its k best
// columns by a low-rank bilinear score"):
//   * propagation top-k        native/jakal_net_native_cuda.cu:1029-1183 (per target row,
//                              no mask) and the window-intersect-top-k form
//                              (kernel_common.py:433-456 mask, propagation.py:67-88 edges);
//   * per-query transition     native/jakal_net_native.cpp:7089-7246 (rows = query slots,
//                              softmax over the k picked sources, sender-weighted gather);
//   * per-source transition    native/jakal_net_native_cuda.cu:740-878 (rows = sources,
//                              softmax over the k picked destinations, scatter-add).
//
// Per CTA: 128 rows of one batch item, 10 warps.
//   warp 9 (loader): TMA of the row-side projection tile once, the column-side tiles
//          (128 columns x rp) through a shared-memory ring once per selection pass, and
//          for the tensor-core aggregate the source window's value slices.
//   warp 8 (MMA): tcgen05.mma score tiles (M=128 rows, N=128 columns, K=rp) into one of two
//          TMEM accumulators, so the MMA of one tile overlaps the selection work on the
//          previous one (scores are recomputed per pass, never stored); later the
//          aggregate's E.V MMAs.
//   warps 0-7 (selection): two threads per row (warps w and w+4 read the same TMEM lanes),
//          each owning 64 of the 128 columns of every tile.
//     pass A (only when a row sees more than kCap columns): per-row mean and variance of
//          the visible scores -> a threshold tau expected to pass about k + 3 sqrt(k) + 8
//          columns (normal quantile).
//     pass B: every visible column with score >= tau is appended (predicated stores) to
//          the row's candidate stack of its half -- two stacks in ascending column order.
//     pass C (only if some row of the CTA got fewer than min(k, visible) or more than kCap
//          candidates -- a row far from normal): those rows redo an exact streaming
//          selection, each thread keeping a k-entry min-heap in the row's buffer.
//     select: one warp per two rows ranks the candidates (32-bit scores; 64-bit keys
//          score then lower column for rows with exact ties) and keeps the best k as two
//          ascending column runs.
//   Then the k survivors are compressed into edges (sender weighting and the state sum
//   folded in) and aggregated: a windowed CTA on the tensor cores (sparse 64-row edge
//   tiles in shared memory times value slices, O in TMEM, TMA-stored outputs); otherwise
//   16-byte vector gathers from global memory; the per-source transition scatters with
//   vector atomics instead.
#include "jk_host.h"
#include "jk_sm100.cuh"

#include <cfloat>
#include <climits>
#include <type_traits>

namespace jk {
namespace topk {

#ifdef JK_PHASE_PROFILE
// Debug-only timeline: clock64 stamps of the phase boundaries of every CTA, stored by one
// thread (no atomics, so the timeline is not perturbed). Slot 0 = start, 15 = SM id.
constexpr int kTraceCtas = 4096;
static __device__ long long g_trace[kTraceCtas][32];
#define JK_STAMP(i)                                                                  \
  do {                                                                               \
    const int _cta = blockIdx.y * gridDim.x + blockIdx.x;                            \
    if (_cta < kTraceCtas) g_trace[_cta][i] = clock64();                            \
  } while (0)
#define JK_PHASE_MARK(i, t_prev) \
  do {                           \
    if (threadIdx.x == 0) JK_STAMP((i) + 1); \
  } while (0)
#else
#define JK_STAMP(i) \
  do {              \
  } while (0)
#define JK_PHASE_MARK(i, t_prev) \
  do {                           \
  } while (0)
#endif
#define JK_PHASE_TIME(i, expr) (expr)

constexpr int kRows = 128;      // rows per CTA (MMA M)
constexpr int kCols = 128;      // columns per tile (MMA N)
constexpr int kHalfCols = 64;   // columns per selection thread per tile
constexpr int kCap = 128;       // candidate slots per row
constexpr int kQueue = 4;       // fallback queue slots per thread
constexpr int kStride = 137;    // row stride of the candidate buffer (odd: conflict-free)
constexpr int kSelWarps = 8;    // selection / aggregation warps
constexpr int kMmaWarp = kSelWarps;       // tcgen05.mma issuer
constexpr int kLoadWarp = kSelWarps + 1;  // TMA loader
constexpr int kThreads = (kSelWarps + 2) * 32;
constexpr int kSentinel = INT_MAX;
static_assert(kStride >= kCap + 2 * kQueue, "buffer row holds candidates and both fallback queues");
static_assert(kCap / 2 >= 64, "the score-rank permutation sits behind k <= 64 selected slots");

enum Mode { kGather = 0, kScatter = 1 };

// Tensor-core aggregate: 64 source rows per edge tile, value slices of 128 columns.
constexpr int kEK = 64;       // source rows per edge tile (MMA K)
constexpr int kVSlice = 256;  // value columns per slice (MMA N)
constexpr int kVBufs = 2;     // value-slice buffers
constexpr int kVBufBytes = kEK * kVSlice * 2;  // 32 KB: kVSlice / 64 boxes of 64 rows x 64 columns
constexpr int kOCols = 512;   // TMEM columns of the aggregate's accumulator O (dim <= 512)
// Edge tiles: two buffers of 32 KB at the start of region 0, each a hi plane then a lo plane
// of 128 rows x 64 K elements in the K-major 128-byte-swizzled operand layout.
constexpr int kETile = 32768;

// Start (in floats, 16-byte aligned) of a row's packed gather table: (weight, column) pairs
// written over the row's candidate values once the edges are final.
__device__ __forceinline__ int gtab_off(int row) { return (row * kStride + 3) & ~3; }

// TMEM score buffers: two of 128 columns per head while they fit the 512 columns, else one.
__host__ __device__ constexpr int score_buffers(int heads) { return heads <= 2 ? 2 : 1; }

struct Params {
  int64_t n_rows, n_cols, rp, dim;
  int k;
  int64_t window;  // < 0: no mask
  int64_t row_begin, row_count;  // the launch's row block (row_begin a multiple of kRows)
  float bias;
  const float* bias_dev;
  int compress;
  int state_dtype, val_dtype, out_dtype;
  int slab_ok;  // tm_val is valid (windowed gather of 16-bit values, dim % 64 == 0)
  int tma_out;  // tm_out is valid: the tensor-core aggregate stores 16-bit outputs by TMA
  int split3;   // projections are the three-plane bf16 split of f32 values
  // multi-head scorer (heads > 1): head h owns K steps [h * kph, (h + 1) * kph) and its own
  // TMEM plane; the planes are combined (JK_HEADS_*) with head_bias as they are read
  int heads, kph, combine;
  const float* head_bias;
  const void* col_state;
  const void* col_val;
  const void* col_sender;
  // gather outputs
  void* out_state;
  void* out_val;
  float* out_scores;
  int64_t* out_index;
  // scatter: f32 accumulators [B, n_cols] and [B, n_cols, dim]; the row side supplies
  // state / value / sender (col_state / col_val / col_sender are indexed by the row).
  float* acc_state;
  float* acc_val;
  // scatter, routes form: the compressed, sender-weighted route of every selected
  // (source row, destination column) is written to routes [B, n_rows, n_cols] (f32, zeroed
  // by the caller) instead of being scatter-added; the aggregate is then a plain GEMM.
  float* routes;
};

__device__ __forceinline__ bool worse(float av, int ai, float bv, int bi) {
  return av < bv || (av == bv && ai > bi);
}

// A run of (value, index) slots of one row in the candidate buffer.
struct Lane {
  float* v;
  int* i;
  __device__ __forceinline__ float& val(int slot) const { return v[slot]; }
  __device__ __forceinline__ int& idx(int slot) const { return i[slot]; }
};

// Sift (x, id) down from the root of a min-heap of size n ("min" = worst).
__device__ __forceinline__ void heap_sift_root(const Lane& h, int n, float x, int id) {
  int pos = 0;
  while (true) {
    int c = 2 * pos + 1;
    if (c >= n) break;
    float cv = h.val(c);
    int ci = h.idx(c);
    if (c + 1 < n) {
      const float rv = h.val(c + 1);
      const int ri = h.idx(c + 1);
      if (worse(rv, ri, cv, ci)) {
        c = c + 1;
        cv = rv;
        ci = ri;
      }
    }
    if (!worse(cv, ci, x, id)) break;
    h.val(pos) = cv;
    h.idx(pos) = ci;
    pos = c;
  }
  h.val(pos) = x;
  h.idx(pos) = id;
}

// Merges the queued candidates into the heap; returns the new root value.
__device__ __forceinline__ float flush_queue(const Lane& h, const Lane& q, int k, int& qn) {
  float root_v = h.val(0);
  int root_i = h.idx(0);
  for (int e = 0; e < qn; ++e) {
    const float x = q.val(e);
    const int id = q.idx(e);
    if (worse(root_v, root_i, x, id)) {
      heap_sift_root(h, k, x, id);
      root_v = h.val(0);
      root_i = h.idx(0);
    }
  }
  qn = 0;
  return root_v;
}

__device__ __forceinline__ float sgn(float x) { return x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f); }

// Replaces f.val(0..n) (the selected scores, bias included, any order) by compressed edges.
static __device__ void compress_row(const Lane& f, int n, int compress) {
  if (n <= 0) return;
  if (compress == JK_SOFTSIGN) {
    for (int e = 0; e < n; ++e) {
      const float x = f.val(e);
      f.val(e) = x / (1.f + fabsf(x));
    }
  } else if (compress == JK_SOFTMAX) {
    float m = f.val(0);
    for (int e = 1; e < n; ++e) m = fmaxf(m, f.val(e));
    float z = 0.f;
    for (int e = 0; e < n; ++e) z += expf(f.val(e) - m);
    const float inv = 1.f / z;
    for (int e = 0; e < n; ++e) f.val(e) = expf(f.val(e) - m) * inv;
  } else if (compress == JK_SIGNED_ABS_SOFTMAX) {
    float m = 0.f;
    for (int e = 0; e < n; ++e) m = fmaxf(m, fabsf(f.val(e)));
    float z = 0.f;
    for (int e = 0; e < n; ++e) z += expf(fabsf(f.val(e)) - m);
    const float inv = 1.f / z;
    for (int e = 0; e < n; ++e) {
      const float x = f.val(e);
      f.val(e) = sgn(x) * expf(fabsf(x) - m) * inv;
    }
  } else {
    // sign(s) * entmax15(|s|) (kernels.py:155-236). z = (|s| - max|s|) / 2; the threshold
    // tau solves sum_{z_j > tau} (z_j - tau)^2 = 1. The reference finds the support by
    // sorting; here the support is found by the equivalent fixed-point iteration (start
    // from all entries, drop those at or below tau, recompute) with the same closed form
    // tau = mean - sqrt(max(0, (1 - rho * (mean_sq - mean^2)) / rho)) over the support.
    float zmax = 0.f;
    for (int e = 0; e < n; ++e) zmax = fmaxf(zmax, fabsf(f.val(e)));
    float tau = -INFINITY;
    for (int iter = 0; iter < n + 1; ++iter) {
      float sum = 0.f, sum_sq = 0.f;
      int rho = 0;
      for (int e = 0; e < n; ++e) {
        const float z = (fabsf(f.val(e)) - zmax) * 0.5f;
        if (z > tau || iter == 0) {
          sum += z;
          sum_sq += z * z;
          ++rho;
        }
      }
      const float r = static_cast<float>(rho);
      const float mean = sum / r;
      const float mean_sq = sum_sq / r;
      const float delta = fmaxf((1.f - r * (mean_sq - mean * mean)) / r, 0.f);
      const float next = mean - sqrtf(delta);
      if (iter > 0 && next == tau) break;
      tau = next;
    }
    float z_sum = 0.f;
    for (int e = 0; e < n; ++e) {
      const float pz = fmaxf((fabsf(f.val(e)) - zmax) * 0.5f - tau, 0.f);
      z_sum += pz * pz;
    }
    const float inv = z_sum > 0.f ? 1.f / fmaxf(z_sum, FLT_EPSILON) : 0.f;
    for (int e = 0; e < n; ++e) {
      const float x = f.val(e);
      const float pz = fmaxf((fabsf(x) - zmax) * 0.5f - tau, 0.f);
      f.val(e) = sgn(x) * pz * pz * inv;
    }
  }
}

// ---------------------------------------------------------------- value loads / stores
template <typename VT>
__device__ __forceinline__ void widen8(const uint4& u, float (&f)[8]);

template <>
__device__ __forceinline__ void widen8<__nv_bfloat16>(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <>
__device__ __forceinline__ void widen8<__half>(const uint4& u, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

template <>
__device__ __forceinline__ void widen8<float>(const uint4&, float (&f)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = 0.f;  // f32 values take the generic path
}

template <typename VT>
__device__ __forceinline__ float2 widen2(uint32_t u);

template <>
__device__ __forceinline__ float2 widen2<__nv_bfloat16>(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}

template <>
__device__ __forceinline__ float2 widen2<__half>(uint32_t u) {
  return __half22float2(*reinterpret_cast<const __half2*>(&u));
}

template <>
__device__ __forceinline__ float2 widen2<float>(uint32_t) {
  return make_float2(0.f, 0.f);
}

__device__ __forceinline__ void store2(void* base, int64_t elem, int dtype, float a, float b) {
  if (dtype == JK_F32) {
    *reinterpret_cast<float2*>(reinterpret_cast<float*>(base) + elem) = make_float2(a, b);
  } else if (dtype == JK_BF16) {
    *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(base) + elem) = __floats2bfloat162_rn(a, b);
  } else {
    *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(base) + elem) = __floats2half2_rn(a, b);
  }
}

// ---------------------------------------------------------------- aggregation
// Generic aggregation of one row by one warp (any dim / f32 values): lanes stride the
// value dimension; the final weights already include the sender strength.
static __device__ void gather_row_generic(const float* tab, int n, int64_t col_base, int64_t row, const Params& p, int lane) {
  const int64_t D = p.dim;
  for (int64_t d0 = 0; d0 < D; d0 += 32) {
    const int64_t d = d0 + lane;
    float acc = 0.f;
    for (int e = 0; e < n; ++e) {
      const int j = __float_as_int(tab[2 * e + 1]);
      if (d < D) acc = fmaf(tab[2 * e], ld_elem(p.col_val, (col_base + j) * D + d, p.val_dtype), acc);
    }
    if (d < D) st_elem(p.out_val, row * D + d, p.out_dtype, acc);
  }
}

// Aggregation of `nrows` rows (tile rows rt0 ..) by one warp from global memory.
//
// Work items are (row, 8-element chunk) pairs of a group of rows spread over the 32
// lanes, so every lane keeps up to 16 independent 16-byte loads in flight per step (8
// items x 2 neighbours) whatever the value width, hiding the L2 / HBM latency of random
// gathers. Accumulation is f32; each item is stored once.
template <typename VT>
__device__ void gather_global(const float* bv, const int* nsel, int rt0, int nrows, int64_t t0, int64_t b,
                              const Params& p, int lane) {
  constexpr int kItems = 8;
  const int64_t D = p.dim;
  const int64_t col_base = b * p.n_cols;
  if ((D % 8) != 0 || D > 8 * 32 * kItems || sizeof(VT) == 4) {
    for (int r = 0; r < nrows; ++r) {
      const int rt = rt0 + r;
      const int64_t row = t0 + rt;
      if (row >= p.n_rows) break;
      gather_row_generic(bv + gtab_off(rt), nsel[rt], col_base, b * p.n_rows + row, p, lane);
    }
    return;
  }
  const VT* vbase = reinterpret_cast<const VT*>(p.col_val) + col_base * D;
  const int nch = static_cast<int>(D / 8);
  int rg = (32 * kItems) / nch;
  if (rg < 1) rg = 1;
  for (int g0 = 0; g0 < nrows; g0 += rg) {
    int rq[kItems], nq[kItems], off[kItems];
    float acc[kItems][8];
    int kmax = 0;
#pragma unroll
    for (int m = 0; m < kItems; ++m) {
      const int it = lane + 32 * m;
      const int r = g0 + it / nch;
      const bool act = it < rg * nch && r < nrows && t0 + rt0 + r < p.n_rows;
      rq[m] = rt0 + (act ? r : 0);
      off[m] = (it % nch) * 8;
      nq[m] = act ? nsel[rt0 + r] : 0;
      kmax = nq[m] > kmax ? nq[m] : kmax;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[m][e] = 0.f;
    }
    kmax = __reduce_max_sync(0xffffffffu, kmax);
    for (int i = 0; i < kmax; i += 2) {
      uint4 raw[kItems][2];
      float w[kItems][2];
#pragma unroll
      for (int m = 0; m < kItems; ++m) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const bool on = i + u < nq[m];
          const float2 wj = *reinterpret_cast<const float2*>(bv + gtab_off(rq[m]) + 2 * (on ? i + u : 0));
          const int j = __float_as_int(wj.y);
          w[m][u] = on ? wj.x : 0.f;
          raw[m][u] = on ? __ldg(reinterpret_cast<const uint4*>(vbase + static_cast<int64_t>(j) * D + off[m]))
                         : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int m = 0; m < kItems; ++m) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          float x[8];
          widen8<VT>(raw[m][u], x);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[m][e] = fmaf(w[m][u], x[e], acc[m][e]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < kItems; ++m) {
      const int it = lane + 32 * m;
      const int r = g0 + it / nch;
      if (it < rg * nch && r < nrows && t0 + rt0 + r < p.n_rows) {
        const int64_t row = b * p.n_rows + t0 + rt0 + r;
        store8(p.out_val, row * D + off[m], p.out_dtype, acc[m]);
      }
    }
  }
}

// Scatter of one source row by one warp into the f32 destination accumulators.
template <typename VT>
__device__ void scatter_row(const Lane& f, int n, int64_t b, int64_t src, const Params& p, int lane) {
  const int64_t D = p.dim;
  float sender = 1.f;
  if (p.col_sender) sender = ld_elem(p.col_sender, src, p.state_dtype);
  if (p.routes != nullptr) {  // routes form: one plain store per selected destination
    float* rrow = p.routes + src * p.n_cols;
    for (int e = lane; e < n; e += 32) rrow[f.idx(e)] = f.val(e) * sender;
    return;
  }
  const float sstate = ld_elem(p.col_state, src, p.state_dtype);
  const bool vec = (D % 8) == 0 && D <= 1024 && sizeof(VT) == 2;
  const int nch = static_cast<int>(D / 8);
  float v[4][8];
  if (vec) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int c = lane + 32 * m;
      if (c < nch) {
        const uint4 u =
            __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const VT*>(p.col_val) + src * D + c * 8));
        widen8<VT>(u, v[m]);
      }
    }
  }
  for (int e = 0; e < n; ++e) {
    const int j = f.idx(e);
    const float w = f.val(e) * sender;
    const int64_t dst = b * p.n_cols + j;
    if (lane == 0) atomicAdd(p.acc_state + dst, w * sstate);
    if (vec) {
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int c = lane + 32 * m;
        if (c < nch) {
          float4* q = reinterpret_cast<float4*>(p.acc_val + dst * D + c * 8);
          atomicAdd(q, make_float4(w * v[m][0], w * v[m][1], w * v[m][2], w * v[m][3]));
          atomicAdd(q + 1, make_float4(w * v[m][4], w * v[m][5], w * v[m][6], w * v[m][7]));
        }
      }
    } else {
      for (int64_t d = lane; d < D; d += 32) {
        atomicAdd(p.acc_val + dst * D + d, w * ld_elem(p.col_val, src * D + d, p.val_dtype));
      }
    }
  }
}

// ---------------------------------------------------------------- warp bitonic selection
// Orderable 64-bit key: larger = better (higher score, then lower column).
__device__ __forceinline__ unsigned long long make_key(float v, int idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(u) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(idx));
}

__device__ __forceinline__ float key_val(unsigned long long key) {
  uint32_t u = static_cast<uint32_t>(key >> 32);
  u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
  return __uint_as_float(u);
}

__device__ __forceinline__ int key_idx(unsigned long long key) {
  return static_cast<int>(~static_cast<uint32_t>(key & 0xFFFFFFFFull));
}


// Rank selection: the row's n candidates (logical order: half-0 stack, then half-1 stack)
// become keys in the warp's scratch ks; every lane counts, for its NQ keys, how many keys
// of the row beat them (broadcast reads, independent compares: no shuffle chains) -- on the
// 32-bit scores, or on 64-bit keys (score, then lower column) when the row has exact ties.
// Keys are unique (distinct columns), so the best min(k, real) keys have ranks 0 .. k-1.
// The survivors are written back in column order, as two ascending runs: when the stacks
// hold columns in ascending order (`runs`: the threshold pass appends them that way),
// by a ballot prefix over the logical order, run 0 = survivors of stack 0 and run 1 =
// those of stack 1; otherwise (heap fallback rows) by counting, for every survivor, the
// survivors of lower column -- one run. m0 receives the length of run 0. ri[kCap / 2 + c]
// keeps the score rank of slot c for the ordered score outputs.
// Returns min(k, real candidates). Needs c0 + c1 <= NQ * 32 and k <= kCap / 2.
template <int NQ>
__device__ int warp_rank_select(float* rv, int* ri, int c0, int c1, int k, int lane, unsigned long long* ks,
                                bool runs, int& m0) {
  const int n = c0 + c1;
  const int n4 = (n + 3) & ~3;
  const unsigned long long kNone = make_key(-INFINITY, kSentinel);
  unsigned long long x[NQ];
  uint32_t u[NQ];  // orderable score, 0 = no candidate (below every real score)
  int rank[NQ];
  uint32_t* ku = reinterpret_cast<uint32_t*>(ks);
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    const int i = q * 32 + lane;
    const int e = i < c0 ? i : kCap - 1 - (i - c0);
    const bool real_i = i < n && ri[e] != kSentinel;
    x[q] = real_i ? make_key(rv[e], ri[e]) : kNone;
    u[q] = real_i ? static_cast<uint32_t>(x[q] >> 32) : 0u;
    if (i < n4) ku[i] = u[q];
    rank[q] = 0;
  }
  __syncwarp();  // from here on rv / ri of the row are free: every lane holds its keys
#ifdef JK_PHASE_PROFILE
  long long tq0 = clock64();
#endif
  // Rank on the 32-bit scores (four keys per 16-byte broadcast read) ...
  for (int j = 0; j < n4; j += 4) {
    const uint4 a = *reinterpret_cast<const uint4*>(ku + j);
#pragma unroll
    for (int q = 0; q < NQ; ++q) rank[q] += (a.x > u[q]) + (a.y > u[q]) + (a.z > u[q]) + (a.w > u[q]);
  }
  // ... which is exact unless two candidates tie on the score: the ranks of the real keys are
  // then not a permutation of 0 .. real-1 (tied keys share a rank), and the row is ranked
  // again on the 64-bit keys (score, then lower column).
  int real = 0, rsum = 0;
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    real += __popc(__ballot_sync(0xffffffffu, x[q] != kNone));
    rsum += x[q] != kNone ? rank[q] : 0;
  }
  rsum = __reduce_add_sync(0xffffffffu, rsum);
  if (rsum != real * (real - 1) / 2) {
    __syncwarp();  // every lane has read the 32-bit keys
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const int i = q * 32 + lane;
      if (i < n) ks[i] = x[q];
      rank[q] = 0;
    }
    __syncwarp();
    int j = 0;
    for (; j + 2 <= n; j += 2) {
      const ulonglong2 a = *reinterpret_cast<const ulonglong2*>(ks + j);
#pragma unroll
      for (int q = 0; q < NQ; ++q) rank[q] += (a.x > x[q]) + (a.y > x[q]);
    }
    for (; j < n; ++j) {
      const unsigned long long a = ks[j];
#pragma unroll
      for (int q = 0; q < NQ; ++q) rank[q] += a > x[q];
    }
  }
#ifdef JK_PHASE_PROFILE
  long long tq1 = clock64();
#endif
  bool keep[NQ];
  int col[NQ], slot[NQ];
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    keep[q] = x[q] != kNone && rank[q] < k;
    col[q] = key_idx(x[q]);
  }
  if (runs) {
    const uint32_t lt = (1u << lane) - 1u;
    int before = 0, in0 = 0;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const uint32_t bal = __ballot_sync(0xffffffffu, keep[q]);
      slot[q] = before + __popc(bal & lt);
      before += __popc(bal);
      in0 += __popc(__ballot_sync(0xffffffffu, keep[q] && q * 32 + lane < c0));
    }
    m0 = in0;
  } else {
    __syncwarp();  // every lane has read the keys: the scratch now holds the kept columns
    int* kc = reinterpret_cast<int*>(ks);
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const int i = q * 32 + lane;
      if (i < n) kc[i] = keep[q] ? col[q] : INT_MAX;
      slot[q] = 0;
    }
    __syncwarp();
    int j = 0;
    for (; j + 4 <= n; j += 4) {
      const int4 a = *reinterpret_cast<const int4*>(kc + j);
#pragma unroll
      for (int q = 0; q < NQ; ++q) slot[q] += (a.x < col[q]) + (a.y < col[q]) + (a.z < col[q]) + (a.w < col[q]);
    }
    for (; j < n; ++j) {
      const int a = kc[j];
#pragma unroll
      for (int q = 0; q < NQ; ++q) slot[q] += a < col[q];
    }
    m0 = real < k ? real : k;
  }
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    if (keep[q]) {
      rv[slot[q]] = key_val(x[q]);
      ri[slot[q]] = col[q];
      ri[kCap / 2 + slot[q]] = rank[q];
    }
  }
  __syncwarp();
#ifdef JK_PHASE_PROFILE
  if (threadIdx.x == 0) {
    const int cta = blockIdx.y * gridDim.x + blockIdx.x;
    if (cta < kTraceCtas) {
      g_trace[cta][19] += tq1 - tq0;
      g_trace[cta][20] += clock64() - tq1;
    }
  }
#endif
  return real < k ? real : k;
}

// Two rows at once (the latency of one row's loads and compares hides the other's): the
// 32-bit-score ranking of warp_rank_select for two rows whose stacks hold ascending
// column runs. A row with exact score ties is left untouched (done[] false) for
// warp_rank_select; a done row is written back exactly as warp_rank_select writes it.
template <int NQ>
__device__ void warp_rank_pair(float* const (&rv)[2], int* const (&ri)[2], const int (&c0)[2], const int (&c1)[2],
                               int k, int lane, uint32_t* ku, bool (&done)[2], int (&nout)[2], int (&m0)[2]) {
  int n[2], n4[2];
  float sc[2][NQ];
  int col[2][NQ];
  uint32_t u[2][NQ];
  int rank[2][NQ];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    n[r] = c0[r] + c1[r];
    n4[r] = (n[r] + 3) & ~3;
  }
  const int nmax = n4[0] > n4[1] ? n4[0] : n4[1];
#ifdef JK_PHASE_PROFILE
  const long long tp0 = clock64();
#endif
#pragma unroll
  for (int r = 0; r < 2; ++r) {
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const int i = q * 32 + lane;
      const int e = i < c0[r] ? i : kCap - 1 - (i - c0[r]);
      // both reads unconditional (e stays inside the row's buffer), so they overlap
      const int ci = ri[r][e];
      const float cv = rv[r][e];
      const bool real_i = i < n[r] && ci != kSentinel;
      sc[r][q] = real_i ? cv : 0.f;
      col[r][q] = real_i ? ci : 0;
      u[r][q] = real_i ? static_cast<uint32_t>(make_key(sc[r][q], col[r][q]) >> 32) : 0u;
      if (i < nmax) ku[r * kCap + i] = u[r][q];  // zero beyond the row: never beats a key
      rank[r][q] = 0;
    }
  }
  __syncwarp();
#ifdef JK_PHASE_PROFILE
  const long long tp1 = clock64();
#endif
  // four broadcast reads per row in flight per step
#pragma unroll 4
  for (int j = 0; j < nmax; j += 4) {
    const uint4 a = *reinterpret_cast<const uint4*>(ku + j);
    const uint4 b = *reinterpret_cast<const uint4*>(ku + kCap + j);
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      rank[0][q] += (a.x > u[0][q]) + (a.y > u[0][q]) + (a.z > u[0][q]) + (a.w > u[0][q]);
      rank[1][q] += (b.x > u[1][q]) + (b.y > u[1][q]) + (b.z > u[1][q]) + (b.w > u[1][q]);
    }
  }
#ifdef JK_PHASE_PROFILE
  const long long tp2 = clock64();
#endif
  const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    int real = 0, rsum = 0;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const bool is_real = u[r][q] != 0u;
      real += __popc(__ballot_sync(0xffffffffu, is_real));
      rsum += is_real ? rank[r][q] : 0;
    }
    rsum = __reduce_add_sync(0xffffffffu, rsum);
    done[r] = rsum == real * (real - 1) / 2;
    if (!done[r]) continue;  // warp-uniform
    bool keep[NQ];
    int slot[NQ];
    int before = 0, in0 = 0;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      keep[q] = u[r][q] != 0u && rank[r][q] < k;
      const uint32_t bal = __ballot_sync(0xffffffffu, keep[q]);
      slot[q] = before + __popc(bal & lt);
      before += __popc(bal);
      in0 += __popc(__ballot_sync(0xffffffffu, keep[q] && q * 32 + lane < c0[r]));
    }
    m0[r] = in0;
    nout[r] = real < k ? real : k;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      if (keep[q]) {
        rv[r][slot[q]] = sc[r][q];
        ri[r][slot[q]] = col[r][q];
        ri[r][kCap / 2 + slot[q]] = rank[r][q];
      }
    }
  }
  __syncwarp();
#ifdef JK_PHASE_PROFILE
  if (threadIdx.x == 0) {
    const int cta = blockIdx.y * gridDim.x + blockIdx.x;
    if (cta < kTraceCtas) {
      g_trace[cta][29] += tp1 - tp0;
      g_trace[cta][30] += tp2 - tp1;
      g_trace[cta][31] += clock64() - tp2;
    }
  }
#endif
}

__device__ __forceinline__ void sel_barrier() {
  asm volatile("bar.sync 1, %0;" ::"r"(kSelWarps * 32) : "memory");
}

// Source window of a CTA's tensor-core aggregate: rows [s_lo, s_lo + n) of the values,
// s_lo on the score-tile grid, so that 64-row source tile kt is the first (even kt) or the
// second (odd kt) half of a score tile -- the columns of candidate stack 0 or 1.
// Taken for 16-bit values whose width fits the TMEM accumulator beside the edge tiles, when
// the CTA's sources (its causal window, or every column without a window) are few enough
// that the dense edge-tile MMAs (4 * n * dim * 128 FLOP) beat the latency-bound CUDA-core
// gather of the k selected rows: n <= 1024, or n <= 128 * k + 1024 (identical in every
// thread).
struct SlabRange {
  int s_lo, n;
  bool on;
};

template <typename VT>
__device__ __forceinline__ SlabRange slab_range(const Params& p, int64_t t0) {
  SlabRange r{0, 0, false};
  if (p.slab_ok && sizeof(VT) == 2 && (p.dim % 64) == 0) {
    int64_t hi_col = p.n_cols - 1;
    if (p.window >= 0) {
      const int64_t lo = t0 - p.window;
      r.s_lo = static_cast<int>((lo > 0 ? lo : 0) / kCols * kCols);  // on the score-tile grid
      if (t0 + kRows - 1 < hi_col) hi_col = t0 + kRows - 1;
    }
    r.n = static_cast<int>(hi_col - r.s_lo + 1);
    r.on = r.n > 0 && (r.n <= 1024 || r.n <= 128 * p.k + 1024) && p.dim <= kOCols;
  }
  return r;
}

// ---------------------------------------------------------------- shared-memory layout
template <int KATOMS, int STAGES>
struct Layout {
  static constexpr int kAtomBytes = kRows * 128;  // 128 rows x 64 (16-bit) elements
  static constexpr int kABytes = KATOMS * kAtomBytes;
  static constexpr int kBBytes = KATOMS * kAtomBytes;
  // A + ring; reused by the selection scratch, then by the aggregate's edge tiles
  static constexpr int kRegion0 = kABytes + STAGES * kBBytes;
  static_assert(kRegion0 >= 2 * kETile, "the aggregate's edge tiles reuse region 0");
  static constexpr int kBufBytes = 2 * kRows * kStride * 4;    // candidate values + indices
  static_assert(kBufBytes / 2 - 1023 >= kVBufs * kVBufBytes, "the value slices reuse the candidate-index buffer");
  static constexpr int kRowArrays = 10 * kRows * 4;            // per-row scalars
  static constexpr int kBarBytes = 320;
  static constexpr int kTotal = 1024 + kRegion0 + kBufBytes + kRowArrays + kBarBytes;
};

template <int KATOMS, int STAGES, int MODE, typename VT, bool MH>
__global__ void __launch_bounds__(kThreads, 1)
    topk_kernel(const __grid_constant__ CUtensorMap tm_rows, const __grid_constant__ CUtensorMap tm_cols,
                const __grid_constant__ CUtensorMap tm_val, const __grid_constant__ CUtensorMap tm_out, Params p,
                uint32_t idesc) {
  using L = Layout<KATOMS, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tile = smem;
  uint8_t* b_ring = smem + L::kABytes;
  float* bufv = reinterpret_cast<float*>(smem + L::kRegion0);  // [kRows][kStride]
  int* bufi = reinterpret_cast<int*>(bufv + kRows * kStride);
  int* cnt = bufi + kRows * kStride;                           // [kRows]
  int* nsel = cnt + kRows;                                     // [kRows]
  int* failrow = nsel + kRows;                                 // [kRows]
  float* tau = reinterpret_cast<float*>(failrow + kRows);      // [kRows]
  float* s1 = tau + kRows;                                     // [2][kRows]
  float* s2 = s1 + 2 * kRows;                                  // [2][kRows]
  volatile float* pub = s2 + 2 * kRows;                        // [2][kRows]
  uint64_t* bars = reinterpret_cast<uint64_t*>(const_cast<float*>(pub) + 2 * kRows);
  uint64_t* bar_a = bars;
  uint64_t* decide = bars + 1;
  uint64_t* slab_bar = bars + 2;
  uint64_t* agg_bar = bars + 3;
  uint64_t* vb_full = bars + 4;    // [kVBufs] value slices of the tensor-core aggregate
  uint64_t* vb_empty = bars + 8;   // [kVBufs]
  uint64_t* e_full = bars + 12;    // [2] edge tiles written (one arrival per selection warp)
  uint64_t* e_empty = bars + 14;   // [2] edge tiles retired by their MMAs
  uint64_t* full = bars + 16;
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* any_fail = abort_flag + 1;
  volatile int* agg_mode = any_fail + 1;  // 1: tensor-core aggregate (set before slab_bar)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t b = blockIdx.y;
  const int64_t t0 = p.row_begin + static_cast<int64_t>(blockIdx.x) * kRows;
  const int k = p.k;

  // Column-tile range (identical in every thread).
  int64_t j_lo = 0, j_hi = (p.n_cols + kCols - 1) / kCols - 1;
  if (p.window >= 0) {
    const int64_t lo = t0 - p.window;
    j_lo = lo > 0 ? lo / kCols : 0;
    int64_t hi_col = t0 + kRows - 1;
    if (hi_col > p.n_cols - 1) hi_col = p.n_cols - 1;
    j_hi = hi_col < 0 ? -1 : hi_col / kCols;
  }
  const int ntiles = j_hi >= j_lo ? static_cast<int>(j_hi - j_lo + 1) : 0;
  // Pass A is needed when some row can see more columns than its buffer holds.
  const int64_t max_visible = p.window >= 0 ? (p.window + 1 < p.n_cols ? p.window + 1 : p.n_cols) : p.n_cols;
  // Pass A (a threshold from the row statistics) runs when some row sees more columns than its
  // buffer holds, and also when it sees at least twice the threshold's target count: the
  // select step then ranks ~k + 3 sqrt(k) + 8 candidates instead of every visible column.
  const float sel_target = fminf(static_cast<float>(k) + 3.f * sqrtf(static_cast<float>(k)) + 8.f, 0.75f * kCap);
  const bool has_a = max_visible > kCap || static_cast<float>(max_visible) >= 2.f * sel_target;
  const int pre_passes = has_a ? 2 : 1;

  if (threadIdx.x == 0) {
    mbar_init(bar_a, 1);
    mbar_init(decide, 1);
    mbar_init(slab_bar, 1);
    mbar_init(agg_bar, 1);
    for (int i = 0; i < kVBufs; ++i) {
      mbar_init(&vb_full[i], 1);
      mbar_init(&vb_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&e_full[i], kSelWarps / 2);  // the four warps of one half build a tile
      mbar_init(&e_empty[i], 1);
    }
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kSelWarps);
    }
    *abort_flag = 0;
    *any_fail = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
#ifdef JK_PHASE_PROFILE
  if (threadIdx.x == 0) {
    JK_STAMP(0);
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    const int cta = blockIdx.y * gridDim.x + blockIdx.x;
    if (cta < kTraceCtas) {
      g_trace[cta][15] = smid;
      for (int z = 19; z < 32; ++z) g_trace[cta][z] = 0;
    }
  }
#endif

  if (warp == kLoadWarp) {
    // ------------------------------------------------------------ TMA loader
    // Row tile once, then the column tiles of every pass through the STAGES ring, then
    // (tensor-core aggregate) the value slices of the source window through kVBufs buffers.
    if (lane == 0 && ntiles > 0) {
      prefetch_tmap(&tm_rows);
      prefetch_tmap(&tm_cols);
      if (p.slab_ok) prefetch_tmap(&tm_val);
      bool ok = true;
      mbar_arrive_expect_tx(bar_a, L::kABytes);
#pragma unroll
      for (int a = 0; a < KATOMS; ++a)
        tma_load_3d(a_tile + a * L::kAtomBytes, &tm_rows, bar_a, a * 64, static_cast<int>(t0), static_cast<int>(b));
      int total = pre_passes * ntiles;  // grows by one pass if the fallback pass is needed
      const int decide_at = total - 1;
      for (int i = 0; i < total && ok; ++i) {
        const int s = i % STAGES;
        if (i >= STAGES && !mbar_wait(&empty[s], ((i - STAGES) / STAGES) & 1)) { ok = false; break; }
        if (*abort_flag) { ok = false; break; }
        mbar_arrive_expect_tx(&full[s], L::kBBytes);
        const int col0 = static_cast<int>((j_lo + i % ntiles) * kCols);
#pragma unroll
        for (int a = 0; a < KATOMS; ++a)
          tma_load_3d(b_ring + s * L::kBBytes + a * L::kAtomBytes, &tm_cols, &full[s], a * 64, col0,
                      static_cast<int>(b));
        if (i == decide_at) {
          // The selection warps report whether any row needs the exact fallback pass.
          if (!mbar_wait(decide, 0)) { ok = false; break; }
          if (*any_fail) total += ntiles;
        }
      }
      JK_STAMP(14);
      if (ok) ok = mbar_wait(slab_bar, 0);
      if (ok && *agg_mode) {
        const SlabRange sr = slab_range<VT>(p, t0);
        const int nkt = (sr.n + kEK - 1) / kEK;
        const int nsl = static_cast<int>((p.dim + kVSlice - 1) / kVSlice);
        // the candidate-index buffer: free once compress packed the survivors into bufv
        uint8_t* vbuf = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(bufi) + 1023) & ~uintptr_t(1023));
        for (int pi = 0; pi < nkt * nsl && ok; ++pi) {
          const int vb = pi % kVBufs;
          if (pi >= kVBufs && !JK_PHASE_TIME(10, mbar_wait(&vb_empty[vb], ((pi - kVBufs) / kVBufs) & 1))) {
            ok = false;
            break;
          }
          if (*abort_flag) { ok = false; break; }
          const int kt = pi / nsl, sl = pi % nsl;
          const int w = static_cast<int>(p.dim) - sl * kVSlice;
          const int nb = (w < kVSlice ? w : kVSlice) / 64;
          mbar_arrive_expect_tx(&vb_full[vb], nb * 8192);
          for (int a = 0; a < nb; ++a)
            tma_load_3d(vbuf + vb * kVBufBytes + a * 8192, &tm_val, &vb_full[vb], sl * kVSlice + a * 64,
                        sr.s_lo + kt * kEK, static_cast<int>(b));
        }
      }
      if (!ok) {
        atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
        *abort_flag = 1;
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && ntiles > 0) {
      bool ok = mbar_wait(bar_a, 0);
      int total = pre_passes * ntiles;
      const int decide_at = total - 1;
      const int nb = MH ? score_buffers(p.heads) : 2;
      for (int g = 0; g < total && ok; ++g) {
        const int st = g % STAGES;
        const int buf = g % nb;
        if (!mbar_wait(&full[st], (g / STAGES) & 1)) { ok = false; break; }
        if (g >= nb && !mbar_wait(&tempty[buf], ((g / nb) - 1) & 1)) { ok = false; break; }
        if (*abort_flag) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(a_tile);
        const uint32_t b_addr = smem_u32(b_ring + st * L::kBBytes);
        if (MH)
          head_score_mmas(tmem + buf * p.heads * kCols, kCols, a_addr, b_addr, idesc, p.heads, p.kph);
        else
          score_mmas<KATOMS>(tmem + buf * kCols, a_addr, b_addr, idesc, p.split3 != 0);
        if (g == 0) JK_STAMP(10);
        mma_commit(&empty[st]);
        mma_commit(&tfull[buf]);
        if (g == decide_at) {
          if (!mbar_wait(decide, 0)) { ok = false; break; }
          if (*any_fail) total += ntiles;
        }
      }
      // The MMA-retire arrivals on the ring barriers must land before the CTA exits.
      if (ok) {
        const int last = total - 1;
        ok = mbar_wait(&empty[last % STAGES], (last / STAGES) & 1);
      }
      // Aggregate MMAs: once the selection warps decided (slab_bar), every double-buffered
      // edge tile (TMEM) is multiplied with the value slices the loader streams in.
      if (ok) ok = mbar_wait(slab_bar, 0);
      if (ok && *agg_mode) {
        constexpr bool kHalfV = std::is_same<VT, __half>::value;
        const SlabRange sr = slab_range<VT>(p, t0);
        const int nkt = (sr.n + kEK - 1) / kEK;
        const int nsl = static_cast<int>((p.dim + kVSlice - 1) / kVSlice);
        uint8_t* vbuf = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(bufi) + 1023) & ~uintptr_t(1023));
        JK_STAMP(11);
        for (int kt = 0; kt < nkt && ok; ++kt) {
          const int buf = kt & 1;
#ifdef JK_PHASE_PROFILE
          const long long tw0 = clock64();
#endif
          if (!mbar_wait(&e_full[buf], (kt >> 1) & 1) || *abort_flag) { ok = false; break; }
#ifdef JK_PHASE_PROFILE
          g_trace[(blockIdx.y * gridDim.x + blockIdx.x) % kTraceCtas][22] += clock64() - tw0;
#endif
          tc_fence_after();
          const uint32_t e_addr = smem_u32(smem + buf * kETile);
          for (int sl = 0; sl < nsl; ++sl) {
            const int pi = kt * nsl + sl, vb = pi % kVBufs;
#ifdef JK_PHASE_PROFILE
            const long long tw1 = clock64();
#endif
            if (!mbar_wait(&vb_full[vb], (pi / kVBufs) & 1)) { ok = false; break; }
#ifdef JK_PHASE_PROFILE
            g_trace[(blockIdx.y * gridDim.x + blockIdx.x) % kTraceCtas][23] += clock64() - tw1;
#endif
            const int w = static_cast<int>(p.dim) - sl * kVSlice;
            const uint32_t idesc_pv = idesc_f16(kRows, w < kVSlice ? w : kVSlice, kHalfV ? 0u : 1u) | (1u << 16);
            const uint32_t v_addr = smem_u32(vbuf + vb * kVBufBytes);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
#pragma unroll
              for (int kk = 0; kk < kEK / 16; ++kk) {
                mma_f16_ss(tmem + sl * kVSlice, sdesc_kmajor_sw128(e_addr + q * (kETile / 2) + kk * 32),
                           sdesc_mnmajor_sw128(v_addr + kk * 2048, 8192),
                           idesc_pv, (kt > 0 || q > 0 || kk > 0) ? 1u : 0u);
              }
            }
            mma_commit(&vb_empty[vb]);
          }
          if (ok) mma_commit(&e_empty[buf]);
        }
        if (ok) {
          mma_commit(agg_bar);
          JK_STAMP(12);
          ok = mbar_wait(agg_bar, 0);  // every MMA and commit retired before the CTA exits
          JK_STAMP(13);
        }
      }
      if (!ok) {
        atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
        *abort_flag = 1;
      }
    }
  } else {
    // ------------------------------------------------------------ selection warps
    const int quad = warp & 3;
    const int half = warp >> 2;
    const int row = quad * 32 + lane;  // TMEM lane == row in tile
    const int64_t t = t0 + row;
    const bool row_ok = t < p.n_rows;
    // Visible columns of this row: [lo_t, hi_t] (32-bit; sizes are capped at 2^30).
    int lo_t = 0, hi_t = static_cast<int>(p.n_cols - 1);
    if (p.window >= 0) {
      const int64_t lo = t - p.window;
      lo_t = lo < 0 ? 0 : static_cast<int>(lo);
      hi_t = t < hi_t ? static_cast<int>(t) : hi_t;
    }
    int visible = hi_t - lo_t + 1;
    if (!row_ok || hi_t < lo_t) {  // nothing visible: an unreachable single-column range
      lo_t = INT_MAX / 2;
      hi_t = INT_MAX / 2;
      visible = 0;
    }
    const uint32_t span = static_cast<uint32_t>(hi_t - lo_t);
    const uint32_t tbase = (static_cast<uint32_t>(quad * 32) << 16) + half * kHalfCols;
    float* rv = bufv + row * kStride;
    int* ri = bufi + row * kStride;
    int g = 0;  // global iteration (tile x pass)
    bool ok = true;
    long long t_prev = 0;
    (void)t_prev;

    // Loads this thread's 64 scores of iteration g into v; false on timeout / abort.
    const int nbuf = MH ? score_buffers(p.heads) : 2;
    auto load_tile = [&](uint32_t (&v)[2][32]) -> bool {
      const int buf = g % nbuf;
      if (!JK_PHASE_TIME(18, mbar_wait(&tfull[buf], (g / nbuf) & 1)) || *abort_flag) return false;
      tc_fence_after();
      if (MH) {
        const uint32_t base = tmem + tbase + buf * p.heads * kCols;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float f[16];
          if (p.heads == 2) combine_heads16<2>(base + c * 16, kCols, p.head_bias, p.combine, f);
          else if (p.heads == 3) combine_heads16<3>(base + c * 16, kCols, p.head_bias, p.combine, f);
          else combine_heads16<4>(base + c * 16, kCols, p.head_bias, p.combine, f);
#pragma unroll
          for (int i = 0; i < 16; ++i) v[c >> 1][(c & 1) * 16 + i] = __float_as_uint(f[i]);
        }
      } else {
        tmem_ld_32x32b_x32(tmem + tbase + buf * kCols, v[0]);
        tmem_ld_32x32b_x32(tmem + tbase + buf * kCols + 32, v[1]);
        tmem_ld_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      ++g;
      return true;
    };

    // ---- pass A: row statistics -> threshold
    if (half == 0) cnt[row] = 0;
    if (has_a) {
      float a1 = 0.f, a2 = 0.f;
      for (int it = 0; it < ntiles && ok; ++it) {
        uint32_t v[2][32];
        if (!load_tile(v)) { ok = false; break; }
        const int col0 = static_cast<int>((j_lo + it) * kCols) + half * kHalfCols;
        if (static_cast<uint32_t>(col0 - lo_t) <= span && static_cast<uint32_t>(col0 + kHalfCols - 1 - lo_t) <= span) {
          // every column of this thread's share is visible (the interior of a window)
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const float x = __uint_as_float(v[c][e]);
              a1 += x;
              a2 = fmaf(x, x, a2);
            }
        } else {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const float x = __uint_as_float(v[c][e]);
              const bool vis = static_cast<uint32_t>(col0 + c * 32 + e - lo_t) <= span;
              a1 += vis ? x : 0.f;
              a2 = vis ? fmaf(x, x, a2) : a2;
            }
        }
      }
      s1[half * kRows + row] = a1;
      s2[half * kRows + row] = a2;
      sel_barrier();
      if (half == 0) {
        float th = -INFINITY;
        if (visible > kCap || static_cast<float>(visible) >= 2.f * sel_target) {
          const float n = static_cast<float>(visible);
          const float mean = (s1[row] + s1[kRows + row]) / n;
          const float var = fmaxf((s2[row] + s2[kRows + row]) / n - mean * mean, 0.f);
          // Expected survivors: k plus ~3 standard deviations of the count, so that too few
          // is rare (the exact fallback pass covers it) and most rows fit a 64-key sort.
          const float target = sel_target;
          const float z = 1.41421356f * erfinvf(1.f - 2.f * target / n);
          th = mean + z * sqrtf(var);
        }
        tau[row] = th;
      }
    } else if (half == 0) {
      tau[row] = -INFINITY;
    }
    sel_barrier();
    JK_PHASE_MARK(0, t_prev);

    // ---- pass B: collect the columns at or above the threshold. Half 0 stacks its
    // candidates from slot 0 upwards, half 1 from slot kCap-1 downwards, each with a
    // register counter (no atomics); a row whose stacks meet takes the exact fallback pass.
    {
      const float th = tau[row];
      // slot myc of this half's stack: byte offset o_base + o_step * myc
      const int o_base = half == 0 ? 0 : (kCap - 1) * 4;
      const int o_step = half == 0 ? 4 : -4;
      const uint32_t rv_s = smem_u32(rv) + o_base, ri_s = smem_u32(ri) + o_base;
      int myc = 0;
      // predicated append (no branch): a passing column goes to slot myc of this half's
      // stack while it has room; myc counts every passing column
      auto append = [&](bool pass, float x, int col) {
        const uint32_t off = static_cast<uint32_t>(o_step * myc);
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %0, 0;\n\t"
            "@p st.shared.f32 [%1], %2;\n\t"
            "@p st.shared.b32 [%3], %4;\n\t}" ::"r"(static_cast<int>(pass && myc < kCap)),
            "r"(rv_s + off), "f"(x), "r"(ri_s + off), "r"(col)
            : "memory");
        myc += pass ? 1 : 0;
      };
      for (int it = 0; it < ntiles && ok; ++it) {
        uint32_t v[2][32];
        if (!load_tile(v)) { ok = false; break; }
        const int col0 = static_cast<int>((j_lo + it) * kCols) + half * kHalfCols;
        if (static_cast<uint32_t>(col0 - lo_t) <= span && static_cast<uint32_t>(col0 + kHalfCols - 1 - lo_t) <= span) {
          // interior: every column of this thread's share is visible
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const float x = __uint_as_float(v[c][e]);
              append(x >= th, x, col0 + c * 32 + e);
            }
        } else {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int col = col0 + c * 32 + e;
              const float x = __uint_as_float(v[c][e]);
              append(static_cast<uint32_t>(col - lo_t) <= span && x >= th, x, col);
            }
        }
      }
      (half == 0 ? cnt : nsel)[row] = myc;
    }
    if (!ok) {
      atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
      *abort_flag = 1;
    }
    sel_barrier();
    if (half == 0) {
      const int c0 = cnt[row], c1 = nsel[row];
      const int need = k < visible ? k : visible;
      const bool fail = row_ok && (c0 + c1 > kCap || c0 + c1 < need);
      failrow[row] = fail ? 1 : 0;
      if (fail) *any_fail = 1;
    }
    sel_barrier();
    if (threadIdx.x == 0) mbar_arrive(decide);
    JK_PHASE_MARK(1, t_prev);

    // ---- pass C (rare): exact streaming selection for the rows the threshold missed
    if (*any_fail && !*abort_flag && ntiles > 0) {
      const bool mine = failrow[row] != 0;
      const Lane heap{rv + half * 64, ri + half * 64};
      const Lane queue{rv + kCap + half * kQueue, ri + kCap + half * kQueue};
      if (mine) {
        for (int e = 0; e < 64; ++e) {
          heap.val(e) = -INFINITY;
          heap.idx(e) = kSentinel;
        }
      }
      pub[half * kRows + row] = -INFINITY;
      sel_barrier();
      float thr_own = -INFINITY, thr_part = -INFINITY;
      int qn = 0;
      for (int it = 0; it < ntiles && ok; ++it) {
        uint32_t v[2][32];
        if (!load_tile(v)) { ok = false; break; }
        const int col0 = static_cast<int>((j_lo + it) * kCols) + half * kHalfCols;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int col = col0 + c * 32 + e + u;
              const float x = __uint_as_float(v[c][e + u]);
              if (mine && static_cast<uint32_t>(col - lo_t) <= span && x > thr_own && x >= thr_part) {
                queue.val(qn) = x;
                queue.idx(qn) = col;
                ++qn;
              }
            }
            if (__any_sync(0xffffffffu, qn > 0)) {
              thr_own = flush_queue(heap, queue, k, qn);
              pub[half * kRows + row] = thr_own;
              thr_part = pub[(half ^ 1) * kRows + row];
            }
          }
        }
      }
      if (!ok) {
        atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
        *abort_flag = 1;
      }
      sel_barrier();
      if (half == 0 && mine) {  // both heaps (sentinel padded) are the candidates
        cnt[row] = 64;
        nsel[row] = 64;
      }
    }
    sel_barrier();
    JK_PHASE_MARK(2, t_prev);
    const bool good = !*abort_flag;

    // ---- select: one warp per row keeps the best k of the row's two candidate stacks
    const int rt0 = warp * (kRows / kSelWarps);
    // Key scratch in the (now idle) operand region: 128 keys per warp.
    unsigned long long* ks = reinterpret_cast<unsigned long long*>(smem) + warp * kCap;
    for (int r = 0; r < kRows / kSelWarps; r += 2) {
      // rows rt0 + r and rt0 + r + 1 together; exact-fallback rows and rows with score ties
      // go through warp_rank_select one at a time
      float* wv[2];
      int* wi[2];
      int c0[2], c1[2], n[2] = {0, 0}, m0[2] = {0, 0};
      bool live[2], pairable[2], done[2] = {false, false};
      int mmax = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int rt = rt0 + r + h;
        wv[h] = bufv + rt * kStride;
        wi[h] = bufi + rt * kStride;
        live[h] = good && t0 + rt < p.n_rows;
        c0[h] = live[h] ? cnt[rt] : 0;
        c1[h] = live[h] ? nsel[rt] : 0;
        pairable[h] = live[h] && failrow[rt] == 0;
        if (pairable[h] && c0[h] + c1[h] > mmax) mmax = c0[h] + c1[h];
#ifdef JK_PHASE_PROFILE
        if (threadIdx.x == 0 && blockIdx.y * gridDim.x + blockIdx.x < kTraceCtas)
          g_trace[blockIdx.y * gridDim.x + blockIdx.x][21] += c0[h] + c1[h];
#endif
      }
      if (pairable[0] && pairable[1]) {
        uint32_t* ku = reinterpret_cast<uint32_t*>(ks);
        if (mmax <= 32) warp_rank_pair<1>(wv, wi, c0, c1, k, lane, ku, done, n, m0);
        else if (mmax <= 64) warp_rank_pair<2>(wv, wi, c0, c1, k, lane, ku, done, n, m0);
        else if (mmax <= 96) warp_rank_pair<3>(wv, wi, c0, c1, k, lane, ku, done, n, m0);
        else warp_rank_pair<4>(wv, wi, c0, c1, k, lane, ku, done, n, m0);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (live[h] && !done[h]) {
          const int m = c0[h] + c1[h];
          const bool runs = pairable[h];
          n[h] = m <= 32   ? warp_rank_select<1>(wv[h], wi[h], c0[h], c1[h], k, lane, ks, runs, m0[h])
                 : m <= 64 ? warp_rank_select<2>(wv[h], wi[h], c0[h], c1[h], k, lane, ks, runs, m0[h])
                 : m <= 96 ? warp_rank_select<3>(wv[h], wi[h], c0[h], c1[h], k, lane, ks, runs, m0[h])
                           : warp_rank_select<4>(wv[h], wi[h], c0[h], c1[h], k, lane, ks, runs, m0[h]);
        }
      }
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          nsel[rt0 + r + h] = n[h];
          cnt[rt0 + r + h] = m0[h];  // length of the first ascending column run
        }
      }
    }
    sel_barrier();
    JK_PHASE_MARK(3, t_prev);

    // ---- compress (thread per row), fold the sender strength, form the state output
    const SlabRange sr = slab_range<VT>(p, t0);
    const bool tc_agg = MODE == kGather && good && sr.on && ntiles > 0;
    // The source states of a windowed CTA, staged once (coalesced) in the selection passes'
    // per-row scratch (s1, s2, pub: 6 x kRows contiguous floats, free from here on).
    float* st_stage = s1;
    uint32_t n_stage = 0;
    if (MODE == kGather && good && sr.on) n_stage = static_cast<uint32_t>(sr.n < 6 * kRows ? sr.n : 6 * kRows);
    if (n_stage > 0) {
      for (int i = threadIdx.x; i < static_cast<int>(n_stage); i += kSelWarps * 32)
        st_stage[i] = ld_elem(p.col_state, b * p.n_cols + sr.s_lo + i, p.state_dtype);
      sel_barrier();
    }
    // Softsign is elementwise: unless the ordered scores are requested, both threads of a
    // row share its entries (even / odd) and half 1 hands its state partial over in tau.
    const bool split = p.compress == JK_SOFTSIGN && !(p.out_scores || p.out_index);
    const Lane F{rv, ri};
    const int n_row = nsel[row];
    if (split) {
      const float bias = p.bias + (p.bias_dev ? __ldg(p.bias_dev) : 0.f);
      float acc = 0.f;
      const int64_t cb = b * p.n_cols;
      for (int e = half; e < n_row; e += 2) {
        const float x = F.val(e) + bias;
        float w = x / (1.f + fabsf(x));
        if (MODE == kGather) {
          const int j = F.idx(e);
          const uint32_t js = static_cast<uint32_t>(j - sr.s_lo);
          if (p.col_sender) w *= ld_elem(p.col_sender, cb + j, p.state_dtype);
          const float stv = js < n_stage ? st_stage[js] : ld_elem(p.col_state, cb + j, p.state_dtype);
          acc = fmaf(w, stv, acc);
        }
        F.val(e) = w;
      }
      if (half == 1) tau[row] = acc;
      sel_barrier();
      if (MODE == kGather && half == 0 && row_ok && good)
        st_elem(p.out_state, b * p.n_rows + t, p.out_dtype, acc + tau[row]);
    }
    if (half == 0) {
      const int n = n_row;
      if (!split) {
      const float bias = p.bias + (p.bias_dev ? __ldg(p.bias_dev) : 0.f);
      for (int e = 0; e < n; ++e) F.val(e) += bias;
      if (row_ok && good && (p.out_scores || p.out_index)) {  // the selection, in score order
        const int64_t o = (b * p.n_rows + t) * k;
        // column slot e holds score rank ri[kCap / 2 + e]; outputs go in score order
        for (int e = 0; e < k; ++e) {
          const int r = e < n ? F.idx(kCap / 2 + e) : e;
          if (p.out_scores) p.out_scores[o + r] = e < n ? F.val(e) : -INFINITY;
          if (p.out_index) p.out_index[o + r] = e < n ? static_cast<int64_t>(F.idx(e)) : -1;
        }
      }
      if (threadIdx.x == 0) JK_STAMP(16);
      compress_row(F, n, p.compress);
      if (threadIdx.x == 0) JK_STAMP(17);
      if (MODE == kGather && row_ok && good) {
        const int64_t cb = b * p.n_cols;
        float acc = 0.f;
        for (int e0 = 0; e0 < n; e0 += 8) {
          float st[8], sn[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const bool on = e0 + u < n;
            const int j = on ? F.idx(e0 + u) : 0;
            const uint32_t js = static_cast<uint32_t>(j - sr.s_lo);
            st[u] = !on ? 0.f : (js < n_stage ? st_stage[js] : ld_elem(p.col_state, cb + j, p.state_dtype));
            sn[u] = (on && p.col_sender) ? ld_elem(p.col_sender, cb + j, p.state_dtype) : 1.f;
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            if (e0 + u < n) {
              const float w = F.val(e0 + u) * sn[u];
              F.val(e0 + u) = w;
              acc = fmaf(w, st[u], acc);
            }
          }
        }
        st_elem(p.out_state, b * p.n_rows + t, p.out_dtype, acc);
        if (threadIdx.x == 0) JK_STAMP(18);
      }
      }
      if (MODE == kGather) {
        // Pack (weight, column) pairs for the aggregate, back to front so that every write
        // lands on an already consumed candidate slot of the same row (slot order kept).
        float* tab = bufv + gtab_off(row);
        for (int e = n - 1; e >= 0; --e) {
          const float w = F.val(e);
          const int j = F.idx(e);
          tab[2 * e] = w;
          tab[2 * e + 1] = __int_as_float(j);
        }
      }
    }
    fence_proxy_async_smem();  // candidate slots are reused by TMA and the MMAs next
    sel_barrier();
    JK_PHASE_MARK(4, t_prev);

    // ---- aggregate
    if (threadIdx.x == 0) {  // tell the MMA warp whether it issues the aggregate
      *agg_mode = tc_agg ? 1 : 0;
      mbar_arrive(slab_bar);
    }
    if (good) {
      const int nrows = kRows / kSelWarps;
      if (MODE == kGather) {
        if (tc_agg) {
          // Tensor-core aggregate over the CTA's source window. For every 64-row source
          // tile kt the selected edges of the 128 target rows form a sparse 128 x 64 matrix
          // E (bf16 / f16 hi + lo planes), the MMA's A operand in shared memory. Tile kt lies
          // in half kt & 1 of a score tile, so its columns are exactly the candidates the
          // selection half kt & 1 collected: the four warps of that half build it -- each
          // thread zeroes its row and stores the row's edges of the tile, walking its run
          // of packed (weight, column) survivors -- into buffer kt & 1, and signal e_full;
          // the two halves build alternate tiles. The MMA warp forms
          // O[128 x dim] += E_hi.V + E_lo.V in TMEM. The hi + lo planes keep the edge
          // weights to ~16 bits.
          constexpr bool kHalfV = std::is_same<VT, __half>::value;
          const int nkt = (sr.n + kEK - 1) / kEK;
          const int n = nsel[row];
          const int m0 = cnt[row];
          const float* tab = bufv + gtab_off(row);
          // rows of the exact fallback pass hold one sorted run, filtered by tile parity
          const bool runs = failrow[row] == 0;
          int cur = runs && half == 1 ? m0 : 0;
          const int end = runs && half == 0 ? m0 : n;
          auto next_rel = [&]() -> int {  // window-relative column of the next entry of this half
            while (cur < end) {
              const int rel = __float_as_int(tab[2 * cur + 1]) - sr.s_lo;
              if (((rel >> 6) & 1) == half) return rel;
              ++cur;
            }
            return INT_MAX;
          };
          int rel = next_rel();
          const uint32_t rsw = static_cast<uint32_t>(row & 7);
          const int rbase = (row >> 3) * 1024 + (row & 7) * 128;
          for (int kt = half, use = 0; kt < nkt; kt += 2, ++use) {
#ifdef JK_PHASE_PROFILE
            const long long tb0 = clock64();
#endif
            if (use >= 1 && !mbar_wait(&e_empty[half], (use - 1) & 1)) {
              atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
              *abort_flag = 1;
            }
            if (*abort_flag) break;
#ifdef JK_PHASE_PROFILE
            const long long tb1 = clock64();
#endif
            uint8_t* e_hi = smem + half * kETile + rbase;
            uint8_t* e_lo = e_hi + kETile / 2;
#pragma unroll
            for (int c = 0; c < 8; ++c) {  // through the swizzle: the warp's rows hit distinct banks
              const int o = (c ^ static_cast<int>(rsw)) << 4;
              *reinterpret_cast<uint4*>(e_hi + o) = make_uint4(0, 0, 0, 0);
              *reinterpret_cast<uint4*>(e_lo + o) = make_uint4(0, 0, 0, 0);
            }
            while ((rel >> 6) == kt) {
              const float w = tab[2 * cur];
              const int kin = rel & 63;
              const int off = ((static_cast<uint32_t>(kin >> 3) ^ rsw) << 4) + (kin & 7) * 2;
              if (kHalfV) {
                const __half h = __float2half_rn(w);
                *reinterpret_cast<__half*>(e_hi + off) = h;
                *reinterpret_cast<__half*>(e_lo + off) = __float2half_rn(w - __half2float(h));
              } else {
                const __nv_bfloat16 h = __float2bfloat16_rn(w);
                *reinterpret_cast<__nv_bfloat16*>(e_hi + off) = h;
                *reinterpret_cast<__nv_bfloat16*>(e_lo + off) = __float2bfloat16_rn(w - __bfloat162float(h));
              }
              ++cur;
              rel = next_rel();
            }
#ifdef JK_PHASE_PROFILE
            const long long tb2 = clock64();
#endif
            fence_proxy_async_smem();  // the MMA (async proxy) reads the tile next
#ifdef JK_PHASE_PROFILE
            if (threadIdx.x == 0 || threadIdx.x == 128) {
              const int tr = (blockIdx.y * gridDim.x + blockIdx.x) % kTraceCtas;
              const int o = threadIdx.x == 0 ? 24 : 27;
              g_trace[tr][o] += tb1 - tb0;
              g_trace[tr][o + 1] += tb2 - tb1;
              g_trace[tr][o + 2] += clock64() - tb2;
            }
#endif
            __syncwarp();
            if (lane == 0) mbar_arrive(&e_full[half]);
          }
          JK_PHASE_MARK(6, t_prev);
          if (!*abort_flag && !mbar_wait(agg_bar, 0)) {
            atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
            *abort_flag = 1;
          }
          tc_fence_after();
          JK_PHASE_MARK(7, t_prev);
          if (!*abort_flag && p.tma_out) {
            // O -> 16-bit rows staged in the (now free) candidate buffers as 64-column boxes
            // in the 128-byte-swizzled layout of tm_out, then stored by TMA (rows past
            // n_rows are clipped). Thread = row, half = which half of the columns.
            uint8_t* stg = reinterpret_cast<uint8_t*>(bufv);  // 1024-aligned, >= 96 KB
            const int hcols = static_cast<int>(p.dim / 2);      // multiple of 32
            const bool obf16 = p.out_dtype == JK_BF16;
            for (int c0 = 0; c0 < hcols; c0 += 32) {
              uint32_t v[32];
              tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + half * hcols + c0, v);
              tmem_ld_wait();
              const int col = half * hcols + c0;
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint32_t w4[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  const float a = __uint_as_float(v[8 * q + 2 * u]), c = __uint_as_float(v[8 * q + 2 * u + 1]);
                  if (obf16) {
                    __nv_bfloat162 h = __floats2bfloat162_rn(a, c);
                    w4[u] = *reinterpret_cast<uint32_t*>(&h);
                  } else {
                    __half2 h = __floats2half2_rn(a, c);
                    w4[u] = *reinterpret_cast<uint32_t*>(&h);
                  }
                }
                const int cc = col + 8 * q;
                const int chunk = (cc & 63) >> 3;
                *reinterpret_cast<uint4*>(stg + (cc >> 6) * (kRows * 128) + (row >> 3) * 1024 + (row & 7) * 128 +
                                          ((chunk ^ (row & 7)) << 4)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
              }
            }
            fence_proxy_async_smem();
            sel_barrier();
            if (threadIdx.x == 0) {
              for (int bx = 0; bx < static_cast<int>(p.dim / 64); ++bx)
                tma_store_3d(&tm_out, stg + bx * (kRows * 128), bx * 64, static_cast<int>(t0), static_cast<int>(b));
              bulk_commit_group();
              bulk_wait_group_read0();
            }
          } else if (!*abort_flag) {
            // O -> outputs (thread = row; half = which half of the columns)
            const int hcols = static_cast<int>(p.dim / 2);  // multiple of 32
            for (int c0 = 0; c0 < hcols; c0 += 32) {
              uint32_t v[32];
              tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + half * hcols + c0, v);
              tmem_ld_wait();
              if (row_ok) {
                const int64_t base = (b * p.n_rows + t) * p.dim + half * hcols + c0;
#pragma unroll
                for (int e = 0; e < 32; e += 8) {
                  float f[8];
#pragma unroll
                  for (int u = 0; u < 8; ++u) f[u] = __uint_as_float(v[e + u]);
                  store8(p.out_val, base + e, p.out_dtype, f);
                }
              }
            }
          }
        } else {
          gather_global<VT>(bufv, nsel, rt0, nrows, t0, b, p, lane);
        }
      } else {
        for (int r = 0; r < nrows; ++r) {
          const int rt = rt0 + r;
          if (t0 + rt >= p.n_rows) break;
          scatter_row<VT>(Lane{bufv + rt * kStride, bufi + rt * kStride}, nsel[rt], b, b * p.n_rows + t0 + rt, p,
                          lane);
        }
      }
    }
    JK_PHASE_MARK(5, t_prev);
    tc_fence_before();
  }
  __syncthreads();
  if (threadIdx.x == 0) JK_STAMP(9);
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int KATOMS, int MODE, typename VT>
int launch_vt(const CUtensorMap& tr, const CUtensorMap& tc, const CUtensorMap& tv, const CUtensorMap& to,
              const Params& p, int64_t batch,
              uint32_t idesc, cudaStream_t st) {
  constexpr int STAGES = KATOMS == 1 ? 4 : 1;
  constexpr int sm = Layout<KATOMS, STAGES>::kTotal;
  static_assert(sm <= 232448, "shared memory budget");
  auto kern = p.heads > 1 ? topk_kernel<KATOMS, STAGES, MODE, VT, true> : topk_kernel<KATOMS, STAGES, MODE, VT, false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sm) != cudaSuccess) {
    cudaGetLastError();
    return JK_ERR_LAUNCH;
  }
  const dim3 grid(static_cast<unsigned>((p.row_count + kRows - 1) / kRows), static_cast<unsigned>(batch));
  kern<<<grid, kThreads, sm, st>>>(tr, tc, tv, to, p, idesc);
  return launch_status();
}


// One unit instantiates the launchers of one value type (both score widths, both modes);
// the entry-point unit declares them extern.
#define JK_TOPK_INSTANTIATE(VT) \
  template int launch_vt<1, kGather, VT>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, \
      const CUtensorMap&, const Params&, int64_t, uint32_t, cudaStream_t); \
  template int launch_vt<1, kScatter, VT>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, \
      const CUtensorMap&, const Params&, int64_t, uint32_t, cudaStream_t); \
  template int launch_vt<2, kGather, VT>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, \
      const CUtensorMap&, const Params&, int64_t, uint32_t, cudaStream_t); \
  template int launch_vt<2, kScatter, VT>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, \
      const CUtensorMap&, const Params&, int64_t, uint32_t, cudaStream_t);
#define JK_TOPK_EXTERN(VT) \
  extern template int launch_vt<1, kGather, VT>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, \
      const CUtensorMap&, const Params&, int64_t, uint32_t, cudaStream_t); \
  extern template int launch_vt<1, kScatter, VT>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, \
      const CUtensorMap&, const Params&, int64_t, uint32_t, cudaStream_t); \
  extern template int launch_vt<2, kGather, VT>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, \
      const CUtensorMap&, const Params&, int64_t, uint32_t, cudaStream_t); \
  extern template int launch_vt<2, kScatter, VT>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, \
      const CUtensorMap&, const Params&, int64_t, uint32_t, cudaStream_t);

}  // namespace topk
}  // namespace jk
