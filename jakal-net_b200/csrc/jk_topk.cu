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
// Per CTA: 128 rows of one batch item, 9 warps.
//   warp 8 (producer): TMA-loads the row-side projection tile once and streams the
//          column-side tiles (128 columns x rp) through a smem ring; issues tcgen05.mma
//          (M=128 rows, N=128 columns, K=rp) into one of two TMEM accumulators, so the MMA
//          of one tile overlaps the selection work on the previous one. The column tiles
//          are streamed once per selection pass (scores are recomputed, never stored).
//   warps 0-7 (selection): two threads per row (warps w and w+4 read the same TMEM lanes),
//          each owning 64 of the 128 columns of every tile.
//     pass A (only when a row sees more than kCap columns): per-row mean and variance of
//          the visible scores -> a threshold tau expected to pass about k + 3 sqrt(k) + 8
//          columns (normal quantile).
//     pass B: every visible column with score >= tau is appended to the row's candidate
//          buffer (kCap slots in shared memory).
//     pass C (only if some row of the CTA got fewer than min(k, visible) or more than kCap
//          candidates -- a row far from normal): those rows redo an exact streaming
//          selection, each thread keeping a k-entry min-heap in the row's buffer.
//     select: one warp per row sorts the row's buffer (bitonic, 128 keys ordered by score
//          then lower column) and keeps the best k.
//   Then the k survivors are compressed into edges, and all 8 warps aggregate: a windowed
//   CTA stages its whole source range in shared memory 64 value columns at a time (TMA)
//   and gathers from there; otherwise 16-byte vector gathers from global memory; the
//   per-source transition scatters with vector atomics instead.
#include "jk_host.h"
#include "jk_sm100.cuh"

#include <cfloat>
#include <climits>
#include <type_traits>

namespace jk {
namespace topk {

#ifdef JK_PHASE_PROFILE
// Debug-only phase timer (sum over selection warps of clock64 deltas per phase).
__device__ unsigned long long g_phase[8];
#define JK_PHASE_MARK(i, t_prev)                                                                \
  do {                                                                                         \
    const long long _now = clock64();                                                          \
    if ((threadIdx.x & 31) == 0) atomicAdd(&g_phase[i], (unsigned long long)(_now - (t_prev))); \
    t_prev = _now;                                                                             \
  } while (0)
#else
#define JK_PHASE_MARK(i, t_prev) \
  do {                           \
  } while (0)
#endif

constexpr int kRows = 128;      // rows per CTA (MMA M)
constexpr int kCols = 128;      // columns per tile (MMA N)
constexpr int kHalfCols = 64;   // columns per selection thread per tile
constexpr int kCap = 128;       // candidate slots per row
constexpr int kQueue = 4;       // fallback queue slots per thread
constexpr int kStride = 137;    // row stride of the candidate buffer (odd: conflict-free)
constexpr int kSelWarps = 8;    // selection / aggregation warps
constexpr int kThreads = (kSelWarps + 1) * 32;
constexpr int kSentinel = INT_MAX;
static_assert(kStride >= kCap + 2 * kQueue, "buffer row holds candidates and both fallback queues");

enum Mode { kGather = 0, kScatter = 1 };

// Start (in floats, 16-byte aligned) of a row's packed gather table: (weight, column) pairs
// written over the row's candidate values once the edges are final.
__device__ __forceinline__ int gtab_off(int row) { return (row * kStride + 3) & ~3; }

struct Params {
  int64_t n_rows, n_cols, rp, dim;
  int k;
  int64_t window;  // < 0: no mask
  float bias;
  const float* bias_dev;
  int compress;
  int state_dtype, val_dtype, out_dtype;
  int slab_ok;  // tm_val is valid (windowed gather of 16-bit values, dim % 64 == 0)
  int split3;   // projections are the three-plane bf16 split of f32 values
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

// Replaces f.val(0..n) (sorted scores, bias included) by compressed edges.
__device__ void compress_row(const Lane& f, int n, int compress) {
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

__device__ __forceinline__ void store8(void* base, int64_t elem, int dtype, const float (&f)[8]) {
  if (dtype == JK_F32) {
    float4* q = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + elem);
    q[0] = make_float4(f[0], f[1], f[2], f[3]);
    q[1] = make_float4(f[4], f[5], f[6], f[7]);
  } else if (dtype == JK_BF16) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + elem) = u;
  } else {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(base) + elem) = u;
  }
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
__device__ void gather_row_generic(const float* tab, int n, int64_t col_base, int64_t row, const Params& p, int lane) {
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


// Sorts the valid candidates of a row into descending (score, lower column) order with one
// warp (bitonic network over NQ*32 64-bit keys) and writes the best min(k, valid) back to
// slots 0 ..; returns that count. Needs c0 + c1 <= NQ * 32.
template <int NQ>
__device__ int warp_select_row(float* rv, int* ri, int c0, int c1, int k, int lane) {
  constexpr int kN = NQ * 32;
  const unsigned long long kNone = make_key(-INFINITY, kSentinel);
  unsigned long long x[NQ];
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    // logical candidate i = q*32 + lane: the half-0 stack, then the half-1 stack
    const int i = q * 32 + lane;
    const int e = i < c0 ? i : kCap - 1 - (i - c0);
    x[q] = (i < c0 + c1 && ri[e] != kSentinel) ? make_key(rv[e], ri[e]) : kNone;
  }
#pragma unroll
  for (int size = 2; size <= kN; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        const int e = q * 32 + lane;
        const bool desc = (e & size) == 0;  // direction of this block
        if (stride >= 32) {
          const int qs = stride >> 5;
          if ((q & qs) == 0) {
            const int q2 = q | qs;
            const unsigned long long a = x[q], c = x[q2];
            const bool swap = desc ? (a < c) : (a > c);
            x[q] = swap ? c : a;
            x[q2] = swap ? a : c;
          }
        } else {
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, x[q], stride);
          const bool lower = (lane & stride) == 0;
          const bool take_max = (lower == desc);  // the lower element keeps the larger key
          const unsigned long long mx = x[q] > other ? x[q] : other;
          const unsigned long long mn = x[q] > other ? other : x[q];
          x[q] = take_max ? mx : mn;
        }
      }
    }
  }
  int valid = 0;
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    const int e = q * 32 + lane;
    valid += __popc(__ballot_sync(0xffffffffu, x[q] != kNone && e < k));
  }
  __syncwarp();
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    const int e = q * 32 + lane;
    if (e < valid) {
      rv[e] = key_val(x[q]);
      ri[e] = key_idx(x[q]);
    }
  }
  __syncwarp();
  return valid;
}

__device__ __forceinline__ void sel_barrier() {
  asm volatile("bar.sync 1, %0;" ::"r"(kSelWarps * 32) : "memory");
}

// ---------------------------------------------------------------- shared-memory layout
template <int KATOMS, int STAGES>
struct Layout {
  static constexpr int kAtomBytes = kRows * 128;  // 128 rows x 64 (16-bit) elements
  static constexpr int kABytes = KATOMS * kAtomBytes;
  static constexpr int kBBytes = KATOMS * kAtomBytes;
  static constexpr int kRegion0 = kABytes + STAGES * kBBytes;  // A + ring; reused as the value slab
  static constexpr int kBufBytes = 2 * kRows * kStride * 4;    // candidate values + indices
  static constexpr int kRowArrays = 10 * kRows * 4;            // per-row scalars
  static constexpr int kBarBytes = 256;
  static constexpr int kTotal = 1024 + kRegion0 + kBufBytes + kRowArrays + kBarBytes;
};

template <int KATOMS, int STAGES, int MODE, typename VT>
__global__ void __launch_bounds__(kThreads, 1)
    topk_kernel(const __grid_constant__ CUtensorMap tm_rows, const __grid_constant__ CUtensorMap tm_cols,
                const __grid_constant__ CUtensorMap tm_val, Params p, uint32_t idesc) {
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
  uint64_t* vb_full = bars + 4;   // [2] value tiles of the tensor-core aggregate
  uint64_t* vb_empty = bars + 6;  // [2]
  uint64_t* full = bars + 8;
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* any_fail = abort_flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t b = blockIdx.y;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kRows;
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
  const bool has_a = max_visible > kCap;
  const int pre_passes = has_a ? 2 : 1;

  if (threadIdx.x == 0) {
    mbar_init(bar_a, 1);
    mbar_init(decide, 1);
    mbar_init(slab_bar, 1);
    mbar_init(agg_bar, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&vb_full[i], 1);
      mbar_init(&vb_empty[i], 1);
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

  if (warp == kSelWarps) {
    // ------------------------------------------------------------ producer / MMA issuer
    if (lane == 0 && ntiles > 0) {
      prefetch_tmap(&tm_rows);
      prefetch_tmap(&tm_cols);
      bool ok = true;
      mbar_arrive_expect_tx(bar_a, L::kABytes);
#pragma unroll
      for (int a = 0; a < KATOMS; ++a)
        tma_load_3d(a_tile + a * L::kAtomBytes, &tm_rows, bar_a, a * 64, static_cast<int>(t0), static_cast<int>(b));
      int total = pre_passes * ntiles;  // grows by one pass if the fallback pass is needed
      const int decide_at = total - 1;
      int issued = 0;  // column-tile loads issued, in global iteration order
      auto issue_loads = [&](int upto) -> bool {
        while (issued <= upto && issued < total) {
          const int s = issued % STAGES;
          if (issued >= STAGES) {
            const int prev = issued - STAGES;  // the MMA that last read stage s
            if (!mbar_wait(&empty[s], (prev / STAGES) & 1)) return false;
          }
          mbar_arrive_expect_tx(&full[s], L::kBBytes);
          const int col0 = static_cast<int>((j_lo + issued % ntiles) * kCols);
#pragma unroll
          for (int a = 0; a < KATOMS; ++a)
            tma_load_3d(b_ring + s * L::kBBytes + a * L::kAtomBytes, &tm_cols, &full[s], a * 64, col0,
                        static_cast<int>(b));
          ++issued;
        }
        return true;
      };
      ok = issue_loads(STAGES - 1) && mbar_wait(bar_a, 0);
      for (int g = 0; g < total && ok; ++g) {
        const int st = g % STAGES;
        const int buf = g & 1;
        if (!mbar_wait(&full[st], (g / STAGES) & 1)) { ok = false; break; }
        if (g >= 2 && !mbar_wait(&tempty[buf], ((g >> 1) - 1) & 1)) { ok = false; break; }
        if (*abort_flag) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(a_tile);
        const uint32_t b_addr = smem_u32(b_ring + st * L::kBBytes);
        score_mmas<KATOMS>(tmem + buf * kCols, a_addr, b_addr, idesc, p.split3 != 0);
        mma_commit(&empty[st]);
        mma_commit(&tfull[buf]);
        if (g == decide_at) {
          // The selection warps report whether any row needs the exact fallback pass.
          if (!mbar_wait(decide, 0)) { ok = false; break; }
          if (*any_fail) total += ntiles;
        }
        // Stage reuse: with >= 2 stages load ahead behind the previous MMA, with one stage
        // behind this MMA.
        if (!issue_loads(STAGES == 1 ? g + 1 : g - 1 + STAGES)) { ok = false; break; }
      }
      // The MMA-retire arrivals on the ring barriers must land before the CTA exits.
      if (ok) {
        const int last = total - 1;
        ok = mbar_wait(&empty[last % STAGES], (last / STAGES) & 1);
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
#ifdef JK_PHASE_PROFILE
    long long t_prev = clock64();
#endif

    // Loads this thread's 64 scores of iteration g into v; false on timeout / abort.
    auto load_tile = [&](uint32_t (&v)[2][32]) -> bool {
      const int buf = g & 1;
      if (!mbar_wait(&tfull[buf], (g >> 1) & 1) || *abort_flag) return false;
      tc_fence_after();
      tmem_ld_32x32b_x32(tmem + tbase + buf * kCols, v[0]);
      tmem_ld_32x32b_x32(tmem + tbase + buf * kCols + 32, v[1]);
      tmem_ld_wait();
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
      s1[half * kRows + row] = a1;
      s2[half * kRows + row] = a2;
      sel_barrier();
      if (half == 0) {
        float th = -INFINITY;
        if (visible > kCap) {
          const float n = static_cast<float>(visible);
          const float mean = (s1[row] + s1[kRows + row]) / n;
          const float var = fmaxf((s2[row] + s2[kRows + row]) / n - mean * mean, 0.f);
          // Expected survivors: k plus ~3 standard deviations of the count, so that too few
          // is rare (the exact fallback pass covers it) and most rows fit a 64-key sort.
          const float target = fminf(static_cast<float>(k) + 3.f * sqrtf(static_cast<float>(k)) + 8.f, 0.75f * kCap);
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
      int myc = 0;
      for (int it = 0; it < ntiles && ok; ++it) {
        uint32_t v[2][32];
        if (!load_tile(v)) { ok = false; break; }
        const int col0 = static_cast<int>((j_lo + it) * kCols) + half * kHalfCols;
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int col = col0 + c * 32 + e;
            const float x = __uint_as_float(v[c][e]);
            if (static_cast<uint32_t>(col - lo_t) <= span && x >= th) {
              if (myc < kCap) {
                const int slot = half == 0 ? myc : kCap - 1 - myc;
                rv[slot] = x;
                ri[slot] = col;
              }
              ++myc;
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
    for (int r = 0; r < kRows / kSelWarps; ++r) {
      const int rt = rt0 + r;
      int n = 0;
      if (good && t0 + rt < p.n_rows) {
        float* wv = bufv + rt * kStride;
        int* wi = bufi + rt * kStride;
        const int c0 = cnt[rt];
        const int c1 = nsel[rt];
        n = c0 + c1 <= 64 ? warp_select_row<2>(wv, wi, c0, c1, k, lane)
                          : warp_select_row<4>(wv, wi, c0, c1, k, lane);
      }
      __syncwarp();
      if (lane == 0) nsel[rt] = n;
    }
    sel_barrier();
    JK_PHASE_MARK(3, t_prev);

    // ---- compress (thread per row), fold the sender strength, form the state output
    if (half == 0) {
      const Lane F{rv, ri};
      const int n = nsel[row];
      const float bias = p.bias + (p.bias_dev ? __ldg(p.bias_dev) : 0.f);
      for (int e = 0; e < n; ++e) F.val(e) += bias;
      if (MODE == kGather && row_ok && good && (p.out_scores || p.out_index)) {
        const int64_t o = (b * p.n_rows + t) * k;
        for (int e = 0; e < k; ++e) {
          if (p.out_scores) p.out_scores[o + e] = e < n ? F.val(e) : -INFINITY;
          if (p.out_index) p.out_index[o + e] = e < n ? static_cast<int64_t>(F.idx(e)) : -1;
        }
      }
      compress_row(F, n, p.compress);
      if (MODE == kGather && row_ok && good) {
        const int64_t cb = b * p.n_cols;
        float acc = 0.f;
        for (int e0 = 0; e0 < n; e0 += 8) {
          float st[8], sn[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const bool on = e0 + u < n;
            const int j = on ? F.idx(e0 + u) : 0;
            st[u] = on ? ld_elem(p.col_state, cb + j, p.state_dtype) : 0.f;
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
      }
      if (MODE == kGather) {
        // Pack (weight, column) pairs for the gather, back to front so that every write
        // lands on an already consumed candidate slot of the same row.
        float* tab = bufv + gtab_off(row);
        for (int e = n - 1; e >= 0; --e) {
          const float w = F.val(e);
          const int j = F.idx(e);
          tab[2 * e] = w;
          tab[2 * e + 1] = __int_as_float(j);
        }
      }
    }
    sel_barrier();
    JK_PHASE_MARK(4, t_prev);

    // ---- aggregate
    if (good) {
      const int nrows = kRows / kSelWarps;
      if (MODE == kGather) {
        int s_lo = 0, nslab = 0;
        bool slab = false;
        if (p.slab_ok && p.window >= 0 && sizeof(VT) == 2 && (p.dim % 64) == 0) {
          const int64_t lo = t0 - p.window;
          s_lo = lo > 0 ? static_cast<int>(lo) : 0;
          int64_t hi_col = t0 + kRows - 1;
          if (hi_col > p.n_cols - 1) hi_col = p.n_cols - 1;
          nslab = static_cast<int>(hi_col - s_lo + 1);
          slab = nslab > 0 && nslab <= 1024 && p.dim <= 512;  // dense enough; O fits TMEM
        }
        if (slab) {
          // Tensor-core aggregate over the CTA's source window: for every 128-row source
          // tile, the selected edges of the 128 target rows form a sparse 128 x 128 matrix
          // E, written (bf16 / f16 hi + lo planes) into the MMA operand region; thread 0
          // multiplies it with the tile's values 128 columns at a time (TMA, MN-major 128B
          // swizzle, double-buffered) into a TMEM accumulator O[128 x dim]:
          // O += E_hi.V + E_lo.V. The hi + lo planes keep the edge weights to ~16 bits.
          constexpr bool kHalfV = std::is_same<VT, __half>::value;
          const int ntile = (nslab + 127) / 128;
          const int nsl = static_cast<int>((p.dim + 127) / 128);  // 128-column value slices
          const int npair = ntile * nsl;
          uint8_t* e_hi = smem;              // 2 K atoms (32 KB)
          uint8_t* e_lo = smem + 2 * 16384;  // 2 K atoms (32 KB)
          uint8_t* vbuf = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(bufi) + 1023) & ~uintptr_t(1023));
          const int erow = row;  // this thread's target row
          auto slice_w = [&](int sl) { return static_cast<int>(p.dim - sl * 128 < 128 ? p.dim - sl * 128 : 128); };
          auto load_v = [&](int pi) {  // (tile, slice) pair pi -> buffer pi & 1
            const int st = pi / nsl, sl = pi % nsl, nb = slice_w(sl) / 64;
            mbar_arrive_expect_tx(&vb_full[pi & 1], nb * 16384);
            for (int a = 0; a < nb; ++a)
              tma_load_3d(vbuf + (pi & 1) * 32768 + a * 16384, &tm_val, &vb_full[pi & 1], sl * 128 + a * 64,
                          s_lo + st * 128, static_cast<int>(b));
          };
          if (threadIdx.x == 0) {
            fence_proxy_async_smem();  // the value buffers held generic candidate data before
            load_v(0);
            if (npair > 1) load_v(1);
          }
          for (int st = 0; st < ntile; ++st) {
            const int src0 = s_lo + st * 128;
            uint4* ez = reinterpret_cast<uint4*>(e_hi);
            for (int i = threadIdx.x; i < 4096; i += kSelWarps * 32) ez[i] = make_uint4(0, 0, 0, 0);
            sel_barrier();
            if (t0 + erow < p.n_rows) {
              const float* tab = bufv + gtab_off(erow);
              const int n = nsel[erow];
              for (int e = half; e < n; e += 2) {
                const int kcol = __float_as_int(tab[2 * e + 1]) - src0;
                if (static_cast<uint32_t>(kcol) < 128u) {
                  const float w = tab[2 * e];
                  const int kin = kcol & 63;
                  const int off = (kcol >> 6) * 16384 + (erow >> 3) * 1024 + (erow & 7) * 128 +
                                  (((kin >> 3) ^ (erow & 7)) << 4) + (kin & 7) * 2;
                  if (kHalfV) {
                    const __half h = __float2half_rn(w);
                    *reinterpret_cast<__half*>(e_hi + off) = h;
                    *reinterpret_cast<__half*>(e_lo + off) = __float2half_rn(w - __half2float(h));
                  } else {
                    const __nv_bfloat16 h = __float2bfloat16_rn(w);
                    *reinterpret_cast<__nv_bfloat16*>(e_hi + off) = h;
                    *reinterpret_cast<__nv_bfloat16*>(e_lo + off) = __float2bfloat16_rn(w - __bfloat162float(h));
                  }
                }
              }
            }
            fence_proxy_async_smem();
            sel_barrier();
            if (threadIdx.x == 0) {
              bool okm = true;
              for (int sl = 0; sl < nsl && okm; ++sl) {
                const int pi = st * nsl + sl;
                if (!mbar_wait(&vb_full[pi & 1], (pi >> 1) & 1)) { okm = false; break; }
                tc_fence_after();
                const int w = slice_w(sl);
                const uint32_t idesc_pv = idesc_f16(128, w, kHalfV ? 0u : 1u) | (1u << 16);
                const uint32_t vaddr = smem_u32(vbuf + (pi & 1) * 32768);
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                  const uint32_t eaddr = smem_u32(q == 0 ? e_hi : e_lo);
#pragma unroll
                  for (int kk = 0; kk < 8; ++kk) {
                    mma_f16_ss(tmem + sl * 128, sdesc_kmajor_sw128(eaddr + (kk >> 2) * 16384 + (kk & 3) * 32),
                               sdesc_mnmajor_sw128(vaddr + kk * 2048, 16384), idesc_pv,
                               (st > 0 || q > 0 || kk > 0) ? 1u : 0u);
                  }
                }
                mma_commit(&vb_empty[pi & 1]);
                if (pi + 2 < npair) {  // refill this buffer once its MMAs retired
                  if (!mbar_wait(&vb_empty[pi & 1], (pi >> 1) & 1)) { okm = false; break; }
                  load_v(pi + 2);
                }
              }
              if (okm) {
                mma_commit(agg_bar);
              } else {
                atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
                *abort_flag = 1;
              }
            }
            sel_barrier();
            if (*abort_flag) break;
            if (!mbar_wait(agg_bar, st & 1)) {  // E may be rewritten once its MMAs retired
              atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
              *abort_flag = 1;
              break;
            }
            tc_fence_after();
          }
          sel_barrier();
          if (!*abort_flag) {
            // O -> outputs (thread = row; half = which half of the columns)
            const int hcols = static_cast<int>(p.dim / 2);  // multiple of 32
            for (int c0 = 0; c0 < hcols; c0 += 32) {
              uint32_t v[32];
              tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + half * hcols + c0, v);
              tmem_ld_wait();
              if (t0 + erow < p.n_rows) {
                const int64_t base = (b * p.n_rows + t0 + erow) * p.dim + half * hcols + c0;
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
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Converts the f32 destination accumulators of the scatter mode into the outputs.
__global__ void finalize_scatter(const float* acc_state, const float* acc_val, int64_t n_state, int64_t n_val,
                                 void* out_state, void* out_val, int out_dtype) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t j = i; j < n_val; j += stride) st_elem(out_val, j, out_dtype, acc_val[j]);
  for (int64_t j = i; j < n_state; j += stride) st_elem(out_state, j, out_dtype, acc_state[j]);
}

template <int KATOMS, int MODE, typename VT>
int launch_vt(const CUtensorMap& tr, const CUtensorMap& tc, const CUtensorMap& tv, const Params& p, int64_t batch,
              uint32_t idesc, cudaStream_t st) {
  constexpr int STAGES = KATOMS == 1 ? 4 : 1;
  constexpr int sm = Layout<KATOMS, STAGES>::kTotal;
  static_assert(sm <= 232448, "shared memory budget");
  auto kern = topk_kernel<KATOMS, STAGES, MODE, VT>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sm) != cudaSuccess) {
    cudaGetLastError();
    return JK_ERR_LAUNCH;
  }
  const dim3 grid(static_cast<unsigned>((p.n_rows + kRows - 1) / kRows), static_cast<unsigned>(batch));
  kern<<<grid, kThreads, sm, st>>>(tr, tc, tv, p, idesc);
  return launch_status();
}

template <int KATOMS, int MODE>
int launch_k(const CUtensorMap& tr, const CUtensorMap& tc, const CUtensorMap& tv, const Params& p, int64_t batch,
             uint32_t idesc, cudaStream_t st) {
  switch (p.val_dtype) {
    case JK_F32: return launch_vt<KATOMS, MODE, float>(tr, tc, tv, p, batch, idesc, st);
    case JK_BF16: return launch_vt<KATOMS, MODE, __nv_bfloat16>(tr, tc, tv, p, batch, idesc, st);
    default: return launch_vt<KATOMS, MODE, __half>(tr, tc, tv, p, batch, idesc, st);
  }
}

template <int MODE>
int launch(const void* row_proj, const void* col_proj, int64_t batch, int64_t n_rows, int64_t n_cols, int64_t rp,
           int proj_dtype, Params& p, cudaStream_t st) {
  CUtensorMap tr, tc, tv;
  const bool bf16 = proj_dtype != JK_F16;
  p.split3 = proj_dtype == JK_BF16X3 ? 1 : 0;
  int status = make_tmap_3d_16bit(&tr, row_proj, rp, n_rows, batch, 64, kRows, bf16);
  if (status != JK_OK) return status;
  status = make_tmap_3d_16bit(&tc, col_proj, rp, n_cols, batch, 64, kCols, bf16);
  if (status != JK_OK) return status;
  tv = tc;  // placeholder when the slab path is off
  p.slab_ok = 0;
  if (MODE == kGather && p.window >= 0 && p.val_dtype != JK_F32 && p.dim % 64 == 0 && aligned16(p.col_val)) {
    if (make_tmap_3d_16bit(&tv, p.col_val, p.dim, n_cols, batch, 64, 128, p.val_dtype == JK_BF16, true) == JK_OK)
      p.slab_ok = 1;
  }
  const uint32_t idesc = idesc_f16(kRows, kCols, bf16 ? 1u : 0u);
  if (rp == 64) return launch_k<1, MODE>(tr, tc, tv, p, batch, idesc, st);
  return launch_k<2, MODE>(tr, tc, tv, p, batch, idesc, st);
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

extern "C" int jk_propagation_topk_forward(const void* row_proj, const void* col_proj, int64_t batch, int64_t n_rows,
                                           int64_t n_cols, int64_t rp, int proj_dtype, const void* col_state,
                                           const void* col_sender, int state_dtype, const void* col_val, int64_t dim,
                                           int val_dtype, int64_t k, int64_t window, float score_bias,
                                           const float* bias_dev, int compress, void* out_state, void* out_val,
                                           int out_dtype, float* out_scores, int64_t* out_index, jk_stream_t stream) {
  using namespace jk;
  int st = topk::validate_common(row_proj, col_proj, batch, n_rows, n_cols, rp, proj_dtype, col_state, state_dtype,
                                 col_val, dim, val_dtype, k, compress, out_dtype);
  if (st != JK_OK) return st;
  if (out_state == nullptr || out_val == nullptr) return JK_ERR_BAD_ARG;
  if (dim % 8 == 0 && !aligned16(out_val)) return JK_ERR_ALIGNMENT;
  if (window < -1) return JK_ERR_BAD_ARG;
  st = check_device();
  if (st != JK_OK) return st;
  topk::Params p{};
  p.n_rows = n_rows;
  p.n_cols = n_cols;
  p.rp = rp;
  p.dim = dim;
  p.k = static_cast<int>(k);
  p.window = window;
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
  return topk::launch<topk::kGather>(row_proj, col_proj, batch, n_rows, n_cols, rp, proj_dtype, p,
                                     reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int jk_transition_query_topk_forward(const void* query_proj, const void* source_proj, int64_t batch,
                                                int64_t n_query, int64_t n_source, int64_t rp, int proj_dtype,
                                                const void* source_state, const void* source_sender, int state_dtype,
                                                const void* source_val, int64_t dim, int val_dtype, int64_t k,
                                                float score_bias, const float* bias_dev, int compress,
                                                void* out_state, void* out_val, int out_dtype, float* out_scores,
                                                int64_t* out_index, jk_stream_t stream) {
  return jk_propagation_topk_forward(query_proj, source_proj, batch, n_query, n_source, rp, proj_dtype, source_state,
                                     source_sender, state_dtype, source_val, dim, val_dtype, k, -1, score_bias,
                                     bias_dev, compress, out_state, out_val, out_dtype, out_scores, out_index, stream);
}

extern "C" int jk_transition_pairwise_topk_forward(const void* src_proj, const void* dst_proj, int64_t batch,
                                                   int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                                   const void* src_state, const void* src_sender, int state_dtype,
                                                   const void* src_val, int64_t dim, int val_dtype, int64_t k,
                                                   float score_bias, const float* bias_dev, int compress,
                                                   float* accum, void* out_state, void* out_val, int out_dtype,
                                                   jk_stream_t stream) {
  using namespace jk;
  int st = topk::validate_common(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, src_state, state_dtype,
                                 src_val, dim, val_dtype, k, compress, out_dtype);
  if (st != JK_OK) return st;
  if (accum == nullptr || out_state == nullptr || out_val == nullptr) return JK_ERR_BAD_ARG;
  if (!aligned16(accum)) return JK_ERR_ALIGNMENT;
  st = check_device();
  if (st != JK_OK) return st;
  auto cs = reinterpret_cast<cudaStream_t>(stream);
  const int64_t n_state = batch * n_dst;
  const int64_t n_val = batch * n_dst * dim;
  // Value accumulators first (16-byte aligned for the vector atomics), then state.
  float* acc_val = accum;
  float* acc_state = accum + n_val;
  if (cudaMemsetAsync(accum, 0, sizeof(float) * (n_state + n_val), cs) != cudaSuccess) return launch_status();
  topk::Params p{};
  p.n_rows = n_src;
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
  st = topk::launch<topk::kScatter>(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, p, cs);
  if (st != JK_OK) return st;
  const int64_t work = n_val > n_state ? n_val : n_state;
  int blocks = static_cast<int>((work + 255) / 256);
  if (blocks > 4 * 148 * 8) blocks = 4 * 148 * 8;
  if (blocks < 1) blocks = 1;
  topk::finalize_scatter<<<blocks, 256, 0, cs>>>(acc_state, acc_val, n_state, n_val, out_state, out_val, out_dtype);
  return launch_status();
}

#ifdef JK_PHASE_PROFILE
extern "C" int jk_debug_phase(unsigned long long* out, int reset) {
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(out, jk::topk::g_phase, sizeof(unsigned long long) * 8);
  if (reset) {
    unsigned long long z[8] = {0};
    cudaMemcpyToSymbol(jk::topk::g_phase, z, sizeof(z));
  }
  return 0;
}
#endif
