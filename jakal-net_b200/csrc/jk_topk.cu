// Fused low-rank score -> streaming top-k -> edge compress -> aggregate kernel.
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
//   warp 8  (producer): TMA-loads the row-side projection tile once and streams the
//           column-side tiles (128 columns x rp) through a multi-stage smem ring; issues
//           tcgen05.mma (M=128 rows, N=128 columns, K=rp) into one of two TMEM
//           accumulators, so the MMA of tile j+1 overlaps the selection of tile j.
//   warps 0-7 (selection): two threads per row (warps w and w+4 read the same TMEM lanes);
//           each owns 64 of the 128 columns of every tile. A thread keeps a k-entry
//           min-heap (root = its current k-th best) in shared memory laid out
//           [slot][row] so every access is bank-conflict free. Candidates are filtered
//           against max(own root, partner's published root) -- a valid lower bound of the
//           row's k-th best -- queued per thread and merged into the heap in warp-wide
//           flushes, so lanes do not diverge per candidate. After the last tile both heaps
//           are sorted and merged, compressed into edges, and all 8 warps aggregate the
//           128 rows with 16-byte vector loads of the picked value rows (gather) or vector
//           atomics into the destination rows (scatter).
#include "jk_host.h"
#include "jk_sm100.cuh"

#include <cfloat>
#include <climits>

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

constexpr int kRows = 128;       // rows per CTA (MMA M)
constexpr int kCols = 128;       // columns per tile (MMA N)
constexpr int kHalfCols = 64;    // columns per selection thread per tile
constexpr int kQueue = 8;        // per-thread candidate queue depth
constexpr int kSelWarps = 8;     // selection / aggregation warps
constexpr int kThreads = (kSelWarps + 1) * 32;
constexpr int kSentinel = INT_MAX;

enum Mode { kGather = 0, kScatter = 1 };

struct Params {
  int64_t n_rows, n_cols, rp, dim;
  int k;
  int64_t window;  // < 0: no mask
  float bias;
  const float* bias_dev;
  int compress;
  int state_dtype, val_dtype, out_dtype;
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

// One thread's slice of a [slot][row] array pair (stride kRows).
struct Lane {
  float* v;
  int* i;
  __device__ __forceinline__ float& val(int slot) const { return v[slot * kRows]; }
  __device__ __forceinline__ int& idx(int slot) const { return i[slot * kRows]; }
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

// In-place heapsort of a min-heap -> entries sorted best first.
__device__ __forceinline__ void heap_sort(const Lane& h, int k) {
  for (int end = k - 1; end > 0; --end) {
    const float x = h.val(end);
    const int id = h.idx(end);
    h.val(end) = h.val(0);
    h.idx(end) = h.idx(0);
    heap_sift_root(h, end, x, id);
  }
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
    const float m = f.val(0);  // sorted: first is the max
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

// Generic aggregation of one row by one warp (any dim / f32 values): lanes stride the
// value dimension; the final weights already include the sender strength.
__device__ void gather_row_generic(const Lane& f, int n, int64_t col_base, int64_t row, const Params& p, int lane) {
  const int64_t D = p.dim;
  for (int64_t d0 = 0; d0 < D; d0 += 32) {
    const int64_t d = d0 + lane;
    float acc = 0.f;
    for (int e = 0; e < n; ++e) {
      const int j = f.idx(e);
      if (d < D) acc = fmaf(f.val(e), ld_elem(p.col_val, (col_base + j) * D + d, p.val_dtype), acc);
    }
    if (d < D) st_elem(p.out_val, row * D + d, p.out_dtype, acc);
  }
}

// Aggregation of `nrows` rows (tile rows rt0 ..) by one warp for 16-bit values.
//
// Work items are (row, 8-element chunk) pairs of a group of rows spread over the 32
// lanes, so every lane keeps up to 16 independent 16-byte loads in flight per step (8
// items x 2 neighbours) whatever the value width, which hides the L2 / HBM latency of the
// random gathers. Accumulation is f32; each item is stored once.
template <typename VT>
__device__ void gather_warp(float* fv, int* fi, int* nsel, int rt0, int nrows, int64_t t0, int64_t b,
                            const Params& p, int lane) {
  constexpr int kItems = 8;
  const int64_t D = p.dim;
  const int64_t col_base = b * p.n_cols;
  if ((D % 8) != 0 || D > 8 * 32 * kItems || sizeof(VT) == 4) {
    for (int r = 0; r < nrows; ++r) {
      const int rt = rt0 + r;
      const int64_t row = t0 + rt;
      if (row >= p.n_rows) break;
      gather_row_generic(Lane{fv + rt, fi + rt}, nsel[rt], col_base, b * p.n_rows + row, p, lane);
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
          const int slot = (on ? i + u : 0) * kRows + rq[m];
          const int j = fi[slot];
          w[m][u] = on ? fv[slot] : 0.f;
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

__device__ __forceinline__ void sel_barrier() {
  asm volatile("bar.sync 1, %0;" ::"r"(kSelWarps * 32) : "memory");
}

template <int KMAX, int KATOMS, int STAGES>
struct Layout {
  static constexpr int kAtomBytes = kRows * 128;  // 128 rows x 64 (16-bit) elements
  static constexpr int kABytes = KATOMS * kAtomBytes;
  static constexpr int kBBytes = KATOMS * kAtomBytes;
  static constexpr int kRegion0 = kABytes + STAGES * kBBytes;  // A + ring; reused for the final lists
  static constexpr int kFinalBytes = 2 * KMAX * kRows * 4;
  static_assert(kFinalBytes <= kRegion0, "final lists must fit in the MMA operand region");
  static constexpr int kHeapBytes = 2 * 2 * KMAX * kRows * 4;  // 2 halves x (value, index)
  static constexpr int kQueueBytes = 2 * 2 * kQueue * kRows * 4;
  static constexpr int kPubBytes = 2 * kRows * 4;
  static constexpr int kNselBytes = kRows * 4;
  static constexpr int kBarBytes = 256;
  static constexpr int kTotal = 1024 + kRegion0 + kHeapBytes + kQueueBytes + kPubBytes + kNselBytes + kBarBytes;
};

template <int KMAX, int KATOMS, int STAGES, int MODE, typename VT>
__global__ void __launch_bounds__(kThreads, 1)
    topk_kernel(const __grid_constant__ CUtensorMap tm_rows, const __grid_constant__ CUtensorMap tm_cols,
                Params p, uint32_t idesc) {
  using L = Layout<KMAX, KATOMS, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tile = smem;
  uint8_t* b_ring = smem + L::kABytes;
  float* fv = reinterpret_cast<float*>(smem);  // final lists (after streaming)
  int* fi = reinterpret_cast<int*>(fv + KMAX * kRows);
  float* hv = reinterpret_cast<float*>(smem + L::kRegion0);  // [2][KMAX][kRows]
  int* hi = reinterpret_cast<int*>(hv + 2 * KMAX * kRows);
  float* qv = reinterpret_cast<float*>(hi + 2 * KMAX * kRows);  // [2][kQueue][kRows]
  int* qi = reinterpret_cast<int*>(qv + 2 * kQueue * kRows);
  volatile float* pub = reinterpret_cast<volatile float*>(qi + 2 * kQueue * kRows);  // [2][kRows]
  int* nsel = reinterpret_cast<int*>(const_cast<float*>(pub) + 2 * kRows);
  uint64_t* bars = reinterpret_cast<uint64_t*>(nsel + kRows);
  uint64_t* bar_a = bars;
  uint64_t* full = bars + 1;
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t b = blockIdx.y;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kRows;
  const int k = p.k;

  // Column-tile range.
  int64_t j_lo = 0, j_hi = (p.n_cols + kCols - 1) / kCols - 1;
  if (p.window >= 0) {
    const int64_t lo = t0 - p.window;
    j_lo = lo > 0 ? lo / kCols : 0;
    int64_t hi_col = t0 + kRows - 1;
    if (hi_col > p.n_cols - 1) hi_col = p.n_cols - 1;
    j_hi = hi_col < 0 ? -1 : hi_col / kCols;
  }
  const int ntiles = j_hi >= j_lo ? static_cast<int>(j_hi - j_lo + 1) : 0;

  if (threadIdx.x == 0) {
    mbar_init(bar_a, 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kSelWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 256);
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
      const int pre = ntiles < STAGES ? ntiles : STAGES;
      for (int it = 0; it < pre; ++it) {
        mbar_arrive_expect_tx(&full[it], L::kBBytes);
        const int col0 = static_cast<int>((j_lo + it) * kCols);
#pragma unroll
        for (int a = 0; a < KATOMS; ++a)
          tma_load_3d(b_ring + it * L::kBBytes + a * L::kAtomBytes, &tm_cols, &full[it], a * 64, col0,
                      static_cast<int>(b));
      }
      ok = mbar_wait(bar_a, 0);
      for (int it = 0; it < ntiles && ok; ++it) {
        const int st = it % STAGES;
        const int buf = it & 1;
        if (!mbar_wait(&full[st], (it / STAGES) & 1)) { ok = false; break; }
        if (it >= 2 && !mbar_wait(&tempty[buf], ((it >> 1) - 1) & 1)) { ok = false; break; }
        if (*abort_flag) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(a_tile);
        const uint32_t b_addr = smem_u32(b_ring + st * L::kBBytes);
#pragma unroll
        for (int kk = 0; kk < 4 * KATOMS; ++kk) {
          const uint32_t off = (kk >> 2) * L::kAtomBytes + (kk & 3) * 32;
          mma_f16_ss(tmem + buf * kCols, sdesc_kmajor_sw128(a_addr + off), sdesc_kmajor_sw128(b_addr + off), idesc,
                     kk > 0 ? 1u : 0u);
        }
        mma_commit(&empty[st]);
        mma_commit(&tfull[buf]);
        // Refill the stage the previous tile used (its MMA has most likely retired); with a
        // single stage, the stage of this tile once its own MMA retires.
        const int ip = STAGES == 1 ? it : it - 1;
        if (ip >= 0 && ip + STAGES < ntiles) {
          const int sp = ip % STAGES;
          if (!mbar_wait(&empty[sp], (ip / STAGES) & 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[sp], L::kBBytes);
          const int col0 = static_cast<int>((j_lo + ip + STAGES) * kCols);
#pragma unroll
          for (int a = 0; a < KATOMS; ++a)
            tma_load_3d(b_ring + sp * L::kBBytes + a * L::kAtomBytes, &tm_cols, &full[sp], a * 64, col0,
                        static_cast<int>(b));
        }
      }
      // The MMA-retire arrivals on the ring barriers must land before the CTA exits.
      if (ok) {
        const int last = ntiles - 1;
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
    if (!row_ok || hi_t < lo_t) {  // nothing visible: an unreachable single-column range
      lo_t = INT_MAX / 2;
      hi_t = INT_MAX / 2;
    }
    const uint32_t span = static_cast<uint32_t>(hi_t - lo_t);
    const Lane heap{hv + half * KMAX * kRows + row, hi + half * KMAX * kRows + row};
    const Lane queue{qv + half * kQueue * kRows + row, qi + half * kQueue * kRows + row};
    for (int e = 0; e < k; ++e) {
      heap.val(e) = -INFINITY;
      heap.idx(e) = kSentinel;
    }
    pub[half * kRows + row] = -INFINITY;
    float thr_own = -INFINITY, thr_part = -INFINITY;
    int qn = 0;
    bool ok = true;
    const uint32_t tbase = (static_cast<uint32_t>(quad * 32) << 16) + half * kHalfCols;
#ifdef JK_PHASE_PROFILE
    long long t_prev = clock64();
#endif
    sel_barrier();  // heaps and published roots initialised
    for (int it = 0; it < ntiles; ++it) {
      const int buf = it & 1;
      if (!mbar_wait(&tfull[buf], (it >> 1) & 1) || *abort_flag) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t v[2][32];
      tmem_ld_32x32b_x32(tmem + tbase + buf * kCols, v[0]);
      tmem_ld_32x32b_x32(tmem + tbase + buf * kCols + 32, v[1]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      const int col0 = static_cast<int>((j_lo + it) * kCols) + half * kHalfCols;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int col = col0 + c * 32 + e + u;
            const float x = __uint_as_float(v[c][e + u]);
            const bool pass = static_cast<uint32_t>(col - lo_t) <= span && x > thr_own && x >= thr_part;
            if (pass) {
              queue.val(qn) = x;
              queue.idx(qn) = col;
              ++qn;
            }
          }
          if (__any_sync(0xffffffffu, qn > kQueue - 4)) {
            thr_own = flush_queue(heap, queue, k, qn);
            pub[half * kRows + row] = thr_own;
            thr_part = pub[(half ^ 1) * kRows + row];
          }
        }
      }
    }
    if (ok) {
      flush_queue(heap, queue, k, qn);
      JK_PHASE_MARK(0, t_prev);
      heap_sort(heap, k);
    }
    sel_barrier();  // both halves sorted; MMA operand region is free
    JK_PHASE_MARK(1, t_prev);
    if (!ok) {
      atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
      *abort_flag = 1;
    }
    sel_barrier();
    const bool good = !*abort_flag;
    if (half == 0) {
      // Merge the two sorted halves (best first, ties to the lower column) into the
      // final list, compress it, fold in the sender strength and form the state output.
      const Lane A{hv + row, hi + row};
      const Lane Bh{hv + KMAX * kRows + row, hi + KMAX * kRows + row};
      const Lane F{fv + row, fi + row};
      int ia = 0, ib = 0, n = 0;
      if (good && row_ok) {
        while (n < k) {
          const float av = ia < k ? A.val(ia) : -INFINITY;
          const float bv = ib < k ? Bh.val(ib) : -INFINITY;
          const int ai = ia < k ? A.idx(ia) : kSentinel;
          const int bi = ib < k ? Bh.idx(ib) : kSentinel;
          const bool take_a = worse(bv, bi, av, ai);
          const int id = take_a ? ai : bi;
          if (id == kSentinel) break;
          F.val(n) = take_a ? av : bv;
          F.idx(n) = id;
          ++n;
          if (take_a) ++ia; else ++ib;
        }
      }
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
      nsel[row] = n;
    }
    sel_barrier();  // final lists ready
    JK_PHASE_MARK(2, t_prev);
    if (good) {
      // Aggregate: warp w handles rows 16w .. 16w+15.
      const int rt0 = warp * (kRows / kSelWarps);
      if (MODE == kGather) {
        gather_warp<VT>(fv, fi, nsel, rt0, kRows / kSelWarps, t0, b, p, lane);
      } else {
        for (int r = 0; r < kRows / kSelWarps; ++r) {
          const int rt = rt0 + r;
          if (t0 + rt >= p.n_rows) break;
          scatter_row<VT>(Lane{fv + rt, fi + rt}, nsel[rt], b, b * p.n_rows + t0 + rt, p, lane);
        }
      }
    }
    JK_PHASE_MARK(3, t_prev);
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
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

template <int KMAX, int KATOMS, int MODE, typename VT>
int launch_vt(const CUtensorMap& tr, const CUtensorMap& tc, const Params& p, int64_t batch, uint32_t idesc,
              cudaStream_t st) {
  constexpr int STAGES = KATOMS == 1 ? (KMAX > 32 ? 3 : 4) : (KMAX > 32 ? 1 : 2);
  constexpr int sm = Layout<KMAX, KATOMS, STAGES>::kTotal;
  static_assert(sm <= 232448, "shared memory budget");
  auto kern = topk_kernel<KMAX, KATOMS, STAGES, MODE, VT>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sm) != cudaSuccess) {
    cudaGetLastError();
    return JK_ERR_LAUNCH;
  }
  const dim3 grid(static_cast<unsigned>((p.n_rows + kRows - 1) / kRows), static_cast<unsigned>(batch));
  kern<<<grid, kThreads, sm, st>>>(tr, tc, p, idesc);
  return launch_status();
}

template <int KMAX, int KATOMS, int MODE>
int launch_k(const CUtensorMap& tr, const CUtensorMap& tc, const Params& p, int64_t batch, uint32_t idesc,
             cudaStream_t st) {
  switch (p.val_dtype) {
    case JK_F32: return launch_vt<KMAX, KATOMS, MODE, float>(tr, tc, p, batch, idesc, st);
    case JK_BF16: return launch_vt<KMAX, KATOMS, MODE, __nv_bfloat16>(tr, tc, p, batch, idesc, st);
    default: return launch_vt<KMAX, KATOMS, MODE, __half>(tr, tc, p, batch, idesc, st);
  }
}

template <int MODE>
int launch(const void* row_proj, const void* col_proj, int64_t batch, int64_t n_rows, int64_t n_cols, int64_t rp,
           int proj_dtype, Params& p, cudaStream_t st) {
  CUtensorMap tr, tc;
  const bool bf16 = proj_dtype == JK_BF16;
  int status = make_tmap_3d_16bit(&tr, row_proj, rp, n_rows, batch, 64, kRows, bf16);
  if (status != JK_OK) return status;
  status = make_tmap_3d_16bit(&tc, col_proj, rp, n_cols, batch, 64, kCols, bf16);
  if (status != JK_OK) return status;
  const uint32_t idesc = idesc_f16(kRows, kCols, bf16 ? 1u : 0u);
  const bool small_k = p.k <= 32;
  if (rp == 64) {
    return small_k ? launch_k<32, 1, MODE>(tr, tc, p, batch, idesc, st)
                   : launch_k<64, 1, MODE>(tr, tc, p, batch, idesc, st);
  }
  return small_k ? launch_k<32, 2, MODE>(tr, tc, p, batch, idesc, st)
                 : launch_k<64, 2, MODE>(tr, tc, p, batch, idesc, st);
}

int validate_common(const void* row_proj, const void* col_proj, int64_t batch, int64_t n_rows, int64_t n_cols,
                    int64_t rp, int proj_dtype, const void* state, int state_dtype, const void* val, int64_t dim,
                    int val_dtype, int64_t k, int compress, int out_dtype) {
  if (row_proj == nullptr || col_proj == nullptr || state == nullptr || val == nullptr) return JK_ERR_BAD_ARG;
  if (proj_dtype != JK_BF16 && proj_dtype != JK_F16) return JK_ERR_BAD_DTYPE;
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
