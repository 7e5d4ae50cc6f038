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
// Per CTA: 128 rows of one batch item.
//   warp 4  (producer): TMA-loads the row-side projection tile once and streams the
//           column-side tiles (128 columns x rp) through a multi-stage smem ring; issues
//           tcgen05.mma (M=128 rows, N=128 columns, K=rp) into one of two TMEM
//           accumulators, so the MMA of tile j+1 overlaps the epilogue of tile j.
//   warps 0-3 (epilogue): thread i owns row i (TMEM lane i). It reads its 128 scores with
//           tcgen05.ld, applies the visibility mask, and keeps a k-entry min-heap (root =
//           current k-th best) in shared memory laid out [slot][thread] so every access
//           is bank-conflict free. Candidates above the root are queued per thread and
//           merged into the heap in warp-wide flushes, so lanes do not diverge per
//           candidate. After the last tile the heap is sorted, compressed into edges, and
//           each warp aggregates its 32 rows with 16-byte vector loads of the selected
//           value rows (gather) or vector atomics into the destination rows (scatter).
#include "jk_host.h"
#include "jk_sm100.cuh"

#include <cfloat>
#include <climits>

namespace jk {
namespace topk {

constexpr int kRows = 128;     // rows per CTA (MMA M)
constexpr int kCols = 128;     // columns per tile (MMA N)
constexpr int kQueue = 8;      // per-thread candidate queue depth
constexpr int kThreads = 160;  // 4 epilogue warps + 1 producer warp
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
  // state / value / sender (row_state etc.).
  float* acc_state;
  float* acc_val;
};

__device__ __forceinline__ bool worse(float av, int ai, float bv, int bi) {
  return av < bv || (av == bv && ai > bi);
}

struct Smem {
  float* hv;  // [KMAX][128]
  int* hi;    // [KMAX][128]
  float* qv;  // [kQueue][128]
  int* qi;    // [kQueue][128]
  float* aux; // [KMAX][128]
  int* nsel;  // [128]
};

// Sift (v, id) down from the root of the thread's heap of size k.
__device__ __forceinline__ void heap_sift_root(const Smem& s, int tid, int k, float v, int id) {
  int pos = 0;
  while (true) {
    int c = 2 * pos + 1;
    if (c >= k) break;
    float cv = s.hv[c * kRows + tid];
    int ci = s.hi[c * kRows + tid];
    if (c + 1 < k) {
      const float rv = s.hv[(c + 1) * kRows + tid];
      const int ri = s.hi[(c + 1) * kRows + tid];
      if (worse(rv, ri, cv, ci)) { c = c + 1; cv = rv; ci = ri; }
    }
    if (worse(cv, ci, v, id)) {
      s.hv[pos * kRows + tid] = cv;
      s.hi[pos * kRows + tid] = ci;
      pos = c;
    } else {
      break;
    }
  }
  s.hv[pos * kRows + tid] = v;
  s.hi[pos * kRows + tid] = id;
}

// Merge the queued candidates of this thread into its heap; returns the new threshold.
__device__ __forceinline__ float flush_queue(const Smem& s, int tid, int k, int& qn) {
  float root_v = s.hv[tid];
  int root_i = s.hi[tid];
  for (int q = 0; q < qn; ++q) {
    const float v = s.qv[q * kRows + tid];
    const int id = s.qi[q * kRows + tid];
    if (worse(root_v, root_i, v, id)) {
      heap_sift_root(s, tid, k, v, id);
      root_v = s.hv[tid];
      root_i = s.hi[tid];
    }
  }
  qn = 0;
  return root_v;
}

// In-place heapsort of the thread's min-heap -> entries sorted best first.
__device__ __forceinline__ void heap_sort(const Smem& s, int tid, int k) {
  for (int end = k - 1; end > 0; --end) {
    const float v = s.hv[end * kRows + tid];
    const int id = s.hi[end * kRows + tid];
    s.hv[end * kRows + tid] = s.hv[tid];
    s.hi[end * kRows + tid] = s.hi[tid];
    heap_sift_root(s, tid, end, v, id);
  }
}

// Replaces hv[0..n) (sorted scores, bias included) by compressed edges.
__device__ void compress_row(const Smem& s, int tid, int n, int compress) {
  if (n <= 0) return;
  if (compress == JK_SOFTSIGN) {
    for (int i = 0; i < n; ++i) {
      const float x = s.hv[i * kRows + tid];
      s.hv[i * kRows + tid] = x / (1.f + fabsf(x));
    }
  } else if (compress == JK_SOFTMAX) {
    const float m = s.hv[tid];  // sorted: first is the max
    float z = 0.f;
    for (int i = 0; i < n; ++i) z += expf(s.hv[i * kRows + tid] - m);
    const float inv = 1.f / z;
    for (int i = 0; i < n; ++i) s.hv[i * kRows + tid] = expf(s.hv[i * kRows + tid] - m) * inv;
  } else if (compress == JK_SIGNED_ABS_SOFTMAX) {
    float m = 0.f;
    for (int i = 0; i < n; ++i) m = fmaxf(m, fabsf(s.hv[i * kRows + tid]));
    float z = 0.f;
    for (int i = 0; i < n; ++i) z += expf(fabsf(s.hv[i * kRows + tid]) - m);
    const float inv = 1.f / z;
    for (int i = 0; i < n; ++i) {
      const float x = s.hv[i * kRows + tid];
      const float sg = x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
      s.hv[i * kRows + tid] = sg * expf(fabsf(x) - m) * inv;
    }
  } else {  // JK_SIGNED_ENTMAX15 over |s| (kernels.py:155-210 restated)
    // Magnitudes sorted descending by insertion sort into aux.
    for (int i = 0; i < n; ++i) {
      const float a = fabsf(s.hv[i * kRows + tid]);
      int j = i;
      while (j > 0 && s.aux[(j - 1) * kRows + tid] < a) {
        s.aux[j * kRows + tid] = s.aux[(j - 1) * kRows + tid];
        --j;
      }
      s.aux[j * kRows + tid] = a;
    }
    const float zmax = s.aux[tid];
    // tau_rho for rho = 1..n on shifted = (z - zmax) / 2; support = #{rho : tau_rho <= z_rho}.
    float cum = 0.f, cum_sq = 0.f, tau_star = 0.f;
    int support = 0;
    float tau_first = 0.f;
    for (int r = 0; r < n; ++r) {
      const float x = (s.aux[r * kRows + tid] - zmax) * 0.5f;
      cum += x;
      cum_sq += x * x;
      const float rho = static_cast<float>(r + 1);
      const float mean = cum / rho;
      const float mean_sq = cum_sq / rho;
      const float var = rho * (mean_sq - mean * mean);
      const float delta = fmaxf((1.f - var) / rho, 0.f);
      const float tau = mean - sqrtf(delta);
      if (r == 0) tau_first = tau;
      if (tau <= x) { ++support; tau_star = tau; }
    }
    // torch: tau.gather(support - 1) with support >= 1 -> tau at index (support-1).
    // Recompute tau at that rho exactly as the reference (cumulative formula).
    if (support == 0) tau_star = tau_first;
    else {
      cum = 0.f; cum_sq = 0.f;
      for (int r = 0; r < support; ++r) {
        const float x = (s.aux[r * kRows + tid] - zmax) * 0.5f;
        cum += x;
        cum_sq += x * x;
      }
      const float rho = static_cast<float>(support);
      const float mean = cum / rho;
      const float mean_sq = cum_sq / rho;
      const float var = rho * (mean_sq - mean * mean);
      const float delta = fmaxf((1.f - var) / rho, 0.f);
      tau_star = mean - sqrtf(delta);
    }
    float z = 0.f;
    for (int i = 0; i < n; ++i) {
      const float x = (fabsf(s.hv[i * kRows + tid]) - zmax) * 0.5f;
      const float pv = fmaxf(x - tau_star, 0.f);
      z += pv * pv;
    }
    const float inv = z > 0.f ? 1.f / fmaxf(z, FLT_EPSILON) : 0.f;
    for (int i = 0; i < n; ++i) {
      const float x = s.hv[i * kRows + tid];
      const float sh = (fabsf(x) - zmax) * 0.5f;
      const float pv = fmaxf(sh - tau_star, 0.f);
      const float sg = x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
      s.hv[i * kRows + tid] = sg * pv * pv * inv;
    }
  }
}

template <typename T>
struct Vec8;  // 16-byte vector of T loaded and widened to float

template <>
struct Vec8<__nv_bfloat16> {
  static constexpr int kElems = 8;
  __device__ __forceinline__ static void load(const void* base, int64_t elem, float (&f)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + elem));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
};

template <>
struct Vec8<__half> {
  static constexpr int kElems = 8;
  __device__ __forceinline__ static void load(const void* base, int64_t elem, float (&f)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(base) + elem));
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
};

template <>
struct Vec8<float> {
  static constexpr int kElems = 8;
  __device__ __forceinline__ static void load(const void* base, int64_t elem, float (&f)[8]) {
    const float4* q = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + elem);
    const float4 a = __ldg(q), b = __ldg(q + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
};

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

// Gather-aggregate of one row by one warp: out[row] = sum_i w_i * val[idx_i].
template <typename VT>
__device__ void gather_row(const Smem& s, int col_tid, int n, int64_t b, int64_t row,
                           const Params& p, int lane) {
  const int64_t D = p.dim;
  const int64_t col_base = b * p.n_cols;
  float acc_state = 0.f;
  const bool vec = (D % 8) == 0;
  if (vec && D <= 1024) {
    const int nch = static_cast<int>(D / 8);
    float acc[4][8];
#pragma unroll
    for (int m = 0; m < 4; ++m)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[m][e] = 0.f;
    for (int i = 0; i < n; ++i) {
      const int j = s.hi[i * kRows + col_tid];
      float w = s.hv[i * kRows + col_tid];
      if (p.col_sender) w *= ld_elem(p.col_sender, col_base + j, p.state_dtype);
      if (lane == 0) acc_state += w * ld_elem(p.col_state, col_base + j, p.state_dtype);
      const int64_t rbase = (col_base + j) * D;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int c = lane + 32 * m;
        if (c < nch) {
          float f[8];
          Vec8<VT>::load(p.col_val, rbase + c * 8, f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[m][e] = fmaf(w, f[e], acc[m][e]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int c = lane + 32 * m;
      if (c < nch) store8(p.out_val, row * D + c * 8, p.out_dtype, acc[m]);
    }
  } else {
    // Generic path: any dim, one element per lane per step.
    for (int64_t d0 = 0; d0 < D; d0 += 32) {
      const int64_t d = d0 + lane;
      float acc = 0.f;
      for (int i = 0; i < n; ++i) {
        const int j = s.hi[i * kRows + col_tid];
        float w = s.hv[i * kRows + col_tid];
        if (p.col_sender) w *= ld_elem(p.col_sender, col_base + j, p.state_dtype);
        if (d0 == 0 && lane == 0) acc_state += w * ld_elem(p.col_state, col_base + j, p.state_dtype);
        if (d < D) acc = fmaf(w, ld_elem(p.col_val, (col_base + j) * D + d, p.val_dtype), acc);
      }
      if (d < D) st_elem(p.out_val, row * D + d, p.out_dtype, acc);
    }
  }
  if (lane == 0) st_elem(p.out_state, row, p.out_dtype, acc_state);
}

// Scatter of one source row by one warp into the f32 destination accumulators.
template <typename VT>
__device__ void scatter_row(const Smem& s, int col_tid, int n, int64_t b, int64_t src,
                            const Params& p, int lane) {
  // In scatter mode the "row side" is the source: state / value / sender are indexed by
  // the row, destinations are the selected columns.
  const int64_t D = p.dim;
  float sender = 1.f;
  if (p.col_sender) sender = ld_elem(p.col_sender, src, p.state_dtype);
  const float sstate = ld_elem(p.col_state, src, p.state_dtype);
  const bool vec = (D % 8) == 0 && D <= 1024;
  const int nch = static_cast<int>(D / 8);
  float v[4][8];
  if (vec) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int c = lane + 32 * m;
      if (c < nch) Vec8<VT>::load(p.col_val, src * D + c * 8, v[m]);
    }
  }
  for (int i = 0; i < n; ++i) {
    const int j = s.hi[i * kRows + col_tid];
    const float w = s.hv[i * kRows + col_tid] * sender;
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

template <int KMAX, int KATOMS, int STAGES, int MODE, typename VT>
__global__ void __launch_bounds__(kThreads, 1)
    topk_kernel(const __grid_constant__ CUtensorMap tm_rows, const __grid_constant__ CUtensorMap tm_cols,
                Params p, uint32_t idesc) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kAtomBytes = kRows * 128;  // 128 rows x 64 (16-bit) elements
  constexpr int kABytes = KATOMS * kAtomBytes;
  constexpr int kBBytes = KATOMS * kAtomBytes;
  uint8_t* a_tile = smem;
  uint8_t* b_ring = smem + kABytes;
  uint8_t* tail = b_ring + STAGES * kBBytes;
  Smem s;
  s.hv = reinterpret_cast<float*>(tail);
  s.hi = reinterpret_cast<int*>(s.hv + KMAX * kRows);
  s.qv = reinterpret_cast<float*>(s.hi + KMAX * kRows);
  s.qi = reinterpret_cast<int*>(s.qv + kQueue * kRows);
  s.aux = reinterpret_cast<float*>(s.qi + kQueue * kRows);
  s.nsel = reinterpret_cast<int*>(s.aux + KMAX * kRows);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s.nsel + kRows);
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
    int64_t hi = t0 + kRows - 1;
    if (hi > p.n_cols - 1) hi = p.n_cols - 1;
    j_hi = hi < 0 ? -1 : hi / kCols;
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
      mbar_init(&tempty[i], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ producer / MMA issuer
    if (lane == 0 && ntiles > 0) {
      prefetch_tmap(&tm_rows);
      prefetch_tmap(&tm_cols);
      bool ok = true;
      mbar_arrive_expect_tx(bar_a, kABytes);
#pragma unroll
      for (int a = 0; a < KATOMS; ++a)
        tma_load_3d(a_tile + a * kAtomBytes, &tm_rows, bar_a, a * 64, static_cast<int>(t0), static_cast<int>(b));
      const int pre = ntiles < STAGES ? ntiles : STAGES;
      for (int it = 0; it < pre; ++it) {
        mbar_arrive_expect_tx(&full[it], kBBytes);
        const int col0 = static_cast<int>((j_lo + it) * kCols);
#pragma unroll
        for (int a = 0; a < KATOMS; ++a)
          tma_load_3d(b_ring + it * kBBytes + a * kAtomBytes, &tm_cols, &full[it], a * 64, col0, static_cast<int>(b));
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
        const uint32_t b_addr = smem_u32(b_ring + st * kBBytes);
#pragma unroll
        for (int kk = 0; kk < 4 * KATOMS; ++kk) {
          const uint32_t off = (kk >> 2) * kAtomBytes + (kk & 3) * 32;
          mma_f16_ss(tmem + buf * kCols, sdesc_kmajor_sw128(a_addr + off), sdesc_kmajor_sw128(b_addr + off),
                     idesc, kk > 0 ? 1u : 0u);
        }
        mma_commit(&empty[st]);
        mma_commit(&tfull[buf]);
        const int ip = it - 1;
        if (ip >= 0 && ip + STAGES < ntiles) {
          const int sp = ip % STAGES;
          if (!mbar_wait(&empty[sp], (ip / STAGES) & 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[sp], kBBytes);
          const int col0 = static_cast<int>((j_lo + ip + STAGES) * kCols);
#pragma unroll
          for (int a = 0; a < KATOMS; ++a)
            tma_load_3d(b_ring + sp * kBBytes + a * kAtomBytes, &tm_cols, &full[sp], a * 64, col0, static_cast<int>(b));
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
    // ------------------------------------------------------------ epilogue warps
    const int tid = threadIdx.x;  // 0..127 == TMEM lane == row in tile
    const int64_t t = t0 + tid;
    const bool row_ok = t < p.n_rows;
    // Visible columns of this row: [lo_t, hi_t] (32-bit; sizes are capped at 2^30).
    int lo_t = 0, hi_t = static_cast<int>(p.n_cols - 1);
    if (p.window >= 0) {
      const int64_t lo = t - p.window;
      lo_t = lo < 0 ? 0 : static_cast<int>(lo);
      hi_t = t < hi_t ? static_cast<int>(t) : hi_t;
    }
    if (!row_ok || hi_t < lo_t) {
      // Nothing visible: an unreachable single-column range.
      lo_t = INT_MAX / 2;
      hi_t = INT_MAX / 2;
    }
    const uint32_t span = static_cast<uint32_t>(hi_t - lo_t);
    for (int i = 0; i < k; ++i) {
      s.hv[i * kRows + tid] = -INFINITY;
      s.hi[i * kRows + tid] = kSentinel;
    }
    float thr = -INFINITY;
    int qn = 0;
    bool ok = true;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    for (int it = 0; it < ntiles; ++it) {
      const int buf = it & 1;
      if (!mbar_wait(&tfull[buf], (it >> 1) & 1) || *abort_flag) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t v[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(tmem + lane_base + buf * kCols + c * 32, v[c]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      const int col0 = static_cast<int>((j_lo + it) * kCols);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int col = col0 + c * 32 + e + u;
            const float x = __uint_as_float(v[c][e + u]);
            const bool vis = static_cast<uint32_t>(col - lo_t) <= span;
            if (vis && x > thr) {
              s.qv[qn * kRows + tid] = x;
              s.qi[qn * kRows + tid] = col;
              ++qn;
            }
          }
          if (__any_sync(0xffffffffu, qn > kQueue - 4)) thr = flush_queue(s, tid, k, qn);
        }
      }
    }
    if (ok) {
      thr = flush_queue(s, tid, k, qn);
      heap_sort(s, tid, k);
      int n = 0;
      while (n < k && s.hi[n * kRows + tid] != kSentinel) ++n;
      // Scores (bias added after selection; constant per op so the selection is unchanged).
      const float bias = p.bias + (p.bias_dev ? __ldg(p.bias_dev) : 0.f);
      for (int i = 0; i < n; ++i) s.hv[i * kRows + tid] += bias;
      if (MODE == kGather && row_ok && (p.out_scores || p.out_index)) {
        const int64_t o = (b * p.n_rows + t) * k;
        for (int i = 0; i < k; ++i) {
          if (p.out_scores) p.out_scores[o + i] = i < n ? s.hv[i * kRows + tid] : -INFINITY;
          if (p.out_index) p.out_index[o + i] = i < n ? static_cast<int64_t>(s.hi[i * kRows + tid]) : -1;
        }
      }
      compress_row(s, tid, n, p.compress);
      s.nsel[tid] = row_ok ? n : 0;
    } else {
      s.nsel[tid] = 0;
      atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
      *abort_flag = 1;
    }
    __syncwarp();
    if (ok) {
      // Aggregate: warp w handles rows 32w .. 32w+31.
      for (int r = 0; r < 32; ++r) {
        const int rt = warp * 32 + r;
        const int64_t row = t0 + rt;
        if (row >= p.n_rows) break;
        const int n = s.nsel[rt];
        if (MODE == kGather) {
          gather_row<VT>(s, rt, n, b, b * p.n_rows + row, p, lane);
        } else {
          scatter_row<VT>(s, rt, n, b, b * p.n_rows + row, p, lane);
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

template <int KMAX, int KATOMS, int STAGES>
constexpr int smem_bytes() {
  return 1024 + (1 + STAGES) * KATOMS * kRows * 128 + (2 * KMAX + 2 * kQueue + KMAX) * kRows * 4 + kRows * 4 +
         256;
}

// Converts the f32 destination accumulators of the scatter mode into the outputs.
__global__ void finalize_scatter(const float* acc_state, const float* acc_val, int64_t n_state,
                                 int64_t n_val, void* out_state, void* out_val, int out_dtype) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t j = i; j < n_val; j += stride) st_elem(out_val, j, out_dtype, acc_val[j]);
  for (int64_t j = i; j < n_state; j += stride) st_elem(out_state, j, out_dtype, acc_state[j]);
}

template <int KMAX, int KATOMS, int MODE, typename VT>
int launch_vt(const CUtensorMap& tr, const CUtensorMap& tc, const Params& p, int64_t batch,
              uint32_t idesc, cudaStream_t st) {
  constexpr int STAGES = KATOMS == 1 ? 4 : 2;
  constexpr int sm = smem_bytes<KMAX, KATOMS, STAGES>();
  auto kern = topk_kernel<KMAX, KATOMS, STAGES, MODE, VT>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sm) != cudaSuccess)
    return launch_status() == JK_OK ? JK_ERR_LAUNCH : JK_ERR_LAUNCH;
  const dim3 grid(static_cast<unsigned>((p.n_rows + kRows - 1) / kRows), static_cast<unsigned>(batch));
  kern<<<grid, kThreads, sm, st>>>(tr, tc, p, idesc);
  return launch_status();
}

template <int KMAX, int KATOMS, int MODE>
int launch_k(const CUtensorMap& tr, const CUtensorMap& tc, const Params& p, int64_t batch,
             uint32_t idesc, cudaStream_t st) {
  switch (p.val_dtype) {
    case JK_F32: return launch_vt<KMAX, KATOMS, MODE, float>(tr, tc, p, batch, idesc, st);
    case JK_BF16: return launch_vt<KMAX, KATOMS, MODE, __nv_bfloat16>(tr, tc, p, batch, idesc, st);
    default: return launch_vt<KMAX, KATOMS, MODE, __half>(tr, tc, p, batch, idesc, st);
  }
}

template <int MODE>
int launch(const void* row_proj, const void* col_proj, int64_t batch, int64_t n_rows, int64_t n_cols,
           int64_t rp, int proj_dtype, Params& p, cudaStream_t st) {
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

int validate_common(const void* row_proj, const void* col_proj, int64_t batch, int64_t n_rows,
                    int64_t n_cols, int64_t rp, int proj_dtype, const void* state, int state_dtype,
                    const void* val, int64_t dim, int val_dtype, int64_t k, int compress, int out_dtype) {
  if (row_proj == nullptr || col_proj == nullptr || state == nullptr || val == nullptr) return JK_ERR_BAD_ARG;
  if (proj_dtype != JK_BF16 && proj_dtype != JK_F16) return JK_ERR_BAD_DTYPE;
  if (val_dtype < JK_F32 || val_dtype > JK_F16 || out_dtype < JK_F32 || out_dtype > JK_F16 ||
      state_dtype < JK_F32 || state_dtype > JK_F16)
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

extern "C" int jk_propagation_topk_forward(const void* row_proj, const void* col_proj, int64_t batch,
                                           int64_t n_rows, int64_t n_cols, int64_t rp, int proj_dtype,
                                           const void* col_state, const void* col_sender, int state_dtype,
                                           const void* col_val, int64_t dim, int val_dtype, int64_t k,
                                           int64_t window, float score_bias, const float* bias_dev, int compress,
                                           void* out_state, void* out_val, int out_dtype, float* out_scores,
                                           int64_t* out_index, jk_stream_t stream) {
  using namespace jk;
  int st = topk::validate_common(row_proj, col_proj, batch, n_rows, n_cols, rp, proj_dtype, col_state,
                                 state_dtype, col_val, dim, val_dtype, k, compress, out_dtype);
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
                                                const void* source_state, const void* source_sender,
                                                int state_dtype, const void* source_val, int64_t dim,
                                                int val_dtype, int64_t k, float score_bias,
                                                const float* bias_dev, int compress, void* out_state,
                                                void* out_val, int out_dtype, float* out_scores,
                                                int64_t* out_index, jk_stream_t stream) {
  return jk_propagation_topk_forward(query_proj, source_proj, batch, n_query, n_source, rp, proj_dtype,
                                     source_state, source_sender, state_dtype, source_val, dim, val_dtype, k,
                                     -1, score_bias, bias_dev, compress, out_state, out_val, out_dtype,
                                     out_scores, out_index, stream);
}

extern "C" int jk_transition_pairwise_topk_forward(const void* src_proj, const void* dst_proj, int64_t batch,
                                                   int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                                   const void* src_state, const void* src_sender,
                                                   int state_dtype, const void* src_val, int64_t dim,
                                                   int val_dtype, int64_t k, float score_bias,
                                                   const float* bias_dev, int compress, float* accum,
                                                   void* out_state, void* out_val, int out_dtype,
                                                   jk_stream_t stream) {
  using namespace jk;
  int st = topk::validate_common(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, src_state,
                                 state_dtype, src_val, dim, val_dtype, k, compress, out_dtype);
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
