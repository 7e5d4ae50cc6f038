// Fused window / dense propagation (no top-k):
//   score[t,s] = row_proj[t] . col_proj[s] + bias          (tcgen05, f32)
//   e[t,s]     = compress over the visible s of row t       (softsign | signed_abs_softmax
//                                                            | signed_entmax15)
//   out_val[t] = sum_s e[t,s] * col_val[s],  out_state[t] = sum_s e[t,s] * col_state[s]
// with visibility = causal window [t - window, t] (window >= 0) or every column (-1).
//
// Reference semantics: SparsePropagation(sparse_type="window") propagation.py:453-480
// (edges compressed over the visible sources, propagation.py:67-88), the dense Propagation
// propagation.py:207-220 and the query-dense op jakal_net_native.cpp:6078-6188; replaces
// the CUDA window kernels jakal_net_native_cuda.cu:1579-1750 (softsign / signed-abs) and
// :2023-2109 (entmax, O(W^2) serial sort there) and the dense kernels :1388-1576.
//
// Flash-style on tcgen05. One CTA = 128 target rows x one slice of <= 256 value columns
// (<= 128 when f32 values come as hi + lo planes).
//   warp 8: TMA of the target projection tile, source projection tiles (ring), value tiles
//           (ring, MN-major 128B-swizzled boxes); tcgen05.mma S = Pt . Ps^T into two TMEM
//           score buffers, and in the final pass O += E . V into a TMEM accumulator.
//   warps 0-7: two threads per row, 64 source columns each. Normalising compressors first
//           run statistics passes over the score tiles (recomputed, never stored):
//           signed_abs_softmax -> row max|s| and sum exp(|s| - max); signed_entmax15 -> row
//           max|s|, then the fixed-point iteration of the threshold tau (support =
//           {z > tau}, z = (|s| - max) / 2, tau from the closed form over the support) until
//           the support stops changing. The final pass turns every score tile into exact
//           normalised f32 edges, splits them into bf16 (or f16) hi + lo halves, writes the
//           two edge tiles into shared memory in the tcgen05 K-major layout and hands them
//           to warp 8, which multiplies them with the value tile. The hi + lo split keeps
//           the edge weights at ~16 significant bits, so the aggregate matches an f32
//           gather to ~1e-5 relative.
#include "jk_host.h"
#include "jk_sm100.cuh"

#include <cfloat>

namespace jk {
namespace win {

constexpr int kRows = 128;
constexpr int kCols = 128;
constexpr int kHalfCols = 64;
constexpr int kSelWarps = 8;
constexpr int kThreads = (kSelWarps + 1) * 32;
constexpr int kMaxSlice = 256;   // value columns per CTA (TMEM: 2 x 128 score + 256 output columns)
constexpr int kMaxEntIters = 48;  // cap on threshold iterations (converges in a few)
constexpr int kStageCols = 1024;  // source states staged in shared memory when the CTA's columns fit

enum PassType { kDone = 0, kStatsMax = 1, kStatsEnt = 2, kFinal = 3 };

struct Params {
  int64_t n_rows, n_cols, dim;
  int64_t window;
  float bias;
  const float* bias_dev;
  int compress;
  int state_dtype, out_dtype, f16;
  const void* col_state;
  void* out_state;
  void* out_val;
  int split3;      // projections are the three-plane bf16 split of f32 values
  int vsplit;      // values come as bf16 hi / lo planes (f32 values)
  int d0;          // first value column of this launch's slice
  int slice_cols;  // value columns of the slice (multiple of 64, <= kMaxSlice)
  // Statistics mode (stats_out != null): only the normalising passes run; every row writes
  // (max, row_scale[row] / normaliser, entmax tau) as 3 floats and nothing is aggregated.
  float* stats_out;
  const void* row_scale;  // state dtype; null = 1
  // Column-statistics mode (col_stats != null): a single final pass whose edges are
  // normalised per COLUMN with the (max, scale / normaliser, tau) triples a statistics-mode
  // launch wrote for the columns (the transposed route normalisation of a transition).
  const float* col_stats;
  // multi-head scorer (heads == 2): one 256-column score buffer holding both head planes,
  // combined as they are read (JK_HEADS_*); heads == 1 keeps two 128-column buffers
  int heads, kph, combine;
  const float* head_bias;
  // Failure-path test only (jk_debug_window_stalled_producer): the producer warp issues no
  // load and no MMA, so every consumer wait runs into its bound and the kernel unwinds.
  int debug_stall;
};

// One edge from a score and the (max, scale / normaliser, tau) of its normalisation set.
__device__ __forceinline__ float edge_of(float s, int compress, float m, float inv, float tau) {
  if (compress == JK_SOFTSIGN) return s / (1.f + fabsf(s));
  if (compress == JK_SOFTMAX) return expf(s - m) * inv;
  const float sg = s > 0.f ? 1.f : (s < 0.f ? -1.f : 0.f);
  if (compress == JK_SIGNED_ABS_SOFTMAX) return sg * expf(fabsf(s) - m) * inv;
  const float pz = fmaxf((fabsf(s) - m) * 0.5f - tau, 0.f);
  return sg * pz * pz * inv;
}

template <int KATOMS>
struct Layout {
  static constexpr int kAtom = kRows * 128;  // 16 KB: 128 rows x 128 B
  static constexpr int kPsStages = KATOMS == 1 ? 2 : 1;
  // one value stage: the edge tiles are single-buffered, so the next value tile is only
  // needed once the edges of its source tile exist, which takes longer than its load
  static constexpr int kVStages = 1;
  static constexpr int kA = KATOMS * kAtom;
  static constexpr int kPs = kPsStages * KATOMS * kAtom;
  static constexpr int kE = 2 * 2 * kAtom;                        // hi + lo, 2 K atoms each
  static constexpr int kVStage = (kMaxSlice / 64) * kAtom;         // 4 boxes of 64 columns
  static constexpr int kV = kVStages * kVStage;
  static constexpr int kRowArrays = 16 * kRows * 4;
  static constexpr int kStage = kStageCols * 4;  // the CTA's source states, f32
  static constexpr int kTotal = 1024 + kA + kPs + kE + kV + kRowArrays + 512 + kStage;
};

__device__ __forceinline__ void sel_barrier() {
  asm volatile("bar.sync 1, %0;" ::"r"(kSelWarps * 32) : "memory");
}

// Packs 8 f32 edges into 8 16-bit hi parts and 8 lo parts (e - hi).
__device__ __forceinline__ void split8(const float (&e)[8], bool f16, uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (f16) {
      const __half2 a = __floats2half2_rn(e[2 * i], e[2 * i + 1]);
      const float2 af = __half22float2(a);
      const __half2 b = __floats2half2_rn(e[2 * i] - af.x, e[2 * i + 1] - af.y);
      h[i] = *reinterpret_cast<const uint32_t*>(&a);
      l[i] = *reinterpret_cast<const uint32_t*>(&b);
    } else {
      const __nv_bfloat162 a = __floats2bfloat162_rn(e[2 * i], e[2 * i + 1]);
      const float2 af = __bfloat1622float2(a);
      const __nv_bfloat162 b = __floats2bfloat162_rn(e[2 * i] - af.x, e[2 * i + 1] - af.y);
      h[i] = *reinterpret_cast<const uint32_t*>(&a);
      l[i] = *reinterpret_cast<const uint32_t*>(&b);
    }
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

template <int KATOMS>
__global__ void __launch_bounds__(kThreads, 1)
    window_kernel(const __grid_constant__ CUtensorMap tm_rows, const __grid_constant__ CUtensorMap tm_cols,
                  const __grid_constant__ CUtensorMap tm_val, const __grid_constant__ CUtensorMap tm_val_lo, Params p,
                  uint32_t idesc_s, uint32_t idesc_pv) {
  using L = Layout<KATOMS>;
  constexpr int PS = L::kPsStages;
  constexpr int VS = L::kVStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tile = smem;
  uint8_t* ps_ring = a_tile + L::kA;
  uint8_t* e_hi = ps_ring + L::kPs;        // 2 atoms (K 0-63, K 64-127)
  uint8_t* e_lo = e_hi + 2 * L::kAtom;
  uint8_t* v_ring = e_hi + L::kE;
  float* arr = reinterpret_cast<float*>(v_ring + L::kV);
  float* pm = arr;                 // [2][kRows] partial max / count
  float* pz = pm + 2 * kRows;      // [2][kRows] partial sum exp / sum z
  float* ps2 = pz + 2 * kRows;     // [2][kRows] partial sum z^2
  float* pst = ps2 + 2 * kRows;    // [2][kRows] partial state
  float* rmax = pst + 2 * kRows;   // [kRows] row max |s|
  float* rnorm = rmax + kRows;     // [kRows] row normaliser
  float* rtau = rnorm + kRows;     // [kRows] entmax threshold (z units)
  int* rcount = reinterpret_cast<int*>(rtau + kRows);  // [kRows] support size
  int* rconv = rcount + kRows;                         // [kRows] converged flag
  volatile int* next_pass = rconv + kRows;
  volatile int* abort_flag = next_pass + 1;
  volatile int* vote = abort_flag + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(const_cast<int*>(vote) + 1);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(arr) + 16 * kRows * 4 + 64);
  float* st_stage = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(arr) + 16 * kRows * 4 + 512);
  uint64_t* bar_a = bars;
  uint64_t* decide = bars + 1;
  uint64_t* eready = bars + 2;
  uint64_t* efree = bars + 3;
  uint64_t* obar = bars + 4;
  uint64_t* full = bars + 5;       // [PS]
  uint64_t* empty = full + PS;     // [PS]
  uint64_t* vfull = empty + PS;    // [VS]
  uint64_t* vempty = vfull + VS;   // [VS]
  uint64_t* tfull = vempty + VS;   // [2]
  uint64_t* tempty = tfull + 2;    // [2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t b = blockIdx.y;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kRows;
  const int d0 = p.d0;
  const int dc = p.slice_cols;
  const int nbox = dc / 64;

  int64_t j_lo = 0, j_hi = (p.n_cols + kCols - 1) / kCols - 1;
  if (p.window >= 0) {
    const int64_t lo = t0 - p.window;
    j_lo = lo > 0 ? lo / kCols : 0;
    int64_t hc = t0 + kRows - 1;
    if (hc > p.n_cols - 1) hc = p.n_cols - 1;
    j_hi = hc < 0 ? -1 : hc / kCols;
  }
  const int ntiles = j_hi >= j_lo ? static_cast<int>(j_hi - j_lo + 1) : 0;

  if (threadIdx.x == 0) {
    mbar_init(bar_a, 1);
    mbar_init(decide, 1);
    mbar_init(eready, kSelWarps);
    mbar_init(efree, 1);
    mbar_init(obar, 1);
    for (int i = 0; i < PS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < VS; ++i) {
      mbar_init(&vfull[i], 1);
      mbar_init(&vempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kSelWarps);
    }
    *abort_flag = 0;
    *next_pass = kDone;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_o = tmem + 256;

  if (warp == kSelWarps) {
    // ------------------------------------------------------------ producer / MMA issuer
    if (lane == 0 && ntiles > 0 && !p.debug_stall) {
      prefetch_tmap(&tm_rows);
      prefetch_tmap(&tm_cols);
      prefetch_tmap(&tm_val);
      bool ok = true;
      mbar_arrive_expect_tx(bar_a, L::kA);
      for (int a = 0; a < KATOMS; ++a)
        tma_load_3d(a_tile + a * L::kAtom, &tm_rows, bar_a, a * 64, static_cast<int>(t0), static_cast<int>(b));
      int g = 0;       // score tiles issued (all passes)
      int total = 0;   // score-tile loads planned
      int issued = 0;  // score-tile loads issued
      auto issue_ps = [&](int upto) -> bool {
        while (issued <= upto && issued < total) {
          const int s = issued % PS;
          if (issued >= PS && !mbar_wait(&empty[s], ((issued - PS) / PS) & 1)) return false;
          mbar_arrive_expect_tx(&full[s], KATOMS * L::kAtom);
          const int col0 = static_cast<int>((j_lo + issued % ntiles) * kCols);
          for (int a = 0; a < KATOMS; ++a)
            tma_load_3d(ps_ring + s * KATOMS * L::kAtom + a * L::kAtom, &tm_cols, &full[s], a * 64, col0,
                        static_cast<int>(b));
          ++issued;
        }
        return true;
      };
      const int nb = p.heads > 1 ? 1 : 2;  // TMEM score buffers
      auto issue_s = [&]() -> bool {  // score MMA of global tile g
        const int st = g % PS;
        const int buf = g % nb;
        if (!mbar_wait(&full[st], (g / PS) & 1)) return false;
        if (g >= nb && !mbar_wait(&tempty[buf], ((g / nb) - 1) & 1)) return false;
        if (*abort_flag) return false;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(a_tile);
        const uint32_t b_addr = smem_u32(ps_ring + st * KATOMS * L::kAtom);
        if (p.heads > 1)
          head_score_mmas(tmem, kCols, a_addr, b_addr, idesc_s, p.heads, p.kph);
        else
          score_mmas<KATOMS>(tmem + buf * kCols, a_addr, b_addr, idesc_s, p.split3 != 0);
        mma_commit(&empty[st]);
        mma_commit(&tfull[buf]);
        ++g;
        return issue_ps(PS == 1 ? g : g - 2 + PS);
      };
      auto issue_v = [&](int it) {  // value tile `it` of the final pass into stage it % VS
        const int s = it % VS;
        const int col0 = static_cast<int>((j_lo + it) * kCols);
        if (p.vsplit) {  // <= 128 columns: the hi plane boxes, then the lo plane boxes from atom 2
          mbar_arrive_expect_tx(&vfull[s], 2 * nbox * L::kAtom);
          for (int a = 0; a < nbox; ++a) {
            tma_load_3d(v_ring + s * L::kVStage + a * L::kAtom, &tm_val, &vfull[s], d0 + a * 64, col0,
                        static_cast<int>(b));
            tma_load_3d(v_ring + s * L::kVStage + (2 + a) * L::kAtom, &tm_val_lo, &vfull[s], d0 + a * 64, col0,
                        static_cast<int>(b));
          }
        } else {
          mbar_arrive_expect_tx(&vfull[s], nbox * L::kAtom);
          for (int a = 0; a < nbox; ++a)
            tma_load_3d(v_ring + s * L::kVStage + a * L::kAtom, &tm_val, &vfull[s], d0 + a * 64, col0,
                        static_cast<int>(b));
        }
      };
      ok = mbar_wait(bar_a, 0);
      int dp = 0;
      while (ok) {
        if (!mbar_wait(decide, dp & 1)) { ok = false; break; }
        ++dp;
        const int type = *next_pass;
        if (type == kDone) break;
        total += ntiles;
        if (!issue_ps(g - 1 + PS)) { ok = false; break; }
        if (type != kFinal) {
          for (int it = 0; it < ntiles && ok; ++it) ok = issue_s();
          continue;
        }
        for (int it = 0; it < VS && it < ntiles; ++it) issue_v(it);
        ok = issue_s();
        for (int it = 0; it < ntiles && ok; ++it) {
          if (it + 1 < ntiles && !(ok = issue_s())) break;
          const int vs = it % VS;
          if (!mbar_wait(&vfull[vs], (it / VS) & 1) || !mbar_wait(eready, it & 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(v_ring + vs * L::kVStage);
          // E_hi.V + E_lo.V (+ E_hi.V_lo for split f32 values)
          const int nprod = p.vsplit ? 3 : 2;
          for (int q = 0; q < nprod; ++q) {
            const uint32_t e_addr = smem_u32(q == 1 ? e_lo : e_hi);
            const uint32_t vb = v_addr + (q == 2 ? 2u * L::kAtom : 0u);
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t aoff = (kk >> 2) * L::kAtom + (kk & 3) * 32;
              mma_f16_ss(tmem_o, sdesc_kmajor_sw128(e_addr + aoff), sdesc_mnmajor_sw128(vb + kk * 2048, L::kAtom),
                         idesc_pv, (it > 0 || q > 0 || kk > 0) ? 1u : 0u);
            }
          }
          mma_commit(efree);
          mma_commit(&vempty[vs]);
          if (it + VS < ntiles) {
            if (!mbar_wait(&vempty[vs], (it / VS) & 1)) { ok = false; break; }
            issue_v(it + VS);
          }
        }
        if (ok) mma_commit(obar);
        break;
      }
      if (ok && g > 0) ok = mbar_wait(&empty[(g - 1) % PS], ((g - 1) / PS) & 1);
      if (!ok) {
        atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
        *abort_flag = 1;
      }
    }
  } else {
    // ------------------------------------------------------------ edge warps
    const int quad = warp & 3;
    const int half = warp >> 2;
    const int row = quad * 32 + lane;
    const int64_t t = t0 + row;
    const bool row_ok = t < p.n_rows;
    int lo_t = 0, hi_t = static_cast<int>(p.n_cols - 1);
    if (p.window >= 0) {
      const int64_t lo = t - p.window;
      lo_t = lo < 0 ? 0 : static_cast<int>(lo);
      hi_t = t < hi_t ? static_cast<int>(t) : hi_t;
    }
    if (!row_ok || hi_t < lo_t) {
      lo_t = 0x3FFFFFFF;
      hi_t = 0x3FFFFFFF;
    }
    const uint32_t span = static_cast<uint32_t>(hi_t - lo_t);
    const uint32_t tbase = (static_cast<uint32_t>(quad * 32) << 16) + half * kHalfCols;
    const float bias = p.bias + (p.bias_dev ? __ldg(p.bias_dev) : 0.f);
    const int64_t cb = b * p.n_cols;
    int g = 0;
    bool ok = true;

    // The CTA's source states, staged once (f32, coalesced) when its columns fit: the final
    // pass's state sum then reads shared memory instead of one global load per edge. The
    // condition is the same in every thread of the CTA, so every edge warp reaches the barrier.
    const int c_lo = static_cast<int>(j_lo * kCols);
    int n_stage = 0;
    if (ntiles > 0 && p.stats_out == nullptr) {
      int64_t c_hi = (j_hi + 1) * kCols;
      if (c_hi > p.n_cols) c_hi = p.n_cols;
      const int64_t cnt = c_hi - c_lo;
      if (cnt > 0 && cnt <= kStageCols) {
        n_stage = static_cast<int>(cnt);
        for (int i = threadIdx.x; i < n_stage; i += kSelWarps * 32)
          st_stage[i] = ld_elem(p.col_state, cb + c_lo + i, p.state_dtype);
        sel_barrier();
      }
    }

    const int nbuf = p.heads > 1 ? 1 : 2;
    auto load_tile = [&](float (&x)[64]) -> bool {
      const int buf = g % nbuf;
      if (!mbar_wait(&tfull[buf], (g / nbuf) & 1) || *abort_flag) return false;
      tc_fence_after();
      uint32_t v[2][32];
      if (p.heads > 1) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float f[16];
          combine_heads16<2>(tmem + tbase + c * 16, kCols, p.head_bias, p.combine, f);
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
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int e = 0; e < 32; ++e) x[c * 32 + e] = __uint_as_float(v[c][e]) + bias;
      return true;
    };

    // First pass.
    const bool stats_mode = p.stats_out != nullptr;
    const bool col_mode = p.col_stats != nullptr;
    const bool plain = p.compress == JK_SOFTMAX;  // normalised over s, not |s|
    int pass = (p.compress == JK_SOFTSIGN || col_mode) ? kFinal : kStatsMax;
    if (threadIdx.x == 0) {
      *next_pass = ntiles > 0 ? pass : kDone;
      mbar_arrive(decide);
    }
    if (ntiles == 0) pass = kDone;
    int iters = 0;
    while (ok && pass != kFinal && pass != kDone) {
      if (pass == kStatsMax) {
        float m = -INFINITY, z = 0.f;
        for (int it = 0; it < ntiles && ok; ++it) {
          float x[64];
          if (!load_tile(x)) { ok = false; break; }
          const int col0 = static_cast<int>((j_lo + it) * kCols) + half * kHalfCols;
          float tm = m;
#pragma unroll
          for (int e = 0; e < 64; ++e)
            if (static_cast<uint32_t>(col0 + e - lo_t) <= span) tm = fmaxf(tm, plain ? x[e] : fabsf(x[e]));
          if ((p.compress == JK_SIGNED_ABS_SOFTMAX || plain) && tm > -INFINITY) {
            z = (m > -INFINITY) ? z * expf(m - tm) : 0.f;
#pragma unroll
            for (int e = 0; e < 64; ++e)
              if (static_cast<uint32_t>(col0 + e - lo_t) <= span) z += expf((plain ? x[e] : fabsf(x[e])) - tm);
          }
          m = tm;
        }
        pm[half * kRows + row] = m;
        pz[half * kRows + row] = z;
        sel_barrier();
        if (half == 0) {
          const float m0 = pm[row], m1 = pm[kRows + row];
          const float mm = fmaxf(m0, m1);
          float zz = 0.f;
          if (mm > -INFINITY) {
            if (m0 > -INFINITY) zz += pz[row] * expf(m0 - mm);
            if (m1 > -INFINITY) zz += pz[kRows + row] * expf(m1 - mm);
          }
          rmax[row] = mm;
          rnorm[row] = zz;
          rtau[row] = -1.f;  // entmax: the support lies in z > -1
          rcount[row] = 0x7FFFFFFF;
          rconv[row] = 0;
        }
        pass = (p.compress == JK_SIGNED_ABS_SOFTMAX || plain) ? kFinal : kStatsEnt;
      } else {  // kStatsEnt: support statistics for z > tau
        const float mrow = rmax[row], tau = rtau[row];
        float c = 0.f, s1 = 0.f, s2 = 0.f;
        for (int it = 0; it < ntiles && ok; ++it) {
          float x[64];
          if (!load_tile(x)) { ok = false; break; }
          const int col0 = static_cast<int>((j_lo + it) * kCols) + half * kHalfCols;
#pragma unroll
          for (int e = 0; e < 64; ++e) {
            const float zv = (fabsf(x[e]) - mrow) * 0.5f;
            if (static_cast<uint32_t>(col0 + e - lo_t) <= span && zv > tau) {
              c += 1.f;
              s1 += zv;
              s2 = fmaf(zv, zv, s2);
            }
          }
        }
        pm[half * kRows + row] = c;
        pz[half * kRows + row] = s1;
        ps2[half * kRows + row] = s2;
        sel_barrier();
        if (half == 0) {
          const float cnt = pm[row] + pm[kRows + row];
          const float a1 = pz[row] + pz[kRows + row];
          const float a2 = ps2[row] + ps2[kRows + row];
          const int ci = static_cast<int>(cnt);
          float tau_new = rtau[row];
          if (ci > 0) {
            const float mean = a1 / cnt;
            const float mean_sq = a2 / cnt;
            const float delta = fmaxf((1.f - cnt * (mean_sq - mean * mean)) / cnt, 0.f);
            tau_new = mean - sqrtf(delta);
          }
          rconv[row] = (ci == rcount[row] || ci == 0) ? 1 : 0;
          rcount[row] = ci;
          rtau[row] = tau_new;
          // sum over the support of (z - tau)^2 (the reference renormalises by this sum)
          rnorm[row] = a2 - 2.f * tau_new * a1 + cnt * tau_new * tau_new;
        }
        ++iters;
        pass = kStatsEnt;
      }
      sel_barrier();
      if (pass == kStatsEnt) {
        // Another threshold iteration while any row's support still changes.
        if (threadIdx.x == 0) *vote = 0;
        sel_barrier();
        if (half == 0 && row_ok && !rconv[row]) *vote = 1;
        sel_barrier();
        if (!*vote || iters >= kMaxEntIters) pass = kFinal;
      }
      if (threadIdx.x == 0) {
        // a statistics-mode launch ends where the final pass would start
        *next_pass = (ok && !*abort_flag && !(stats_mode && pass == kFinal)) ? pass : kDone;
        mbar_arrive(decide);
      }
      if (*abort_flag) ok = false;
    }
    if (stats_mode) {
      if (ok && pass == kFinal && half == 0 && row_ok) {
        const float norm = rnorm[row];
        const float inv = (p.compress == JK_SIGNED_ENTMAX15) ? (norm > 0.f ? 1.f / fmaxf(norm, FLT_EPSILON) : 0.f)
                                                              : (norm > 0.f ? 1.f / norm : 0.f);
        const float scale = p.row_scale ? ld_elem(p.row_scale, b * p.n_rows + t, p.state_dtype) : 1.f;
        float* o = p.stats_out + (b * p.n_rows + t) * 3;
        o[0] = rmax[row];
        o[1] = inv * scale;
        o[2] = rtau[row];
      }
      pass = kDone;
    }

    // Final pass: exact edges -> hi / lo edge tiles -> producer multiplies with the values.
    float state_acc = 0.f;
    if (ok && pass == kFinal) {
      const float mrow = rmax[row], norm = rnorm[row], tau = rtau[row];
      const float inv = (p.compress == JK_SIGNED_ENTMAX15) ? (norm > 0.f ? 1.f / fmaxf(norm, FLT_EPSILON) : 0.f)
                                                            : (norm > 0.f ? 1.f / norm : 0.f);
      const bool f16 = p.f16 != 0;
      uint8_t* rowp_hi = e_hi + half * L::kAtom + (row >> 3) * 1024 + (row & 7) * 128;
      uint8_t* rowp_lo = e_lo + half * L::kAtom + (row >> 3) * 1024 + (row & 7) * 128;
      for (int it = 0; it < ntiles; ++it) {
        float x[64];
        if (!load_tile(x)) { ok = false; break; }
        const int col0 = static_cast<int>((j_lo + it) * kCols) + half * kHalfCols;
        float ev[64];
        if (col_mode) {
          // per-column normalisation: the column's triple (broadcast loads, L1-resident)
#pragma unroll 8
          for (int e = 0; e < 64; ++e) {
            const int col = col0 + e;
            const float* cs = p.col_stats + (cb + (col < p.n_cols ? col : 0)) * 3;
            const float w = edge_of(x[e], p.compress, __ldg(cs), __ldg(cs + 1), __ldg(cs + 2));
            ev[e] = static_cast<uint32_t>(col - lo_t) <= span ? w : 0.f;
          }
        } else if (p.compress == JK_SOFTSIGN) {  // one loop per compressor: a tight hot loop
#pragma unroll
          for (int e = 0; e < 64; ++e) {
            const float w = x[e] / (1.f + fabsf(x[e]));
            ev[e] = static_cast<uint32_t>(col0 + e - lo_t) <= span ? w : 0.f;
          }
        } else if (p.compress == JK_SIGNED_ABS_SOFTMAX) {
#pragma unroll
          for (int e = 0; e < 64; ++e) {
            const float sg = x[e] > 0.f ? 1.f : (x[e] < 0.f ? -1.f : 0.f);
            const float w = sg * expf(fabsf(x[e]) - mrow) * inv;
            ev[e] = static_cast<uint32_t>(col0 + e - lo_t) <= span ? w : 0.f;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 64; ++e) {
            const float w = edge_of(x[e], p.compress, mrow, inv, tau);
            ev[e] = static_cast<uint32_t>(col0 + e - lo_t) <= span ? w : 0.f;
          }
        }
        // state: sum_s e * state[s] over this thread's visible columns
        if (n_stage > 0) {
          const float* sv = st_stage + (col0 - c_lo);  // col0 - c_lo + 64 <= n_stage or masked
#pragma unroll
          for (int e = 0; e < 64; ++e) {
            const bool in = col0 + e - c_lo < n_stage;
            state_acc = fmaf(ev[e], in ? sv[in ? e : 0] : 0.f, state_acc);
          }
        } else {
          for (int e0 = 0; e0 < 64; e0 += 8) {
            float sv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int col = col0 + e0 + u;
              sv[u] = (ev[e0 + u] != 0.f && col < p.n_cols) ? ld_elem(p.col_state, cb + col, p.state_dtype) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) state_acc = fmaf(ev[e0 + u], sv[u], state_acc);
          }
        }
        if (it > 0 && !mbar_wait(efree, (it - 1) & 1)) { ok = false; break; }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float e8[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) e8[u] = ev[c * 8 + u];
          uint4 hi, lo;
          split8(e8, f16, hi, lo);
          const int pos = (c ^ (row & 7)) * 16;
          *reinterpret_cast<uint4*>(rowp_hi + pos) = hi;
          *reinterpret_cast<uint4*>(rowp_lo + pos) = lo;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(eready);
      }
      if (!ok) {
        atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
        *abort_flag = 1;
      }
    }
    // Epilogue: O from TMEM, state from the two halves (not in statistics mode).
    if (!stats_mode) {
      pst[half * kRows + row] = state_acc;
      const bool have_o = ok && pass == kFinal && !*abort_flag;
      bool got_o = false;
      if (have_o) got_o = mbar_wait(obar, 0);
      if (have_o && !got_o) {
        atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
        *abort_flag = 1;
      }
      sel_barrier();
      if (half == 0 && row_ok && d0 == 0) {
        st_elem(p.out_state, b * p.n_rows + t, p.out_dtype, pst[row] + pst[kRows + row]);
      }
      tc_fence_after();
      const int hcols = dc / 2;  // multiple of 32
      for (int c0 = 0; c0 < hcols; c0 += 32) {
        uint32_t v[32];
        if (got_o) {
          tmem_ld_32x32b_x32(tmem_o + (static_cast<uint32_t>(quad * 32) << 16) + half * hcols + c0, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = 0u;
        }
        if (row_ok) {
          const int64_t base = (b * p.n_rows + t) * p.dim + d0 + half * hcols + c0;
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
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int KATOMS>
int launch(const void* row_proj, const void* col_proj, const void* col_val, const void* col_val_lo, int64_t batch,
           int64_t n_rows, int64_t n_cols, int64_t rp, bool bf16, Params& p, cudaStream_t st) {
  CUtensorMap tr, tc, tv, tvl;
  int status = make_tmap_3d_16bit(&tr, row_proj, rp, n_rows, batch, 64, kRows, bf16);
  if (status != JK_OK) return status;
  status = make_tmap_3d_16bit(&tc, col_proj, rp, n_cols, batch, 64, kCols, bf16);
  if (status != JK_OK) return status;
  tv = tc;  // statistics mode reads no values
  if (col_val != nullptr) {
    status = make_tmap_3d_16bit(&tv, col_val, p.dim, n_cols, batch, 64, kCols, bf16);
    if (status != JK_OK) return status;
  }
  tvl = tv;
  if (p.vsplit) {
    status = make_tmap_3d_16bit(&tvl, col_val_lo, p.dim, n_cols, batch, 64, kCols, bf16);
    if (status != JK_OK) return status;
  }
  const int nslice = static_cast<int>((p.dim + kMaxSlice - 1) / kMaxSlice);
  const int nslice_split = static_cast<int>((p.dim + 127) / 128);  // hi + lo planes: <= 128 columns
  const int per = p.vsplit ? static_cast<int>(((p.dim / 64 + nslice_split - 1) / nslice_split) * 64)
                           : static_cast<int>(((p.dim / 64 + nslice - 1) / nslice) * 64);
  const uint32_t fmt = bf16 ? 1u : 0u;
  const uint32_t idesc_s = idesc_f16(kRows, kCols, fmt);
  constexpr int sm = Layout<KATOMS>::kTotal;
  static_assert(sm <= 232448, "shared memory budget");
  auto kern = window_kernel<KATOMS>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sm) != cudaSuccess) {
    cudaGetLastError();
    return JK_ERR_LAUNCH;
  }
  // One launch per value-column slice (the value MMA's N is the slice width; the last
  // slice may be narrower). Every slice recomputes the scores and edges.
  const dim3 grid(static_cast<unsigned>((n_rows + kRows - 1) / kRows), static_cast<unsigned>(batch), 1);
  if (p.stats_out != nullptr) {  // one launch: the statistics do not depend on the values
    Params q = p;
    q.d0 = 0;
    q.slice_cols = 64;
    kern<<<grid, kThreads, sm, st>>>(tr, tc, tv, tvl, q, idesc_s, idesc_f16(kRows, 64, fmt) | (1u << 16));
    return launch_status();
  }
  for (int d0 = 0; d0 < p.dim; d0 += per) {
    const int width = static_cast<int>(p.dim - d0 < per ? p.dim - d0 : per);
    Params q = p;
    q.d0 = d0;
    q.slice_cols = width;
    const uint32_t idesc_pv = idesc_f16(kRows, width, fmt) | (1u << 16);  // B (values) MN-major
    kern<<<grid, kThreads, sm, st>>>(tr, tc, tv, tvl, q, idesc_s, idesc_pv);
    const int status2 = launch_status();
    if (status2 != JK_OK) return status2;
  }
  return JK_OK;
}

}  // namespace win
}  // namespace jk

namespace jk {
namespace win {

// Checks shared by the window entry points; fills the common Params.
int prepare(const void* row_proj, const void* col_proj, int64_t batch, int64_t n_rows, int64_t n_cols, int64_t rp,
            int proj_dtype, const void* col_state, int state_dtype, const void* col_val, const void* col_val_lo,
            int64_t dim, float score_bias, const float* bias_dev, int compress, void* out_state, void* out_val,
            int out_dtype, const jk_heads_t* heads, Params& p) {
  if (row_proj == nullptr || col_proj == nullptr || col_state == nullptr || col_val == nullptr ||
      out_state == nullptr || out_val == nullptr)
    return JK_ERR_BAD_ARG;
  if (proj_dtype != JK_BF16 && proj_dtype != JK_F16 && proj_dtype != JK_BF16X3) return JK_ERR_BAD_DTYPE;
  if (proj_dtype == JK_BF16X3 && rp != 128) return JK_ERR_BAD_SHAPE;
  if (col_val_lo != nullptr && proj_dtype == JK_F16) return JK_ERR_BAD_DTYPE;
  if (state_dtype < JK_F32 || state_dtype > JK_F16 || out_dtype < JK_F32 || out_dtype > JK_F16) return JK_ERR_BAD_DTYPE;
  if (batch <= 0 || n_rows <= 0 || n_cols <= 0 || dim <= 0 || dim % 64 != 0) return JK_ERR_BAD_SHAPE;
  if (batch > 65535 || n_rows > (int64_t(1) << 30) || n_cols > (int64_t(1) << 30)) return JK_ERR_BAD_SHAPE;
  if (rp != 64 && rp != 128) return JK_ERR_BAD_SHAPE;
  if (!aligned16(row_proj) || !aligned16(col_proj) || !aligned16(col_val) || !aligned16(out_val) ||
      (col_val_lo != nullptr && !aligned16(col_val_lo)))
    return JK_ERR_ALIGNMENT;
  Heads hd;
  const int hs = read_heads(heads, rp, proj_dtype, 2, hd);
  if (hs != JK_OK) return hs;
  p = Params{};
  p.heads = hd.heads;
  p.kph = hd.kph;
  p.combine = hd.combine;
  p.head_bias = hd.bias;
  p.n_rows = n_rows;
  p.n_cols = n_cols;
  p.dim = dim;
  p.window = -1;
  p.bias = score_bias;
  p.bias_dev = bias_dev;
  p.compress = compress;
  p.state_dtype = state_dtype;
  p.out_dtype = out_dtype;
  p.f16 = proj_dtype == JK_F16 ? 1 : 0;
  p.split3 = proj_dtype == JK_BF16X3 ? 1 : 0;
  p.vsplit = col_val_lo != nullptr ? 1 : 0;
  p.col_state = col_state;
  p.out_state = out_state;
  p.out_val = out_val;
  return check_device();
}

int run(const void* row_proj, const void* col_proj, const void* col_val, const void* col_val_lo, int64_t batch,
        int64_t n_rows, int64_t n_cols, int64_t rp, int proj_dtype, Params& p, jk_stream_t stream) {
  auto cs = reinterpret_cast<cudaStream_t>(stream);
  const bool bf16 = proj_dtype != JK_F16;
  if (rp == 64) return launch<1>(row_proj, col_proj, col_val, col_val_lo, batch, n_rows, n_cols, rp, bf16, p, cs);
  return launch<2>(row_proj, col_proj, col_val, col_val_lo, batch, n_rows, n_cols, rp, bf16, p, cs);
}

}  // namespace win
}  // namespace jk

namespace jk {
namespace win {

int window_forward(const void* row_proj, const void* col_proj, int64_t batch, int64_t n_rows, int64_t n_cols,
                   int64_t rp, int proj_dtype, const void* col_state, int state_dtype, const void* col_val,
                   const void* col_val_lo, int64_t dim, int64_t window, float score_bias, const float* bias_dev,
                   int compress, void* out_state, void* out_val, int out_dtype, const jk_heads_t* heads,
                   jk_stream_t stream, int debug_stall = 0) {
  if (compress != JK_SOFTSIGN && compress != JK_SIGNED_ABS_SOFTMAX && compress != JK_SIGNED_ENTMAX15)
    return JK_ERR_UNSUPPORTED_KIND;
  if (window < -1) return JK_ERR_BAD_ARG;
  Params p;
  const int st = prepare(row_proj, col_proj, batch, n_rows, n_cols, rp, proj_dtype, col_state, state_dtype, col_val,
                         col_val_lo, dim, score_bias, bias_dev, compress, out_state, out_val, out_dtype, heads, p);
  if (st != JK_OK) return st;
  p.window = window;
  p.debug_stall = debug_stall;
  return run(row_proj, col_proj, col_val, col_val_lo, batch, n_rows, n_cols, rp, proj_dtype, p, stream);
}

int transition_dense_forward(const void* src_proj, const void* dst_proj, int64_t batch, int64_t n_src,
                             int64_t n_dst, int64_t rp, int proj_dtype, const void* src_state, const void* sender,
                             int state_dtype, const void* src_val, const void* src_val_lo, int64_t dim,
                             float score_bias, const float* bias_dev, int compress, float* stats, void* out_state,
                             void* out_val, int out_dtype, const jk_heads_t* heads, jk_stream_t stream) {
  if (compress != JK_SOFTMAX && compress != JK_SIGNED_ABS_SOFTMAX && compress != JK_SIGNED_ENTMAX15)
    return JK_ERR_UNSUPPORTED_KIND;
  if (stats == nullptr) return JK_ERR_BAD_ARG;
  // Aggregate launch: rows = destinations, columns = sources, per-column normalisation.
  Params agg;
  int st = prepare(dst_proj, src_proj, batch, n_dst, n_src, rp, proj_dtype, src_state, state_dtype, src_val,
                   src_val_lo, dim, score_bias, bias_dev, compress, out_state, out_val, out_dtype, heads, agg);
  if (st != JK_OK) return st;
  // Statistics launch: rows = sources, columns = destinations; the sender strength scales
  // each source's normaliser.
  Params sp = agg;
  sp.n_rows = n_src;
  sp.n_cols = n_dst;
  sp.stats_out = stats;
  sp.row_scale = sender;
  sp.out_state = nullptr;
  sp.out_val = nullptr;
  st = run(src_proj, dst_proj, nullptr, nullptr, batch, n_src, n_dst, rp, proj_dtype, sp, stream);
  if (st != JK_OK) return st;
  agg.col_stats = stats;
  return run(dst_proj, src_proj, src_val, src_val_lo, batch, n_dst, n_src, rp, proj_dtype, agg, stream);
}

}  // namespace win
}  // namespace jk

// Failure-path test entry: jk_propagation_window_forward with a producer warp that issues
// nothing. Every consumer wait gives up after its bound (about 2 s), sets the device error
// word, releases TMEM and returns; jk_device_status then reports JK_ERR_DEVICE_TIMEOUT and
// the context stays usable. Outputs are zeros. Only for tests of that path.
extern "C" int jk_debug_window_stalled_producer(const void* row_proj, const void* col_proj, int64_t batch,
                                                int64_t n_rows, int64_t n_cols, int64_t rp, int proj_dtype,
                                                const void* col_state, int state_dtype, const void* col_val,
                                                int64_t dim, int64_t window, void* out_state, void* out_val,
                                                int out_dtype, jk_stream_t stream) {
  return jk::win::window_forward(row_proj, col_proj, batch, n_rows, n_cols, rp, proj_dtype, col_state, state_dtype,
                                 col_val, nullptr, dim, window, 0.f, nullptr, JK_SOFTSIGN, out_state, out_val,
                                 out_dtype, nullptr, stream, 1);
}

extern "C" int jk_propagation_window_forward(const void* row_proj, const void* col_proj, int64_t batch,
                                             int64_t n_rows, int64_t n_cols, int64_t rp, int proj_dtype,
                                             const void* col_state, int state_dtype, const void* col_val,
                                             const void* col_val_lo, int64_t dim, int64_t window, float score_bias,
                                             const float* bias_dev, int compress, void* out_state, void* out_val,
                                             int out_dtype, jk_stream_t stream) {
  return jk::win::window_forward(row_proj, col_proj, batch, n_rows, n_cols, rp, proj_dtype, col_state, state_dtype,
                                 col_val, col_val_lo, dim, window, score_bias, bias_dev, compress, out_state, out_val,
                                 out_dtype, nullptr, stream);
}

extern "C" int jk_propagation_window_forward_mh(const void* row_proj, const void* col_proj, int64_t batch,
                                                int64_t n_rows, int64_t n_cols, int64_t rp, int proj_dtype,
                                                const void* col_state, int state_dtype, const void* col_val,
                                                const void* col_val_lo, int64_t dim, int64_t window,
                                                float score_bias, const float* bias_dev, int compress,
                                                void* out_state, void* out_val, int out_dtype,
                                                const jk_heads_t* heads, jk_stream_t stream) {
  if (heads == nullptr) return JK_ERR_BAD_ARG;
  return jk::win::window_forward(row_proj, col_proj, batch, n_rows, n_cols, rp, proj_dtype, col_state, state_dtype,
                                 col_val, col_val_lo, dim, window, score_bias, bias_dev, compress, out_state, out_val,
                                 out_dtype, heads, stream);
}

extern "C" int jk_transition_pairwise_dense_forward(const void* src_proj, const void* dst_proj, int64_t batch,
                                                    int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                                    const void* src_state, const void* sender, int state_dtype,
                                                    const void* src_val, const void* src_val_lo, int64_t dim,
                                                    float score_bias, const float* bias_dev, int compress,
                                                    float* stats, void* out_state, void* out_val, int out_dtype,
                                                    jk_stream_t stream) {
  return jk::win::transition_dense_forward(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, src_state, sender,
                                           state_dtype, src_val, src_val_lo, dim, score_bias, bias_dev, compress,
                                           stats, out_state, out_val, out_dtype, nullptr, stream);
}

extern "C" int jk_transition_pairwise_dense_forward_mh(const void* src_proj, const void* dst_proj, int64_t batch,
                                                       int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                                       const void* src_state, const void* sender, int state_dtype,
                                                       const void* src_val, const void* src_val_lo, int64_t dim,
                                                       float score_bias, const float* bias_dev, int compress,
                                                       float* stats, void* out_state, void* out_val, int out_dtype,
                                                       const jk_heads_t* heads, jk_stream_t stream) {
  if (heads == nullptr) return JK_ERR_BAD_ARG;
  return jk::win::transition_dense_forward(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, src_state, sender,
                                           state_dtype, src_val, src_val_lo, dim, score_bias, bias_dev, compress,
                                           stats, out_state, out_val, out_dtype, heads, stream);
}

namespace jk {
JK_ERROR_READER(read_error_window)
}  // namespace jk
