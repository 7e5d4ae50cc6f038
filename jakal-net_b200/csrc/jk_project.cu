// Low-rank projection prologue: out = round(x . w^T) [* core] [/ temperature], written
// into a rank-padded [rows, rp] buffer the fused kernels read with TMA.
//
// One CTA per 128 rows: warp 4 issues TMA loads of x / w chunks (64 columns of the
// model dimension per stage, 128-byte swizzle) and the tcgen05 MMAs (M=128, N=rp,
// K=16 steps) into a TMEM accumulator; warps 0-3 read the accumulator back
// (thread = row) and apply the rounding chain of the reference:
//   jakal_net_native.cpp:6236-6239  projected = torch::matmul(val, W^T)   (input dtype)
//                                  weighted  = projected * w.to(dtype)
//   jakal_net_native.cpp:6979-6983  weighted  = weighted / temperature     (routes)
#include "jk_host.h"
#include "jk_sm100.cuh"

namespace jk {
namespace proj {

#ifdef JK_PHASE_PROFILE
__device__ long long g_ptrace[1024][16];
#define JK_PSTAMP(i)                                     \
  do {                                                   \
    if (blockIdx.x < 1024) g_ptrace[blockIdx.x][i] = clock64(); \
  } while (0)
#else
#define JK_PSTAMP(i) \
  do {               \
  } while (0)
#endif

constexpr int kRows = 128;
constexpr int kStages = 6;  // a whole 384-wide row of x in flight: one HBM latency, not two
constexpr int kThreads = 160;

struct Params {
  int64_t rows;
  int64_t dim;
  int64_t rank;
  int64_t rp;
  const void* core;
  float temperature;
  int bf16;
  void* out;
};

__host__ __device__ constexpr int a_bytes() { return kRows * 128; }

// Rounds to the projection dtype and back (round to nearest even).
template <bool BF16>
__device__ __forceinline__ float round16(float x) {
  if (BF16) return __bfloat162float(__float2bfloat16_rn(x));
  return __half2float(__float2half_rn(x));
}

// The dtype, core and temperature steps are template parameters: the epilogue below is
// unrolled over every column of a row, and per-element runtime branches over all variants
// made that straight-line code several times larger -- instruction fetch, not arithmetic,
// then dominated the kernel.
// PAIR: one x tile against two weights (w then w2, rank <= 64 each, stacked into one N = 128
// operand): columns 0-63 are the plain projection (out), 64-127 the core / temperature one
// (out2) -- the target and source projections of a propagation in one pass over x.
template <int RP, bool BF16, bool CORE, bool TEMP, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    project_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_out,
                   const __grid_constant__ CUtensorMap tm_out2, Params p) {
  static_assert(!PAIR || RP == 128, "a pair projection is one N = 128 GEMM");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kABytes = a_bytes();
  constexpr int kBBytes = RP * 128;
  constexpr int kStageBytes = kABytes + kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ float core_s[128];  // core weight widened once per CTA (1.0 when absent)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRows;
  const int nchunks = static_cast<int>((p.dim + 63) / 64);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x < 128) {
    float cw = 1.f;
    if (p.core != nullptr && threadIdx.x < p.rank) {
      cw = p.bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.core)[threadIdx.x])
                  : __half2float(reinterpret_cast<const __half*>(p.core)[threadIdx.x]);
    }
    core_s[threadIdx.x] = cw;
  }
  if (warp == 0) tmem_alloc(tmem_slot, RP < 32 ? 32 : RP);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) JK_PSTAMP(0);

  if (warp == 4) {
    if (lane == 0) {
      prefetch_tmap(&tm_x);
      prefetch_tmap(&tm_w);
      if (PAIR) prefetch_tmap(&tm_w2);
      const uint32_t idesc = idesc_f16(128, RP, p.bf16 ? 1u : 0u);
      bool ok = true;
      // Prefill.
      const int pre = nchunks < kStages ? nchunks : kStages;
      for (int c = 0; c < pre; ++c) {
        uint8_t* st = smem + c * kStageBytes;
        mbar_arrive_expect_tx(&full[c], kStageBytes);
        tma_load_3d(st, &tm_x, &full[c], c * 64, static_cast<int>(row0), 0);
        tma_load_3d(st + kABytes, &tm_w, &full[c], c * 64, 0, 0);
        if (PAIR) tma_load_3d(st + kABytes + 64 * 128, &tm_w2, &full[c], c * 64, 0, 0);
      }
      for (int c = 0; c < nchunks && ok; ++c) {
        const int s = c % kStages;
        if (!mbar_wait(&full[s], (c / kStages) & 1)) { ok = false; break; }
        if (c < 8) JK_PSTAMP(1 + c);
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * kStageBytes);
        const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_f16_ss(tmem, sdesc_kmajor_sw128(a_addr + kk * 32), sdesc_kmajor_sw128(b_addr + kk * 32),
                     idesc, (c > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&empty[s]);
        // Refill the stage of the previous chunk once its MMAs retired.
        const int cp = c - 1;
        if (cp >= 0 && cp + kStages < nchunks) {
          const int sp = cp % kStages;
          if (!mbar_wait(&empty[sp], (cp / kStages) & 1)) { ok = false; break; }
          uint8_t* st = smem + sp * kStageBytes;
          mbar_arrive_expect_tx(&full[sp], kStageBytes);
          tma_load_3d(st, &tm_x, &full[sp], (cp + kStages) * 64, static_cast<int>(row0), 0);
          tma_load_3d(st + kABytes, &tm_w, &full[sp], (cp + kStages) * 64, 0, 0);
          if (PAIR) tma_load_3d(st + kABytes + 64 * 128, &tm_w2, &full[sp], (cp + kStages) * 64, 0, 0);
        }
      }
      if (ok) {
        mma_commit(done);
        const int last = nchunks - 1;
        ok = mbar_wait(&empty[last % kStages], (last / kStages) & 1);
      }
      if (!ok) {
        atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
        *abort_flag = 1;
      }
    }
  } else {
    // Epilogue: thread = row. The rounded row goes into the (now idle) first operand stage
    // in the 128-byte-swizzled layout of the output tensor map -- RP / 64 boxes of 128 rows
    // x 64 columns -- and one thread stores the tile with TMA (rows past p.rows are clipped).
    bool ok = mbar_wait(done, 0);
    if (threadIdx.x == 0) JK_PSTAMP(10);
    if (!ok) {
      atomicExch(&g_device_error, JK_ERR_DEVICE_TIMEOUT);
    } else {
      tc_fence_after();
      const int r_in = warp * 32 + lane;
      uint8_t* stage = smem;  // every MMA has retired: the stages are free
#pragma unroll
      for (int cb = 0; cb < RP; cb += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + cb, v);
        tmem_ld_wait();
        if (threadIdx.x == 0 && cb == 0) JK_PSTAMP(12);
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float f[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = PAIR ? (cb + i + h) & 63 : cb + i + h;
            const bool weighted = !PAIR || cb >= 64;  // a pair's plain half takes no core / 1/T
            float x = round16<BF16>(__uint_as_float(v[i + h]));
            if (CORE && weighted) x = round16<BF16>(x * core_s[c]);
            if (TEMP && weighted) x = round16<BF16>(x / p.temperature);
            f[h] = c < p.rank ? x : 0.f;
          }
          if (BF16) {
            __nv_bfloat162 b2 = __floats2bfloat162_rn(f[0], f[1]);
            packed[i / 2] = *reinterpret_cast<uint32_t*>(&b2);
          } else {
            __half2 h2 = __floats2half2_rn(f[0], f[1]);
            packed[i / 2] = *reinterpret_cast<uint32_t*>(&h2);
          }
        }
        // columns [cb, cb + 32) = 16-byte chunks (cb % 64) / 8 .. + 3 of box cb / 64
        uint8_t* box = stage + (cb / 64) * (kRows * 128) + (r_in >> 3) * 1024 + (r_in & 7) * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = ((cb & 63) >> 3) + q;
          *reinterpret_cast<uint4*>(box + ((chunk ^ (r_in & 7)) << 4)) =
              make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
        if (threadIdx.x == 0 && cb == 0) JK_PSTAMP(13);
      }
      fence_proxy_async_smem();
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
      if (threadIdx.x == 0) {
#pragma unroll
        for (int bx = 0; bx < RP / 64; ++bx) {
          if (PAIR)
            tma_store_3d(bx == 0 ? &tm_out : &tm_out2, stage + bx * kRows * 128, 0, static_cast<int>(row0), 0);
          else
            tma_store_3d(&tm_out, stage + bx * kRows * 128, bx * 64, static_cast<int>(row0), 0);
        }
        bulk_commit_group();
        bulk_wait_group_read0();
      }
    }
    if (threadIdx.x == 0) JK_PSTAMP(14);
    tc_fence_before();
  }
  __syncthreads();
  if (threadIdx.x == 0) JK_PSTAMP(11);
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, RP < 32 ? 32 : RP);
  }
}

template <int RP>
constexpr int smem_bytes() {
  return 1024 + kStages * (a_bytes() + RP * 128) + 256;
}

template <int RP, bool BF16, bool CORE, bool TEMP, bool PAIR = false>
int launch_one(dim3 grid, cudaStream_t s, const CUtensorMap& tm_x, const CUtensorMap& tm_w, const CUtensorMap& tm_out,
               const Params& p, const CUtensorMap* tm_w2 = nullptr, const CUtensorMap* tm_out2 = nullptr) {
  constexpr int sm = smem_bytes<RP>();
  auto kern = project_kernel<RP, BF16, CORE, TEMP, PAIR>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sm) != cudaSuccess) {
    cudaGetLastError();
    return JK_ERR_LAUNCH;
  }
  kern<<<grid, kThreads, sm, s>>>(tm_x, tm_w, tm_w2 ? *tm_w2 : tm_w, tm_out, tm_out2 ? *tm_out2 : tm_out, p);
  return JK_OK;
}

template <int RP>
int dispatch(int variant, dim3 grid, cudaStream_t s, const CUtensorMap& tm_x, const CUtensorMap& tm_w,
             const CUtensorMap& tm_out, const Params& p) {
  switch (variant) {
    case 0: return launch_one<RP, false, false, false>(grid, s, tm_x, tm_w, tm_out, p);
    case 1: return launch_one<RP, false, false, true>(grid, s, tm_x, tm_w, tm_out, p);
    case 2: return launch_one<RP, false, true, false>(grid, s, tm_x, tm_w, tm_out, p);
    case 3: return launch_one<RP, false, true, true>(grid, s, tm_x, tm_w, tm_out, p);
    case 4: return launch_one<RP, true, false, false>(grid, s, tm_x, tm_w, tm_out, p);
    case 5: return launch_one<RP, true, false, true>(grid, s, tm_x, tm_w, tm_out, p);
    case 6: return launch_one<RP, true, true, false>(grid, s, tm_x, tm_w, tm_out, p);
    default: return launch_one<RP, true, true, true>(grid, s, tm_x, tm_w, tm_out, p);
  }
}

}  // namespace proj
}  // namespace jk

extern "C" int jk_lowrank_project(const void* x, int64_t rows, int64_t dim, const void* w,
                                  int64_t rank, const void* core, float temperature, int dtype,
                                  void* out, int64_t out_stride, jk_stream_t stream) {
  using namespace jk;
  if (x == nullptr || w == nullptr || out == nullptr) return JK_ERR_BAD_ARG;
  if (dtype != JK_BF16 && dtype != JK_F16) return JK_ERR_BAD_DTYPE;
  if (rows <= 0 || dim <= 0 || rank <= 0 || rank > 128 || dim % 8 != 0) return JK_ERR_BAD_SHAPE;
  if (rows > (int64_t(1) << 31) - 256 || dim > (int64_t(1) << 30)) return JK_ERR_BAD_SHAPE;
  const int64_t rp = jk_padded_rank(rank);
  if (out_stride != rp) return JK_ERR_BAD_SHAPE;
  if (!(temperature > 0.f)) return JK_ERR_BAD_ARG;
  if (!aligned16(x) || !aligned16(w) || !aligned16(out)) return JK_ERR_ALIGNMENT;
  int st = check_device();
  if (st != JK_OK) return st;

  const bool bf16 = dtype == JK_BF16;
  CUtensorMap tm_x, tm_w;
  st = make_tmap_3d_16bit(&tm_x, x, dim, rows, 1, 64, 128, bf16);
  if (st != JK_OK) return st;
  st = make_tmap_3d_16bit(&tm_w, w, dim, rank, 1, 64, static_cast<uint32_t>(rp), bf16);
  if (st != JK_OK) return st;
  CUtensorMap tm_out;
  st = make_tmap_3d_16bit(&tm_out, out, rp, rows, 1, 64, 128, bf16);
  if (st != JK_OK) return st;

  proj::Params p{rows, dim, rank, rp, core, temperature, bf16 ? 1 : 0, out};
  const dim3 grid(static_cast<unsigned>((rows + 127) / 128));
  auto s = reinterpret_cast<cudaStream_t>(stream);
  const int variant = (bf16 ? 4 : 0) | (core != nullptr ? 2 : 0) | (temperature != 1.f ? 1 : 0);
  if (rp == 64) {
    st = proj::dispatch<64>(variant, grid, s, tm_x, tm_w, tm_out, p);
  } else {
    st = proj::dispatch<128>(variant, grid, s, tm_x, tm_w, tm_out, p);
  }
  if (st != JK_OK) return st;
  return launch_status();
}

extern "C" int jk_lowrank_project_pair(const void* x, int64_t rows, int64_t dim, const void* w, const void* w2,
                                       int64_t rank, const void* core, float temperature, int dtype, void* out,
                                       void* out2, jk_stream_t stream) {
  using namespace jk;
  if (x == nullptr || w == nullptr || w2 == nullptr || out == nullptr || out2 == nullptr) return JK_ERR_BAD_ARG;
  if (dtype != JK_BF16 && dtype != JK_F16) return JK_ERR_BAD_DTYPE;
  if (rows <= 0 || dim <= 0 || rank <= 0 || rank > 64 || dim % 8 != 0) return JK_ERR_BAD_SHAPE;
  if (rows > (int64_t(1) << 31) - 256 || dim > (int64_t(1) << 30)) return JK_ERR_BAD_SHAPE;
  if (!(temperature > 0.f)) return JK_ERR_BAD_ARG;
  if (!aligned16(x) || !aligned16(w) || !aligned16(w2) || !aligned16(out) || !aligned16(out2)) return JK_ERR_ALIGNMENT;
  int st = check_device();
  if (st != JK_OK) return st;
  const bool bf16 = dtype == JK_BF16;
  CUtensorMap tm_x, tm_w, tm_w2, tm_out, tm_out2;
  if ((st = make_tmap_3d_16bit(&tm_x, x, dim, rows, 1, 64, 128, bf16)) != JK_OK) return st;
  if ((st = make_tmap_3d_16bit(&tm_w, w, dim, rank, 1, 64, 64, bf16)) != JK_OK) return st;
  if ((st = make_tmap_3d_16bit(&tm_w2, w2, dim, rank, 1, 64, 64, bf16)) != JK_OK) return st;
  if ((st = make_tmap_3d_16bit(&tm_out, out, 64, rows, 1, 64, 128, bf16)) != JK_OK) return st;
  if ((st = make_tmap_3d_16bit(&tm_out2, out2, 64, rows, 1, 64, 128, bf16)) != JK_OK) return st;
  proj::Params p{rows, dim, rank, 64, core, temperature, bf16 ? 1 : 0, out};
  const dim3 grid(static_cast<unsigned>((rows + 127) / 128));
  auto s = reinterpret_cast<cudaStream_t>(stream);
  const bool c = core != nullptr, t = temperature != 1.f;
  if (bf16) {
    if (c && !t) st = proj::launch_one<128, true, true, false, true>(grid, s, tm_x, tm_w, tm_out, p, &tm_w2, &tm_out2);
    else if (c) st = proj::launch_one<128, true, true, true, true>(grid, s, tm_x, tm_w, tm_out, p, &tm_w2, &tm_out2);
    else st = proj::launch_one<128, true, false, true, true>(grid, s, tm_x, tm_w, tm_out, p, &tm_w2, &tm_out2);
  } else {
    if (c && !t) st = proj::launch_one<128, false, true, false, true>(grid, s, tm_x, tm_w, tm_out, p, &tm_w2, &tm_out2);
    else if (c) st = proj::launch_one<128, false, true, true, true>(grid, s, tm_x, tm_w, tm_out, p, &tm_w2, &tm_out2);
    else st = proj::launch_one<128, false, false, true, true>(grid, s, tm_x, tm_w, tm_out, p, &tm_w2, &tm_out2);
  }
  if (st != JK_OK) return st;
  return launch_status();
}

#ifdef JK_PHASE_PROFILE
extern "C" int jk_debug_ptrace(long long* out, int n) {
  cudaDeviceSynchronize();
  return cudaMemcpyFromSymbol(out, jk::proj::g_ptrace, sizeof(long long) * 16 * (n < 1024 ? n : 1024)) == cudaSuccess ? 0 : -1;
}
#endif

namespace jk {
JK_ERROR_READER(read_error_project)
}  // namespace jk
