// Thin inline-PTX layer for the sm_100a features the Jakal-Net B200 kernels use:
// mbarriers, TMA tiled loads, tcgen05 (TMEM alloc, MMA, commit, load) and the
// shared-memory / instruction descriptors the MMA consumes.
//
// Every wait in this file is bounded: a wait that does not complete within
// JK_WAIT_LIMIT_CYCLES returns false, and the caller records an error status and
// unwinds instead of spinning forever.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#ifndef JK_WAIT_LIMIT_CYCLES
// About 2 s at the B200 boost clock; long enough never to trip on a healthy run.
#define JK_WAIT_LIMIT_CYCLES (4000000000ll)
#endif

namespace jk {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Makes barrier initialisation visible to the async proxy (TMA, tcgen05.commit).
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on the given phase parity. Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - start > JK_WAIT_LIMIT_CYCLES) return false;
  }
}

// ---------------------------------------------------------------- TMA
// 3-D tiled store shared -> global of one box (bulk-group completion). The innermost
// coordinate c0 must be a multiple of 16 bytes / element size and no coordinate negative.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until the shared-memory sources of every committed bulk store have been read.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// 3-D tiled load global -> shared, completion counted on `bar` in bytes.
// The innermost coordinate c0 must be a multiple of 16 bytes / element size.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- tcgen05
// Allocation is warp-wide; the allocated base column is written to *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 or f16 operands, f32 accum).
__device__ __forceinline__ void mma_f16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05 op this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives lane (base_lane+i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16: A (M = 128 rows = TMEM lanes) is read
// from TMEM, one 32-bit column holding two consecutive K elements.
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Warp-collective store of 16 consecutive 32-bit columns of the warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Warp-collective store of 32 consecutive 32-bit columns of the warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand stored in the canonical
// 128-byte-swizzle layout that a TMA load with CU_TENSOR_MAP_SWIZZLE_128B writes:
// rows of 128 B (64 bf16 along K), 8-row groups 1024 B apart. The tile base must be
// 1024-byte aligned; advancing along K inside the 128-byte atom is done by adding
// the byte offset (>>4) to the start-address field.
__device__ __forceinline__ uint64_t sdesc_kmajor_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);  // start address
  d |= static_cast<uint64_t>(1) << 16;                      // leading byte offset (unused)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;              // stride byte offset: 8 rows
  d |= static_cast<uint64_t>(1) << 46;                      // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                      // layout: SWIZZLE_128B
  return d;
}

// Shared-memory matrix descriptor for an MN-major operand in the 128-byte-swizzle layout a
// TMA box of {64 elements along MN, rows along K} writes: each K row is 128 B (64 MN
// elements), 8 K rows form a 1024 B atom (stride byte offset), and the next 64 MN elements
// live `mn_atom_bytes` further (leading byte offset, one TMA box per 64 MN elements).
__device__ __forceinline__ uint64_t sdesc_mnmajor_sw128(uint32_t smem_addr, uint32_t mn_atom_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((mn_atom_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with f32 accumulation, both operands K-major.
// ab_format: 0 = f16, 1 = bf16.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, uint32_t ab_format) {
  return (1u << 4)                      // D format f32
         | (ab_format << 7)             // A format
         | (ab_format << 10)            // B format
         | ((uint32_t)(N >> 3) << 17)   // N / 8
         | ((uint32_t)(M >> 4) << 24);  // M / 16
}

// Score tile MMAs: D = A . B^T over the padded rank. Plain 16-bit projections: K steps
// 0 .. 4*KATOMS-1 pair with themselves. Three-plane bf16 split of f32 projections (rank
// <= 32, planes h | m | l at K steps {0,1} {2,3} {4,5} of a 128-wide row): the six products
// hh, hm, mh, hl, lh, mm reproduce an f32 dot product.
template <int KATOMS>
__device__ __forceinline__ void score_mmas(uint32_t tmem_d, uint32_t a_addr, uint32_t b_addr, uint32_t idesc,
                                           bool split3) {
  constexpr uint32_t kAtom = 128 * 128;
  if (KATOMS == 2 && split3) {
    const int pa[6] = {0, 0, 1, 0, 2, 1};
    const int pb[6] = {0, 1, 0, 2, 0, 1};
#pragma unroll
    for (int q = 0; q < 12; ++q) {
      const int sa = pa[q >> 1] * 2 + (q & 1);
      const int sb = pb[q >> 1] * 2 + (q & 1);
      const uint32_t oa = (sa >> 2) * kAtom + (sa & 3) * 32;
      const uint32_t ob = (sb >> 2) * kAtom + (sb & 3) * 32;
      mma_f16_ss(tmem_d, sdesc_kmajor_sw128(a_addr + oa), sdesc_kmajor_sw128(b_addr + ob), idesc, q > 0 ? 1u : 0u);
    }
  } else {
#pragma unroll
    for (int kk = 0; kk < 4 * KATOMS; ++kk) {
      const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
      mma_f16_ss(tmem_d, sdesc_kmajor_sw128(a_addr + off), sdesc_kmajor_sw128(b_addr + off), idesc, kk > 0 ? 1u : 0u);
    }
  }
}

// Multi-head scores: head h owns the kph K steps [h * kph, (h + 1) * kph) of the projection
// rows and accumulates into its own TMEM plane tmem_d + h * plane_cols.
__device__ __forceinline__ void head_score_mmas(uint32_t tmem_d, uint32_t plane_cols, uint32_t a_addr,
                                                uint32_t b_addr, uint32_t idesc, int heads, int kph) {
  constexpr uint32_t kAtom = 128 * 128;
  for (int h = 0; h < heads; ++h) {
    for (int kk = 0; kk < kph; ++kk) {
      const int g = h * kph + kk;
      const uint32_t off = (g >> 2) * kAtom + (g & 3) * 32;
      mma_f16_ss(tmem_d + h * plane_cols, sdesc_kmajor_sw128(a_addr + off), sdesc_kmajor_sw128(b_addr + off), idesc,
                 kk > 0 ? 1u : 0u);
    }
  }
}

// Head combination of MultiHeadPairwise (modules.py:274-299) for 16 score columns of this
// thread's TMEM lane: every head plane (at taddr + h * plane_cols) plus its bias, then
//   JK_HEADS_MAX: max_h s_h;  JK_HEADS_SMOOTHMAX: logsumexp_h s_h - log H;
//   JK_HEADS_SIGNED_SMOOTHMAX: sum_h s_h * softmax_h(|s_h|)   (online over the heads).
template <int H>
__device__ __forceinline__ void combine_heads16(uint32_t taddr, uint32_t plane_cols, const float* head_bias,
                                                int combine, float (&out)[16]) {
  uint32_t t[H][16];
#pragma unroll
  for (int h = 0; h < H; ++h) tmem_ld_32x32b_x16(taddr + h * plane_cols, t[h]);
  tmem_ld_wait();
  float bh[H];
#pragma unroll
  for (int h = 0; h < H; ++h) bh[h] = head_bias ? __ldg(head_bias + h) : 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float s0 = __uint_as_float(t[0][i]) + bh[0];
    if (combine == JK_HEADS_MAX) {
      float m = s0;
#pragma unroll
      for (int h = 1; h < H; ++h) m = fmaxf(m, __uint_as_float(t[h][i]) + bh[h]);
      out[i] = m;
    } else if (combine == JK_HEADS_SMOOTHMAX) {
      float m = s0;
#pragma unroll
      for (int h = 1; h < H; ++h) m = fmaxf(m, __uint_as_float(t[h][i]) + bh[h]);
      float z = 0.f;
#pragma unroll
      for (int h = 0; h < H; ++h) z += expf(__uint_as_float(t[h][i]) + bh[h] - m);
      out[i] = m + logf(z) - logf(static_cast<float>(H));
    } else {
      float m = fabsf(s0);
#pragma unroll
      for (int h = 1; h < H; ++h) m = fmaxf(m, fabsf(__uint_as_float(t[h][i]) + bh[h]));
      float num = 0.f, den = 0.f;
#pragma unroll
      for (int h = 0; h < H; ++h) {
        const float s = __uint_as_float(t[h][i]) + bh[h];
        const float e = expf(fabsf(s) - m);
        num = fmaf(s, e, num);
        den += e;
      }
      out[i] = num / den;
    }
  }
}

__device__ __forceinline__ uint32_t elect_lane0() {
  return (threadIdx.x & 31) == 0;
}

// ---------------------------------------------------------------- misc
__device__ __forceinline__ float ld_elem(const void* p, long long i, int dtype) {
  // dtype: 0 f32, 1 bf16, 2 f16
  if (dtype == 0) return __ldg(reinterpret_cast<const float*>(p) + i);
  if (dtype == 1) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void st_elem(void* p, long long i, int dtype, float v) {
  if (dtype == 0) {
    reinterpret_cast<float*>(p)[i] = v;
  } else if (dtype == 1) {
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  }
}

// Stores 8 f32 values at base[elem ..] in dtype (f32: two 16-byte stores, 16-bit: one).
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

// softplus as torch.nn.functional.softplus (beta=1, threshold=20).
__device__ __forceinline__ float softplus_f(float x) {
  return x > 20.f ? x : log1pf(expf(x));
}

}  // namespace jk
