// Allocation-free variant of the per-source sparse transition.
//
// jk_transition_pairwise_topk_forward needs f32 scratch for its scatter accumulators and
// expects the caller to allocate it. Some callers cannot: a plain-C or FFI host (Go, Java,
// Rust bindings) that has no device allocator of its own and only holds the input and
// output buffers it was handed, or a latency-critical loop that must not call cudaMalloc /
// cudaFree because they can synchronise the whole device. For them this file keeps the
// scratch in a fixed file-scope device array -- every GPU that loads the library holds it
// until the process exits -- and offers one more entry point that allocates nothing.
//
// Every call resolves the array's device address on the current device
// (cudaGetSymbolAddress with that device current); the first call on a device also loads the
// module there, so make it before any stream capture. All calls on
// a device share the one array, so calls whose kernels overlap on the GPU (different
// streams, or different host threads) race and corrupt each other's results; serialise
// them on one stream.
#include "jk_host.h"

namespace jk {
namespace noalloc {

// 4 Mi floats = 16 MiB per device: B * n_dst * (dim + 1) must not exceed this.
constexpr int64_t kScratchFloats = int64_t(1) << 22;

static __device__ __align__(256) float g_transition_scratch[kScratchFloats];

// Device address of g_transition_scratch on the current device. It is looked up on every
// call, with the caller's device current, instead of being cached: a cached address would go
// stale after a device reset or when a driver-API host calls from another context on the
// same device. (The symbol's host-side name is only a stand-in, not a device address.)
int scratch_address(float** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_transition_scratch) != cudaSuccess || p == nullptr) {
    cudaGetLastError();
    return JK_ERR_LAUNCH;
  }
  *out = static_cast<float*>(p);
  return JK_OK;
}

}  // namespace noalloc
}  // namespace jk

extern "C" int64_t jk_transition_pairwise_topk_noalloc_capacity(void) { return jk::noalloc::kScratchFloats; }

extern "C" int jk_transition_pairwise_topk_forward_noalloc(const void* src_proj, const void* dst_proj, int64_t batch,
                                                           int64_t n_src, int64_t n_dst, int64_t rp, int proj_dtype,
                                                           const void* src_state, const void* src_sender,
                                                           int state_dtype, const void* src_val, int64_t dim,
                                                           int val_dtype, int64_t k, float score_bias,
                                                           const float* bias_dev, int compress, void* out_state,
                                                           void* out_val, int out_dtype, jk_stream_t stream) {
  using namespace jk;
  if (batch <= 0 || n_dst <= 0 || dim <= 0) return JK_ERR_BAD_SHAPE;
  // Reject sizes beyond the fixed scratch (overflow-safe).
  if (n_dst > noalloc::kScratchFloats / batch || dim + 1 > noalloc::kScratchFloats / (batch * n_dst))
    return JK_ERR_BAD_SHAPE;
  int st = check_device();
  if (st != JK_OK) return st;
  float* scratch = nullptr;
  st = noalloc::scratch_address(&scratch);
  if (st != JK_OK) return st;
  // The regular entry point zeroes the accumulators on the stream before use, so the
  // previous call's contents never leak into this one.
  return jk_transition_pairwise_topk_forward(src_proj, dst_proj, batch, n_src, n_dst, rp, proj_dtype, src_state,
                                             src_sender, state_dtype, src_val, dim, val_dtype, k, score_bias,
                                             bias_dev, compress, scratch, out_state, out_val, out_dtype, stream);
}
