// Launchers of the fused top-k kernel for bf16 values (see jk_topk_kernel.cuh); a unit of
// its own so that the library's units compile in parallel. It has its own device error
// word, read by jk_device_status.
#include "jk_topk_kernel.cuh"

namespace jk {
namespace topk {

JK_TOPK_INSTANTIATE(__nv_bfloat16)

}  // namespace topk

JK_ERROR_READER(read_error_topk_bf16)

}  // namespace jk

#ifdef JK_PHASE_PROFILE
extern "C" int jk_debug_trace(long long* out, int n_ctas) {
  cudaDeviceSynchronize();
  const int n = n_ctas < jk::topk::kTraceCtas ? n_ctas : jk::topk::kTraceCtas;
  return cudaMemcpyFromSymbol(out, jk::topk::g_trace, sizeof(long long) * 32 * n) == cudaSuccess ? 0 : -1;
}
#endif
