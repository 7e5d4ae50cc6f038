// Launchers of the fused top-k kernel for f32 values (see jk_topk_kernel.cuh); a unit of
// its own so that the library's units compile in parallel. It has its own device error
// word, read by jk_device_status.
#include "jk_topk_kernel.cuh"

namespace jk {
namespace topk {

JK_TOPK_INSTANTIATE(float)

}  // namespace topk

JK_ERROR_READER(read_error_topk_f32)

}  // namespace jk
