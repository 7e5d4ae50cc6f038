// Host utilities and the status / probe entry points of the C ABI.
#include "jk_host.h"

#include <cudaTypedefs.h>
#include <mutex>

namespace jk {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

}  // namespace

int check_device() {
  constexpr int kMaxDev = 64;
  static int cached[kMaxDev];  // 0 unknown, 1 ok, 2 bad
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
    cudaGetLastError();
    return JK_ERR_UNSUPPORTED_DEVICE;
  }
  if (cached[dev] == 0) {
    int major = 0, minor = 0;
    bool ok = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) ==
                  cudaSuccess &&
              cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) ==
                  cudaSuccess;
    cached[dev] = (ok && major == 10 && minor == 0) ? 1 : 2;
    cudaGetLastError();
  }
  return cached[dev] == 1 ? JK_OK : JK_ERR_UNSUPPORTED_DEVICE;
}

int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? JK_OK : JK_ERR_LAUNCH;
}

int make_tmap_3d_16bit(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                       uint32_t box0, uint32_t box1, bool bf16, bool swizzle128) {
  auto encode = get_encode_fn();
  if (encode == nullptr) return JK_ERR_UNSUPPORTED_DEVICE;
  if (!aligned16(base)) return JK_ERR_ALIGNMENT;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};  // bytes, dims 1..2
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                      3, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE,
                      swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? JK_OK : JK_ERR_BAD_SHAPE;
}

}  // namespace jk

extern "C" {

const char* jk_status_string(int status) {
  switch (status) {
    case JK_OK: return "ok";
    case JK_ERR_BAD_SHAPE: return "bad shape: sizes inconsistent or outside the supported range";
    case JK_ERR_BAD_DTYPE: return "bad dtype: dtype code unknown or unsupported by this op";
    case JK_ERR_UNSUPPORTED_KIND: return "unsupported kind: compress or scorer kind not implemented";
    case JK_ERR_UNSUPPORTED_DEVICE: return "unsupported device: requires an sm_100 (B200) GPU";
    case JK_ERR_LAUNCH: return "CUDA launch or runtime error";
    case JK_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case JK_ERR_BAD_ARG: return "bad argument: null pointer or out-of-range parameter";
    case JK_ERR_ALIGNMENT: return "pointer not 16-byte aligned";
    default: return "unknown status";
  }
}

int jk_device_check(void) { return jk::check_device(); }

int jk_device_status(jk_stream_t stream, int* device_status) {
  if (device_status == nullptr) return JK_ERR_BAD_ARG;
  if (cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) {
    cudaGetLastError();
    return JK_ERR_LAUNCH;
  }
  int (*readers[])(int*) = {jk::read_error_project,  jk::read_error_topk,     jk::read_error_topk_bf16,
                            jk::read_error_topk_f16, jk::read_error_topk_f32, jk::read_error_window};
  int combined = JK_OK;
  for (auto read : readers) {
    int value = JK_OK;
    const int st = read(&value);
    if (st != JK_OK) return st;
    if (value != JK_OK) combined = value;
  }
  *device_status = combined;
  return JK_OK;
}

int64_t jk_padded_rank(int64_t rank) { return rank <= 0 ? 0 : ((rank + 63) / 64) * 64; }

}  // extern "C"
