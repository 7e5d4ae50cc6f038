// Host-side helpers shared by the Jakal-Net B200 entry points: status handling,
// device checks and TMA tensor-map encoding through the driver entry point (so the
// library needs no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/jakal_b200.h"

namespace jk {

// Device-side error word (JK_OK or JK_ERR_DEVICE_TIMEOUT), written by kernels whose
// bounded wait gave up. The library is built from several translation units without
// relocatable device code, so every unit that includes this header has its own copy;
// JK_ERROR_READER defines the unit's host function that reads and clears its copy, and
// jk_device_status combines them.
static __device__ int g_device_error = 0;

#define JK_ERROR_READER(name)                                                             \
  int name(int* value) {                                                                \
    int zero = 0;                                                                       \
    if (cudaMemcpyFromSymbol(value, g_device_error, sizeof(int)) != cudaSuccess ||      \
        cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) {        \
      cudaGetLastError();                                                               \
      return JK_ERR_LAUNCH;                                                             \
    }                                                                                   \
    return JK_OK;                                                                       \
  }

// Readers of the units that launch kernels with bounded waits (jk_project.cu, jk_topk.cu and
// its per-value-type units jk_topk_vt_*.cu, jk_window.cu).
int read_error_project(int* value);
int read_error_topk(int* value);
int read_error_topk_bf16(int* value);
int read_error_topk_f16(int* value);
int read_error_topk_f32(int* value);
int read_error_window(int* value);

// Returns JK_OK when the current device is sm_100 (cached per device ordinal).
int check_device();

// Maps the last CUDA runtime error to a status code (JK_OK when none).
int launch_status();

// Encodes a 3-D tiled tensor map over a contiguous [d2][d1][d0] array of 16-bit elements
// with a {box0, box1, 1} box, 128-byte swizzled (MMA operands) or plain row-major. Returns JK_OK or an error status.
int make_tmap_3d_16bit(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                       uint32_t box0, uint32_t box1, bool bf16, bool swizzle128 = true);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Scorer heads of a call: 1 (single low-rank scorer) when h is null, else h checked
// against the projection width rp and the kernel's head limit.
struct Heads {
  int heads = 1, kph = 0, combine = 0;
  const float* bias = nullptr;
};

inline int read_heads(const jk_heads_t* h, int64_t rp, int proj_dtype, int max_heads, Heads& out) {
  out = Heads{};
  if (h == nullptr) return JK_OK;
  if (proj_dtype == JK_BF16X3) return JK_ERR_UNSUPPORTED_KIND;
  if (h->combine < JK_HEADS_MAX || h->combine > JK_HEADS_SIGNED_SMOOTHMAX) return JK_ERR_UNSUPPORTED_KIND;
  if (h->heads < 2 || h->heads > max_heads || h->kph < 1 || int64_t(h->heads) * 16 * h->kph > rp)
    return JK_ERR_BAD_SHAPE;
  out.heads = h->heads;
  out.kph = h->kph;
  out.combine = h->combine;
  out.bias = h->head_bias;
  return JK_OK;
}

}  // namespace jk
