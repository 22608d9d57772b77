// status.cuh — host-side error state shared by every C-ABI entry point, and
// the per-translation-unit device error word that bounded waits report to.
#pragma once
#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>

#include "../../include/oxf.h"

namespace oxf {

// Records a message for oxf_last_error_string() and returns `st`.
oxf_status set_error(oxf_status st, const char* fmt, ...);

inline oxf_status check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return OXF_OK;
  return set_error(OXF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Counts kernel launches made through this library (oxf_kernel_launches).
void count_launch();

// Launch-error check after a kernel launch (does not synchronise); every
// launch site calls it exactly once, so it also counts launches.
inline oxf_status check_launch(const char* what) {
  count_launch();
  return check_cuda(cudaGetLastError(), what);
}

// Device error codes written by bounded waits (first error wins).
enum DeviceErrorCode : uint32_t {
  DEVERR_NONE = 0,
  DEVERR_GEMM_WAIT_EMPTY = 0x101,
  DEVERR_GEMM_WAIT_FULL = 0x102,
  DEVERR_GEMM_WAIT_TMEM_EMPTY = 0x103,
  DEVERR_GEMM_WAIT_TMEM_FULL = 0x104,
  DEVERR_GEMM_DRAIN = 0x105,
  DEVERR_GEMM_EPI_LOAD = 0x106,
  DEVERR_GEMM_QUEUE = 0x107,  // tile queue (dynamic schedule): entry never published / freed
  DEVERR_ATTN_WAIT = 0x108,  // fused multi-head attention: a pipeline wait expired
  DEVERR_WAIT_SELFTEST = 0x1FF,  // oxf_wait_timeout_selftest: the expected expiry
  DEVERR_ROW_PARAMS = 0x301,  // a norm kernel's gamma/beta copy into shared memory never landed
};

}  // namespace oxf

// One error word per translation unit that includes this header. The GEMM,
// attention, row-kernel and exchange translation units have bounded waits;
// each exposes its word to oxf_device_error().
static __device__ unsigned int g_oxf_device_error = 0;

namespace oxf {
__device__ __forceinline__ void report_device_error(uint32_t code) {
  atomicCAS(&g_oxf_device_error, 0u, code);
}
}  // namespace oxf
