// Shared host/device helpers of the q35b200 library: status handling, the
// per-device error word, bf16 conversions and warp reductions.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/q35b200.h"

namespace q35 {

// ---------------------------------------------------------------- host side
// Records a formatted detail message for q35_last_error_message() and returns
// `status`, so call sites read `return fail(Q35_ERR_SHAPE, "...", ...)`.
int fail(int status, const char *fmt, ...);
// Maps a cudaError_t to Q35_ERR_CUDA with the CUDA error string attached.
int cuda_fail(cudaError_t e, const char *what);
// Device error word of the current device (4 ints: code, site, a, b); lazily
// allocated once per device, zero-initialised.
int *device_error_word();
// Number of SMs of the current device (cached).
int num_sms();
// Raises a kernel's dynamic shared-memory limit to `bytes` on the current
// device, once (cached per device and kernel) so launches inside CUDA-graph
// capture make no attribute calls.
int ensure_smem_attr(const void *kernel, int bytes);
// Counts one kernel launch issued by this library (read by q35_launch_count).
void count_launch();

#define Q35_CHECK_CUDA(expr)                                   \
  do {                                                         \
    cudaError_t _e = (expr);                                   \
    if (_e != cudaSuccess) return ::q35::cuda_fail(_e, #expr); \
  } while (0)

#define Q35_LAUNCH_CHECK(what)                                   \
  do {                                                           \
    ::q35::count_launch();                                       \
    cudaError_t _e = cudaGetLastError();                         \
    if (_e != cudaSuccess) return ::q35::cuda_fail(_e, what);    \
  } while (0)

inline bool aligned16(const void *p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// ------------------------------------------------------------- device side
// Error-word codes written by kernels (never trap: a shared GPU must survive).
enum DevErrCode {
  DEV_ERR_WAIT_TIMEOUT = 1,  // a bounded mbarrier / flag wait ran out
  DEV_ERR_INDEX = 2,         // an index read from memory was out of range
  DEV_ERR_SCHEDULE = 3       // a tile schedule inconsistent with the offsets
};

__device__ __forceinline__ void report_error(int *err, int code, int site,
                                             int a, int b) {
  if (err == nullptr) return;
  if (atomicCAS(err, 0, code) == 0) {
    err[1] = site;
    err[2] = a;
    err[3] = b;
    __threadfence();
  }
}

__device__ __forceinline__ float bf2f(uint16_t v) {
  return __uint_as_float(static_cast<uint32_t>(v) << 16);
}
// Round-to-nearest-even fp32 -> bf16 (NaN kept quiet).
__device__ __forceinline__ uint16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}
__device__ __forceinline__ void unpack_bf2(uint32_t v, float &lo, float &hi) {
  lo = __uint_as_float(v << 16);
  hi = __uint_as_float(v & 0xffff0000u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

}  // namespace q35
