// Shared helpers for the deepseeker_b200 CUDA library (sm_100a).
//
// Error model: every extern "C" entry point returns an int status (DS_OK on
// success) and records a human-readable message retrievable through
// ds_last_error_string().  No C++ exception crosses the ABI.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>

#include "deepseeker_b200.h"

namespace ds {

// Record an error message (thread-local) and return the status.
int set_error(int status, const char* fmt, ...);

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

int cuda_status(cudaError_t e, const char* what);

// Number of SMs of the current device (cached per device).
int sm_count();

}  // namespace ds

#define DS_CHECK_CUDA(expr)                                           \
  do {                                                                \
    cudaError_t _e = (expr);                                          \
    if (_e != cudaSuccess) return ds::cuda_status(_e, #expr);         \
  } while (0)

#define DS_CHECK_LAUNCH(what)                                         \
  do {                                                                \
    cudaError_t _e = cudaGetLastError();                              \
    if (_e != cudaSuccess) return ds::cuda_status(_e, what);          \
  } while (0)

#define DS_REQUIRE(cond, status, ...)                                 \
  do {                                                                \
    if (!(cond)) return ds::set_error((status), __VA_ARGS__);         \
  } while (0)

// ---------------------------------------------------------------------------
// Device-side numeric helpers shared by the dequant / GEMV kernels.

namespace ds {

// e2m1 code (4 bits) -> f32 value of the reference table:
// [0,.5,1,1.5,2,3,4,6, 0,-.5,-1,-1.5,-2,-3,-4,-6]; code 8 is +0.0 (not -0.0).
__device__ __forceinline__ float e2m1_value(uint32_t code) {
  const uint32_t m = code & 7u;
  uint32_t bits;
  if (m == 0u) {
    bits = 0u;                                   // codes 0 and 8 -> +0.0
  } else if (m == 1u) {
    bits = 0x3F000000u;                          // 0.5
  } else {
    bits = ((126u + (m >> 1)) << 23) | ((m & 1u) << 22);  // 1,1.5,2,3,4,6
  }
  if ((code & 8u) && m) bits |= 0x80000000u;
  return __uint_as_float(bits);
}

// ue8m0 byte -> 2^(b-127) as f32; b = 0 -> subnormal 2^-127; b = 0xFF -> NaN.
__device__ __forceinline__ float u8m0_value(uint32_t b) {
  if (b == 0xFFu) return __uint_as_float(0x7FC00000u);
  if (b == 0u) return __uint_as_float(0x00400000u);
  return __uint_as_float(b << 23);
}

}  // namespace ds
