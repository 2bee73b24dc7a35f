// Shared definitions for the swvr_b200 CUDA library (host and device).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/swvr_b200.h"

namespace swvr {

constexpr int kNumSMsB200 = 148;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Device error codes written to g_device_error by bounded waits (0 = none).
// The low byte names the kernel, the next byte the wait site.
enum : uint32_t {
  kErrFwd = 0x100,
  kErrBwdScores = 0x200,
  kErrGemm = 0x300,
  kErrSelftest = 0x7F00,  // swvr_selftest_wait_timeout
};

inline size_t dtype_size(int dt) {
  switch (dt) {
    case SWVR_F32: return 4;
    case SWVR_F64: return 8;
    case SWVR_BF16: return 2;
    case SWVR_F16: return 2;
    default: return 0;
  }
}

// Load one element of a runtime-typed array as float / double.
__device__ __forceinline__ float load_f(const void* p, int dt, int64_t i) {
  switch (dt) {
    case SWVR_F32: return static_cast<const float*>(p)[i];
    case SWVR_F64: return static_cast<float>(static_cast<const double*>(p)[i]);
    case SWVR_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    default: return __half2float(static_cast<const __half*>(p)[i]);
  }
}

__device__ __forceinline__ double load_d(const void* p, int dt, int64_t i) {
  switch (dt) {
    case SWVR_F32: return static_cast<const float*>(p)[i];
    case SWVR_F64: return static_cast<const double*>(p)[i];
    case SWVR_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    default: return __half2float(static_cast<const __half*>(p)[i]);
  }
}

__device__ __forceinline__ void store_f(void* p, int dt, int64_t i, float v) {
  switch (dt) {
    case SWVR_F32: static_cast<float*>(p)[i] = v; break;
    case SWVR_F64: static_cast<double*>(p)[i] = v; break;
    case SWVR_BF16: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    default: static_cast<__half*>(p)[i] = __float2half_rn(v); break;
  }
}

__device__ __forceinline__ void store_d(void* p, int dt, int64_t i, double v) {
  switch (dt) {
    case SWVR_F32: static_cast<float*>(p)[i] = static_cast<float>(v); break;
    case SWVR_F64: static_cast<double*>(p)[i] = v; break;
    case SWVR_BF16: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(static_cast<float>(v)); break;
    default: static_cast<__half*>(p)[i] = __float2half_rn(static_cast<float>(v)); break;
  }
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }
inline size_t align_up(size_t a, size_t b) { return (a + b - 1) / b * b; }

}  // namespace swvr
