// Shared helpers for the xgen_b200 sm_100a kernels: status codes, launch
// checks and the exact-rounding conversions the H3 hot path relies on.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "../../include/xgb.h"

#define XGB_API extern "C" __attribute__((visibility("default")))

namespace xgb {

// Fails the call with XGB_ERR_LAUNCH when the last launch on this thread
// reported an error (bad configuration, missing sm_100a image, ...).
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? XGB_OK : XGB_ERR_LAUNCH;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float load_as_float(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float load_as_float(const __half* p) { return __half2float(*p); }

// fp32 -> e4m3 byte, round-to-nearest-even, saturating to +-448 (callers
// clamp first, as the reference kernels do, so saturation never decides).
__device__ __forceinline__ uint8_t f32_to_e4m3(float x) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
  return __half2float(__half(h));
}

// Block-wide reduction helpers (warp shuffles, then one shared slot per warp).
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace xgb
