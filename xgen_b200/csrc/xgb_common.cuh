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

// Unsigned division by a divisor fixed for a whole launch, as a multiply-high
// and shifts (T. Granlund, P. Montgomery, "Division by Invariant Integers
// using Multiplication", PLDI 1994): with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1, n / d = (t + ((n - t) >> 1)) >> (l - 1)
// where t = mulhi(n, m), for every 32-bit n (d = 1 is special-cased).
struct FastDiv {
  uint32_t d, m, l;
};
inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t l = 0;
  while (l < 32 && (uint64_t{1} << l) < d) ++l;
  const uint64_t m = ((uint64_t{1} << 32) * ((uint64_t{1} << l) - d)) / d + 1;
  return FastDiv{d, static_cast<uint32_t>(m), l};
}
__device__ __forceinline__ uint32_t fast_div(uint32_t n, FastDiv f) {
  if (f.l == 0) return n;
  const uint32_t t = __umulhi(n, f.m);
  return (t + ((n - t) >> 1)) >> (f.l - 1);
}

// a / b correctly rounded for a divisor shared by many quotients: with
// y = RN(1/b), q = RN(a*y) and the exact remainder r = a - b*q (one FMA),
// RN(q + r*y) is the correctly rounded quotient (Markstein's correction,
// P. Markstein, IBM J. Res. Dev. 34(1), 1990) for normal b and quotient.
__device__ __forceinline__ float div_by(float a, float b, float y) {
  const float q = __fmul_rn(a, y);
  const float r = __fmaf_rn(-q, b, a);
  return __fmaf_rn(r, y, q);
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
