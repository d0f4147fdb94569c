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

// Two fp32 -> e4m3 bytes (lo in bits 0-7), round-to-nearest-even, saturating.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3));
}

// Eight bf16 of one 16-byte word as fp32 (exact: bf16 is the top half of fp32).
__device__ __forceinline__ void unpack_bf16x8(const uint4& raw, float (&f)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Two values that are already bf16 (exactly representable), packed losslessly.
__device__ __forceinline__ uint32_t pack_exact_bf16x2(float lo, float hi) {
  return (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xFFFF0000u);
}

// Two fp32 -> packed bf16x2 (lo in bits 0-15), round-to-nearest-even.
__device__ __forceinline__ uint32_t round_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Packed bf16x2 product, one rounding of the exact product: the same bits as
// rounding the fp32 product of the two bf16 values (which is exact) to bf16.
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Packed bf16x2 sum, one rounding of the exact sum.
__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Packed bf16x2 maximum (a NaN operand yields the other operand, as fmaxf).
__device__ __forceinline__ uint32_t max_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Rotate-half RoPE of 8 bf16 channels that sit on one side of the half
// split (x_base/x_base/operator/h3_partial_rope.py:9-29): with c = bf16(cos)
// and s = bf16(sin), out = bf16(bf16(x*c) + bf16(+-partner*s)), the partner
// negated for the first half. The products and the sum are bf16x2
// operations: the product of two bf16 values is exact in fp32, and so is the
// sum of two bf16 values unless the smaller is below 2^-15 of the larger
// (then rounding the fp32 sum and rounding the exact sum both return the
// larger), so one rounding of the exact result gives the bits of the fp32
// operation rounded to bf16. cw/sw hold c and s as packed bf16x2.
__device__ __forceinline__ void load_cos_sin8(const float* cs, const float* sn, uint32_t (&cw)[4],
                                              uint32_t (&sw)[4]) {
  const float4 c_lo = __ldg(reinterpret_cast<const float4*>(cs));
  const float4 c_hi = __ldg(reinterpret_cast<const float4*>(cs + 4));
  const float4 s_lo = __ldg(reinterpret_cast<const float4*>(sn));
  const float4 s_hi = __ldg(reinterpret_cast<const float4*>(sn + 4));
  cw[0] = round_bf16x2(c_lo.x, c_lo.y); cw[1] = round_bf16x2(c_lo.z, c_lo.w);
  cw[2] = round_bf16x2(c_hi.x, c_hi.y); cw[3] = round_bf16x2(c_hi.z, c_hi.w);
  sw[0] = round_bf16x2(s_lo.x, s_lo.y); sw[1] = round_bf16x2(s_lo.z, s_lo.w);
  sw[2] = round_bf16x2(s_hi.x, s_hi.y); sw[3] = round_bf16x2(s_hi.z, s_hi.w);
}

__device__ __forceinline__ uint4 rope8_bf16(const uint4& x, const uint4& partner, bool first,
                                            const uint32_t (&cw)[4], const uint32_t (&sw)[4]) {
  const uint32_t neg = first ? 0x80008000u : 0u;
  const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
  const uint32_t pw[4] = {partner.x ^ neg, partner.y ^ neg, partner.z ^ neg, partner.w ^ neg};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    o[k] = add_bf16x2(mul_bf16x2(xw[k], cw[k]), mul_bf16x2(pw[k], sw[k]));
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// The same with cos/sin read from the 8 fp32 entries at cs/sn (16-byte aligned).
__device__ __forceinline__ uint4 rope8_bf16(const uint4& x, const uint4& partner, bool first,
                                            const float* cs, const float* sn) {
  uint32_t cw[4], sw[4];
  load_cos_sin8(cs, sn, cw, sw);
  return rope8_bf16(x, partner, first, cw, sw);
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
