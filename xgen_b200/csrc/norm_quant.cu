// Fused AdaLN prologue of the H3 block's FP8 GEMMs:
//
//   n   = norm(x)                       LayerNorm (no affine) or RMSNorm x weight,
//                                       fp32 statistics, rounded to bf16 once
//   h   = bf16(bf16(n * bf16(1 + scale[idx])) + shift[idx])      (modulation)
//   out = e4m3(h / s), s = max(amax(|h|)/448, FLT_MIN) per row    (per-token FP8)
//
// which is `norm1/norm2` + `_apply(..., modulation=True)`
// (x_base/x_base/operator/h3_indexed_affine.py:52-61, h3_npu_fusion.py:339-356)
// followed by the activation quantisation of the next FP8 Linear, in one HBM
// pass: read 2 B and write 1 B per element (+ an optional bf16 copy of h).
// One CTA per row; the row stays in registers between the passes. With no
// e4m3 output it is the final layer's output AdaLN, norm_out + modulation
// (x_diffusers/x_diffusers/framework/transformer/minimax_h3.py:672-696).
#include <cfloat>

#include "xgb_common.cuh"

namespace xgb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxPerThread = 24;  // width <= 256 * 24 = 6144

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) r += red[i];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) r = fmaxf(r, red[i]);
  __syncthreads();
  return r;
}

template <bool kRms>
__global__ void __launch_bounds__(kThreads) norm_modulate_quant_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, int width, int seq,
    const __nv_bfloat16* __restrict__ weight, float eps, const __nv_bfloat16* __restrict__ scale,
    int64_t lds, const __nv_bfloat16* __restrict__ shift, int64_t ldsh,
    const int64_t* __restrict__ idx, uint8_t* __restrict__ out, float* __restrict__ out_scale,
    __nv_bfloat16* __restrict__ out_bf16) {
  __shared__ float red[kThreads / 32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * ldx;
  float v[kMaxPerThread];
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxPerThread; ++j) {
    const int c = threadIdx.x + j * kThreads;
    v[j] = c < width ? __bfloat162float(xr[c]) : 0.f;
    s1 += v[j];
    s2 += v[j] * v[j];
  }
  float mean = 0.f, rstd;
  if constexpr (kRms) {
    rstd = rsqrtf(block_sum(s2, red) / width + eps);
  } else {
    mean = block_sum(s1, red) / width;
    float d2 = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxPerThread; ++j) {
      const int c = threadIdx.x + j * kThreads;
      const float d = c < width ? v[j] - mean : 0.f;
      d2 += d * d;
    }
    rstd = rsqrtf(block_sum(d2, red) / width + eps);
  }
  const int64_t t = idx[row % seq];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxPerThread; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < width) {
      float n = (v[j] - mean) * rstd;
      if (kRms && weight) n *= __bfloat162float(weight[c]);
      n = bf16_round(n);
      const float f = bf16_round(__fadd_rn(1.0f, __bfloat162float(scale[t * lds + c])));
      const float h = bf16_round(__fadd_rn(bf16_round(__fmul_rn(n, f)),
                                           __bfloat162float(shift[t * ldsh + c])));
      v[j] = h;
      amax = fmaxf(amax, fabsf(h));
    }
  }
  if (out_bf16) {
#pragma unroll
    for (int j = 0; j < kMaxPerThread; ++j) {
      const int c = threadIdx.x + j * kThreads;
      if (c < width) out_bf16[row * static_cast<int64_t>(width) + c] = __float2bfloat16_rn(v[j]);
    }
  }
  if (!out) return;  // modulation only (the final layer's output AdaLN)
  amax = block_max(amax, red);
  const float sc = fmaxf(__fdiv_rn(amax, 448.0f), FLT_MIN);
  if (threadIdx.x == 0) out_scale[row] = sc;
  uint8_t* orow = out + row * static_cast<int64_t>(width);
#pragma unroll
  for (int j = 0; j < kMaxPerThread; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < width) orow[c] = f32_to_e4m3(fminf(fmaxf(__fdiv_rn(v[j], sc), -448.f), 448.f));
  }
}

}  // namespace
}  // namespace xgb

using namespace xgb;

XGB_API int xgb_norm_modulate_quant(const void* x, int64_t ldx, int64_t rows, int64_t width,
                                    int64_t seq, int norm_kind, const void* weight, float eps,
                                    const void* scale, int64_t lds, const void* shift,
                                    int64_t ldsh, const int64_t* indices, uint8_t* out,
                                    float* out_scale, void* out_bf16, void* stream) {
  if (!x || !scale || !shift || !indices) return XGB_ERR_ARG;
  if ((out == nullptr) != (out_scale == nullptr) || (!out && !out_bf16)) return XGB_ERR_ARG;
  if (rows < 0 || width <= 0 || width > kThreads * kMaxPerThread || seq <= 0 || rows % seq)
    return XGB_ERR_SHAPE;
  if (ldx < width || lds < width || ldsh < width) return XGB_ERR_STRIDE;
  if (norm_kind != 0 && norm_kind != 1) return XGB_ERR_ARG;
  if (!(eps > 0.f)) return XGB_ERR_ARG;
  if (rows == 0) return XGB_OK;
  auto xb = static_cast<const __nv_bfloat16*>(x);
  auto wb = static_cast<const __nv_bfloat16*>(weight);
  auto sb = static_cast<const __nv_bfloat16*>(scale);
  auto hb = static_cast<const __nv_bfloat16*>(shift);
  auto ob = static_cast<__nv_bfloat16*>(out_bf16);
  cudaStream_t st = as_stream(stream);
  const unsigned grid = static_cast<unsigned>(rows);
  if (norm_kind == 1)
    norm_modulate_quant_kernel<true><<<grid, kThreads, 0, st>>>(
        xb, ldx, static_cast<int>(width), static_cast<int>(seq), wb, eps, sb, lds, hb, ldsh,
        indices, out, out_scale, ob);
  else
    norm_modulate_quant_kernel<false><<<grid, kThreads, 0, st>>>(
        xb, ldx, static_cast<int>(width), static_cast<int>(seq), wb, eps, sb, lds, hb, ldsh,
        indices, out, out_scale, ob);
  return launch_status();
}
