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
//
// Rows whose width, strides and pointers allow it take the vector kernel:
// 128 threads, each owning 8-channel chunks moved as 16-byte loads (bf16)
// and 8-byte stores (e4m3), the modulated row kept as packed bf16 between
// the amax reduction and the quantisation, and the per-element division by
// the row scale done as a Markstein-corrected reciprocal multiply (the same
// correctly rounded quotient as a division). Other layouts take the scalar
// kernel, which computes the same values.
#include <cfloat>
#include <type_traits>

#include "xgb_common.cuh"

namespace xgb {
namespace {

constexpr int kVecThreads = 128;
constexpr int kVecMaxChunks = 6;  // 8-channel chunks per thread: width <= 128 * 6 * 8 = 6144

template <bool kMax>
__device__ __forceinline__ float reduce128(float v, float* red) {
  v = kMax ? warp_max(v) : warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  const float r = kMax ? fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]))
                       : (red[0] + red[1]) + (red[2] + red[3]);
  __syncthreads();
  return r;
}

// kVecChunks = ceil(width / 1024) chunks per thread, so narrow rows hold
// fewer registers and more rows are in flight per SM.
template <bool kRms, int kVecChunks>
__global__ void __launch_bounds__(kVecThreads) norm_modulate_quant_vec_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, int width, int seq,
    const __nv_bfloat16* __restrict__ weight, float eps, const __nv_bfloat16* __restrict__ scale,
    int64_t lds, const __nv_bfloat16* __restrict__ shift, int64_t ldsh,
    const int64_t* __restrict__ idx, uint8_t* __restrict__ out, float* __restrict__ out_scale,
    __nv_bfloat16* __restrict__ out_bf16) {
  __shared__ float red[kVecThreads / 32];
  const int64_t row = blockIdx.x;
  const int chunks = width >> 3;
  const __nv_bfloat16* xr = x + row * ldx;
  uint4 raw[kVecChunks];
#pragma unroll
  for (int j = 0; j < kVecChunks; ++j) {
    const int c = threadIdx.x + j * kVecThreads;
    raw[j] = c < chunks ? __ldg(reinterpret_cast<const uint4*>(xr) + c) : make_uint4(0, 0, 0, 0);
  }
  const int64_t t = idx[row % seq];
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < kVecChunks; ++j) {
    float f[8];
    unpack_bf16x8(raw[j], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc = kRms ? fmaf(f[e], f[e], acc) : acc + f[e];
  }
  float mean = 0.f, rstd;
  if constexpr (kRms) {
    rstd = rsqrtf(reduce128<false>(acc, red) / width + eps);
  } else {
    mean = reduce128<false>(acc, red) / width;
    float d2 = 0.f;
#pragma unroll
    for (int j = 0; j < kVecChunks; ++j) {
      if (threadIdx.x + j * kVecThreads < chunks) {
        float f[8];
        unpack_bf16x8(raw[j], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float d = f[e] - mean;
          d2 = fmaf(d, d, d2);
        }
      }
    }
    rstd = rsqrtf(reduce128<false>(d2, red) / width + eps);
  }
  // Modulation on packed bf16x2: m = bf16(1 + scale), h = bf16(bf16(n*m) + shift).
  // With bf16 operands the product is exact in fp32 and the sum is exact in
  // fp32 unless the smaller operand is below 2^-15 of the larger (then both
  // roundings return the larger), so the single-rounding bf16x2 operations
  // give the bits of the fp32 operation rounded to bf16.
  uint32_t amax2 = 0;  // bf16x2 max of |h|
  const uint4* sc4 = reinterpret_cast<const uint4*>(scale + t * lds);
  const uint4* sh4 = reinterpret_cast<const uint4*>(shift + t * ldsh);
#pragma unroll
  for (int j = 0; j < kVecChunks; ++j) {
    const int c = threadIdx.x + j * kVecThreads;
    if (c < chunks) {
      float f[8], w[8];
      unpack_bf16x8(raw[j], f);
      const uint4 sc = __ldg(sc4 + c), sh = __ldg(sh4 + c);
      if (kRms && weight) unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(weight) + c), w);
      const uint32_t scw[4] = {sc.x, sc.y, sc.z, sc.w}, shw[4] = {sh.x, sh.y, sh.z, sh.w};
      uint32_t h2[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float n0 = (f[2 * k] - mean) * rstd, n1 = (f[2 * k + 1] - mean) * rstd;
        if (kRms && weight) {
          n0 *= w[2 * k];
          n1 *= w[2 * k + 1];
        }
        const uint32_t m2 = add_bf16x2(0x3F803F80u /* (1, 1) */, scw[k]);
        h2[k] = add_bf16x2(mul_bf16x2(round_bf16x2(n0, n1), m2), shw[k]);
        amax2 = max_bf16x2(amax2, h2[k] & 0x7FFF7FFFu);
      }
      raw[j] = make_uint4(h2[0], h2[1], h2[2], h2[3]);
      if (out_bf16) reinterpret_cast<uint4*>(out_bf16 + row * static_cast<int64_t>(width))[c] = raw[j];
    }
  }
  float amax = fmaxf(__uint_as_float(amax2 << 16), __uint_as_float(amax2 & 0xFFFF0000u));
  if (!out) return;  // modulation only (the final layer's output AdaLN)
  amax = reduce128<true>(amax, red);
  const float s = fmaxf(__fdiv_rn(amax, 448.0f), FLT_MIN);
  const float y = __frcp_rn(s);
  if (threadIdx.x == 0) out_scale[row] = s;
  uint2* orow = reinterpret_cast<uint2*>(out + row * static_cast<int64_t>(width));
#pragma unroll
  for (int j = 0; j < kVecChunks; ++j) {
    const int c = threadIdx.x + j * kVecThreads;
    if (c < chunks) {
      float h[8];
      unpack_bf16x8(raw[j], h);
      uint32_t q[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2)
        q[e / 2] = e4m3x2(fminf(fmaxf(div_by(h[e], s, y), -448.f), 448.f),
                          fminf(fmaxf(div_by(h[e + 1], s, y), -448.f), 448.f));
      orow[c] = make_uint2(q[0] | (q[1] << 16), q[2] | (q[3] << 16));
    }
  }
}

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
  const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec = width % 8 == 0 && width <= kVecThreads * kVecMaxChunks * 8 && ldx % 8 == 0 &&
                   lds % 8 == 0 && ldsh % 8 == 0 && a16(x) && a16(scale) && a16(shift) &&
                   (!weight || a16(weight)) && (!out_bf16 || a16(out_bf16)) &&
                   (reinterpret_cast<uintptr_t>(out) & 7u) == 0;
  if (vec) {
    const int per_thread = static_cast<int>(cdiv(width / 8, kVecThreads));
    auto run = [&](auto rms, auto chunks) {
      norm_modulate_quant_vec_kernel<decltype(rms)::value, decltype(chunks)::value>
          <<<grid, kVecThreads, 0, st>>>(xb, ldx, static_cast<int>(width), static_cast<int>(seq), wb,
                                         eps, sb, lds, hb, ldsh, indices, out, out_scale, ob);
    };
    auto pick = [&](auto rms) {
      if (per_thread <= 2) run(rms, std::integral_constant<int, 2>{});
      else if (per_thread <= 3) run(rms, std::integral_constant<int, 3>{});
      else if (per_thread <= 4) run(rms, std::integral_constant<int, 4>{});
      else run(rms, std::integral_constant<int, kVecMaxChunks>{});
    };
    if (norm_kind == 1) pick(std::true_type{});
    else pick(std::false_type{});
    return launch_status();
  }
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
