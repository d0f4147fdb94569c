// HBM-bound elementwise operators of the H3 block, bit-exact with the
// reference Triton kernels (which run with enable_fp_fusion=False, i.e. no
// FMA contraction and an explicit bf16 rounding after every eager op).
//
//   partial RoPE        x_base/x_base/operator/h3_partial_rope.py:9-29
//   Q/K RMSNorm (+RoPE) x_base/x_base/operator/h3_qk_rms.py:9-45
//   indexed affine      x_base/x_base/operator/h3_indexed_affine.py:9-30
//   gate-first SwiGLU   x_base/x_base/operator/h3_swiglu.py:15-29
//
// All products/sums below use __fmul_rn/__fadd_rn so nvcc cannot contract
// them into FMAs, which would change the rounding the reference pins.
#include "xgb_common.cuh"

namespace xgb {
namespace {

constexpr int kThreads = 256;

struct Bf16x8 {
  __nv_bfloat16 v[8];
};

__device__ __forceinline__ Bf16x8 load8(const __nv_bfloat16* p) {
  Bf16x8 r;
  *reinterpret_cast<uint4*>(r.v) = __ldg(reinterpret_cast<const uint4*>(p));
  return r;
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const Bf16x8& r) {
  *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(r.v);
}

// One rotate-half RoPE channel with the reference's rounding sequence:
// left = bf16(x*bf16(cos)), right = bf16(+-partner*bf16(sin)), out = left+right.
__device__ __forceinline__ float rope_channel(float x, float partner, bool first, float c, float s) {
  const float cb = bf16_round(c);
  const float sb = bf16_round(s);
  const float left = bf16_round(__fmul_rn(x, cb));
  const float right = bf16_round(__fmul_rn(first ? -partner : partner, sb));
  return __fadd_rn(left, right);
}

// ---------------------------------------------------------------- RoPE
// Vector path: 8 channels per thread; requires width % 8 == 0 and
// (rotary / 2) % 8 == 0 so a vector never straddles the rotary boundary or
// the half split, and its partner vector is 16-byte aligned. Thread u owns
// chunk u of 8 channels; its (row, channel, position) come from 32-bit
// invariant divisions.
__global__ void __launch_bounds__(kThreads) partial_rope_vec_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const float* __restrict__ cos, const float* __restrict__ sin, __nv_bfloat16* __restrict__ qo,
    __nv_bfloat16* __restrict__ ko, uint32_t chunks, FastDiv div_cpr, FastDiv div_heads,
    FastDiv div_seq, int rotary) {
  const bool is_key = blockIdx.y == 1;
  const __nv_bfloat16* src = is_key ? k : q;
  __nv_bfloat16* dst = is_key ? ko : qo;
  const uint32_t u = blockIdx.x * kThreads + threadIdx.x;
  if (u >= chunks) return;
  const uint32_t row = fast_div(u, div_cpr);
  const int ch = static_cast<int>(u - row * div_cpr.d) * 8;
  const int64_t e = static_cast<int64_t>(u) * 8;
  uint4 x = __ldg(reinterpret_cast<const uint4*>(src + e));
  if (ch < rotary) {
    const int half = rotary / 2;
    const bool first = ch < half;
    const uint32_t bs = fast_div(row, div_heads);  // batch * seq + s
    const uint32_t s = bs - fast_div(bs, div_seq) * div_seq.d;
    const uint4 p = __ldg(reinterpret_cast<const uint4*>(src + e + (first ? half : -half)));
    x = rope8_bf16(x, p, first, cos + static_cast<int64_t>(s) * rotary + ch,
                   sin + static_cast<int64_t>(s) * rotary + ch);
  }
  *reinterpret_cast<uint4*>(dst + e) = x;
}

// Scalar path for any even rotary <= width.
__global__ void __launch_bounds__(kThreads) partial_rope_scalar_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const float* __restrict__ cos, const float* __restrict__ sin, __nv_bfloat16* __restrict__ qo,
    __nv_bfloat16* __restrict__ ko, int64_t n, int64_t seq, int64_t heads, int64_t width,
    int64_t rotary) {
  const bool is_key = blockIdx.y == 1;
  const __nv_bfloat16* src = is_key ? k : q;
  __nv_bfloat16* dst = is_key ? ko : qo;
  const int64_t e = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (e >= n) return;
  const int64_t ch = e % width;
  const float x = __bfloat162float(src[e]);
  float r = x;
  if (ch < rotary) {
    const int64_t half = rotary / 2;
    const bool first = ch < half;
    const int64_t s = (e / (heads * width)) % seq;
    const float p = __bfloat162float(src[e + (first ? half : -half)]);
    r = rope_channel(x, p, first, cos[s * rotary + ch], sin[s * rotary + ch]);
  }
  dst[e] = __float2bfloat16_rn(r);
}

// ---------------------------------------------------------------- QK RMS
// One warp per (batch, seq, head) row; lane l owns channels l, l+32, ...
constexpr int kRmsMaxPerLane = 8;  // width <= 256

__global__ void __launch_bounds__(kThreads) qk_rms_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
    __nv_bfloat16* __restrict__ qo, __nv_bfloat16* __restrict__ ko, const float* __restrict__ cos,
    const float* __restrict__ sin, int64_t rows, int64_t seq, int64_t heads, int width,
    int64_t qsb, int64_t qss, int64_t qsh, int64_t ksb, int64_t kss, int64_t ksh, float q_eps,
    float k_eps, int rotary) {
  const bool is_key = blockIdx.y == 1;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t b = row / (seq * heads);
  const int64_t s = (row / heads) % seq;
  const int64_t h = row % heads;
  const __nv_bfloat16* src =
      is_key ? k + b * ksb + s * kss + h * ksh : q + b * qsb + s * qss + h * qsh;
  const __nv_bfloat16* w = is_key ? kw : qw;
  __nv_bfloat16* dst = (is_key ? ko : qo) + row * width;
  const float eps = is_key ? k_eps : q_eps;

  float val[kRmsMaxPerLane];
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < kRmsMaxPerLane; ++j) {
    const int c = lane + 32 * j;
    val[j] = c < width ? __bfloat162float(src[c]) : 0.f;
    sq = __fadd_rn(sq, __fmul_rn(val[j], val[j]));
  }
  sq = warp_sum(sq);
  const float scale = rsqrtf(__fadd_rn(__fdiv_rn(sq, static_cast<float>(width)), eps));
#pragma unroll
  for (int j = 0; j < kRmsMaxPerLane; ++j) {
    const int c = lane + 32 * j;
    if (c >= width) continue;
    const float normed = __fmul_rn(__fmul_rn(val[j], scale), __bfloat162float(w[c]));
    float out = normed;  // stored as bf16 below
    if (c < rotary) {
      const int half = rotary / 2;
      const bool first = c < half;
      const int pc = first ? c + half : c - half;
      const float partner =
          bf16_round(__fmul_rn(__fmul_rn(__bfloat162float(src[pc]), scale), __bfloat162float(w[pc])));
      out = rope_channel(bf16_round(normed), partner, first, cos[s * rotary + c], sin[s * rotary + c]);
    }
    dst[c] = __float2bfloat16_rn(out);
  }
}

// Vector path: width % 8 == 0, rotary % 16 == 0, 8-element strides and
// 16-byte aligned pointers. A group of G = next_pow2(width / 8) lanes owns a
// row, each lane 8 contiguous channels moved as one 16-byte load/store; the
// normalised partner channels of the RoPE come from the partner lane by a
// shuffle. Same arithmetic as qk_rms_kernel except the order of the fp32
// sum of squares.
struct RmsStrides {
  int64_t b, s, h;
};

__global__ void __launch_bounds__(kThreads) qk_rms_vec_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
    __nv_bfloat16* __restrict__ qo, __nv_bfloat16* __restrict__ ko, const float* __restrict__ cos,
    const float* __restrict__ sin, uint32_t rows, FastDiv div_heads, FastDiv div_seq, int width,
    int group, RmsStrides qs, RmsStrides ks, float q_eps, float k_eps, int rotary) {
  const bool is_key = blockIdx.y == 1;
  const int lane = threadIdx.x & 31;
  const int sub = lane & (group - 1);
  const uint32_t row = (blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5)) * (32 / group) + lane / group;
  const bool live = row < rows;
  const uint32_t r = live ? row : 0u;
  const uint32_t bs = fast_div(r, div_heads);
  const uint32_t h = r - bs * div_heads.d;
  const uint32_t b = fast_div(bs, div_seq);
  const uint32_t s = bs - b * div_seq.d;
  const RmsStrides st = is_key ? ks : qs;
  const __nv_bfloat16* src = (is_key ? k : q) + b * st.b + s * st.s + h * st.h;
  const int c0 = sub * 8;
  const bool has = live && c0 < width;
  float v[8];
  unpack_bf16x8(has ? __ldg(reinterpret_cast<const uint4*>(src + c0)) : make_uint4(0, 0, 0, 0), v);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) sq = __fadd_rn(sq, __fmul_rn(v[i], v[i]));
  for (int o = group / 2; o > 0; o >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
  const float scale =
      rsqrtf(__fadd_rn(__fdiv_rn(sq, static_cast<float>(width)), is_key ? k_eps : q_eps));
  float w[8];
  unpack_bf16x8(has ? __ldg(reinterpret_cast<const uint4*>((is_key ? kw : qw) + c0)) : make_uint4(0, 0, 0, 0), w);
  uint32_t nw[4];
#pragma unroll
  for (int i = 0; i < 8; i += 2)
    nw[i / 2] = round_bf16x2(__fmul_rn(__fmul_rn(v[i], scale), w[i]),
                             __fmul_rn(__fmul_rn(v[i + 1], scale), w[i + 1]));
  uint4 out = make_uint4(nw[0], nw[1], nw[2], nw[3]);
  if (rotary > 0) {
    const int half = rotary / 2;
    const bool first = c0 < half;
    const int psub = c0 >= rotary ? sub : (first ? sub + half / 8 : sub - half / 8);
    const int src_lane = (lane & ~(group - 1)) | psub;
    uint32_t pw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pw[i] = __shfl_sync(0xffffffffu, nw[i], src_lane);
    if (has && c0 < rotary)
      out = rope8_bf16(out, make_uint4(pw[0], pw[1], pw[2], pw[3]), first,
                       cos + static_cast<int64_t>(s) * rotary + c0, sin + static_cast<int64_t>(s) * rotary + c0);
  }
  if (has)
    *reinterpret_cast<uint4*>((is_key ? ko : qo) + static_cast<int64_t>(row) * width + c0) = out;
}

// ---------------------------------------------------------------- indexed affine
template <bool kModulation, bool kVec>
__global__ void __launch_bounds__(kThreads) indexed_affine_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ table,
    const __nv_bfloat16* __restrict__ addend, const int64_t* __restrict__ indices,
    __nv_bfloat16* __restrict__ out, int64_t n, int64_t width, int64_t seq, int64_t table_stride,
    int64_t addend_stride) {
  constexpr int kVecN = kVec ? 8 : 1;
  const int64_t e = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) * kVecN;
  if (e >= n) return;
  const int64_t ch = e % width;
  const int64_t row = indices[(e / width) % seq];
  const __nv_bfloat16* tp = table + row * table_stride + ch;
  const __nv_bfloat16* ap = kModulation ? addend + row * addend_stride + ch : addend + e;
  if constexpr (kVec) {
    const Bf16x8 xv = load8(x + e), tv = load8(tp), av = load8(ap);
    Bf16x8 o;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float f = __bfloat162float(tv.v[i]);
      if (kModulation) f = bf16_round(__fadd_rn(1.0f, f));
      const float prod = bf16_round(__fmul_rn(__bfloat162float(xv.v[i]), f));
      o.v[i] = __float2bfloat16_rn(__fadd_rn(prod, __bfloat162float(av.v[i])));
    }
    store8(out + e, o);
  } else {
    float f = __bfloat162float(*tp);
    if (kModulation) f = bf16_round(__fadd_rn(1.0f, f));
    const float prod = bf16_round(__fmul_rn(__bfloat162float(x[e]), f));
    out[e] = __float2bfloat16_rn(__fadd_rn(prod, __bfloat162float(*ap)));
  }
}

// ---------------------------------------------------------------- SwiGLU
__device__ __forceinline__ float swiglu_one(float g, float v) {
  const float act = bf16_round(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))));
  return bf16_round(__fmul_rn(act, v));
}

template <bool kVec>
__global__ void __launch_bounds__(kThreads) swiglu_kernel(const __nv_bfloat16* __restrict__ x,
                                                          __nv_bfloat16* __restrict__ out,
                                                          int64_t n, int64_t width,
                                                          float* __restrict__ amax) {
  constexpr int kVecN = kVec ? 8 : 1;
  const int64_t e = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) * kVecN;
  float peak = 0.f;
  if (e < n) {
    const int64_t src = e + (e / width) * width;
    if constexpr (kVec) {
      const Bf16x8 g = load8(x + src), v = load8(x + src + width);
      Bf16x8 o;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float r = swiglu_one(__bfloat162float(g.v[i]), __bfloat162float(v.v[i]));
        o.v[i] = __float2bfloat16_rn(r);
        peak = (isnan(r) || isnan(peak)) ? __int_as_float(0x7fc00000) : fmaxf(peak, fabsf(r));
      }
      store8(out + e, o);
    } else {
      const float r = swiglu_one(__bfloat162float(x[src]), __bfloat162float(x[src + width]));
      out[e] = __float2bfloat16_rn(r);
      peak = isnan(r) ? r : fabsf(r);
    }
  }
  if (amax != nullptr) {
    // Warp-level NaN-aware reduction on the integer image, then one atomic.
    int bits = __float_as_int(fabsf(peak));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) bits = max(bits, __shfl_xor_sync(0xffffffffu, bits, o));
    if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<int*>(amax), bits);
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace xgb

using namespace xgb;

XGB_API int xgb_partial_rope(const void* q, const void* k, const float* cos, const float* sin,
                             void* q_out, void* k_out, int64_t batch, int64_t seq, int64_t heads,
                             int64_t width, int64_t rotary, void* stream) {
  if (!q || !k || !cos || !sin || !q_out || !k_out) return XGB_ERR_ARG;
  if (batch < 0 || seq < 0 || heads < 0 || width <= 0) return XGB_ERR_SHAPE;
  if (rotary <= 0 || rotary % 2 || rotary > width) return XGB_ERR_SHAPE;
  const int64_t n = batch * seq * heads * width;
  if (n == 0) return XGB_OK;
  const bool vec = width % 8 == 0 && (rotary / 2) % 8 == 0 && aligned16(q) && aligned16(k) &&
                   aligned16(q_out) && aligned16(k_out) && aligned16(cos) && aligned16(sin) &&
                   n / 8 <= UINT32_MAX && batch * seq <= UINT32_MAX;
  cudaStream_t st = as_stream(stream);
  auto qb = static_cast<const __nv_bfloat16*>(q);
  auto kb = static_cast<const __nv_bfloat16*>(k);
  auto qo = static_cast<__nv_bfloat16*>(q_out);
  auto ko = static_cast<__nv_bfloat16*>(k_out);
  if (vec) {
    dim3 grid(static_cast<unsigned>(cdiv(n / 8, kThreads)), 2);
    partial_rope_vec_kernel<<<grid, kThreads, 0, st>>>(
        qb, kb, cos, sin, qo, ko, static_cast<uint32_t>(n / 8),
        make_fastdiv(static_cast<uint32_t>(width / 8)), make_fastdiv(static_cast<uint32_t>(heads)),
        make_fastdiv(static_cast<uint32_t>(seq)), static_cast<int>(rotary));
  } else {
    dim3 grid(static_cast<unsigned>(cdiv(n, kThreads)), 2);
    partial_rope_scalar_kernel<<<grid, kThreads, 0, st>>>(qb, kb, cos, sin, qo, ko, n, seq, heads,
                                                          width, rotary);
  }
  return launch_status();
}

XGB_API int xgb_qk_rms(const void* q, const int64_t* q_strides, const void* k,
                       const int64_t* k_strides, const void* q_weight, const void* k_weight,
                       float q_eps, float k_eps, const float* cos, const float* sin,
                       int64_t rotary, void* q_out, void* k_out, int64_t batch, int64_t seq,
                       int64_t heads, int64_t width, void* stream) {
  if (!q || !k || !q_strides || !k_strides || !q_weight || !k_weight || !q_out || !k_out)
    return XGB_ERR_ARG;
  if (batch < 0 || seq < 0 || heads < 0 || width <= 0 || width > 32 * kRmsMaxPerLane)
    return XGB_ERR_SHAPE;
  if (rotary < 0 || rotary % 2 || rotary > width) return XGB_ERR_SHAPE;
  if (rotary > 0 && (!cos || !sin)) return XGB_ERR_ARG;
  const int64_t rows = batch * seq * heads;
  if (rows == 0) return XGB_OK;
  bool vec = width % 8 == 0 && rotary % 16 == 0 && rows <= UINT32_MAX && aligned16(q) &&
             aligned16(k) && aligned16(q_weight) && aligned16(k_weight) && aligned16(q_out) &&
             aligned16(k_out) && (rotary == 0 || (aligned16(cos) && aligned16(sin)));
  for (int d = 0; d < 3; ++d) vec = vec && q_strides[d] % 8 == 0 && k_strides[d] % 8 == 0;
  if (vec) {
    int group = 1;
    while (group < width / 8) group <<= 1;
    const int64_t rows_per_block = (kThreads / 32) * (32 / group);
    dim3 grid(static_cast<unsigned>(cdiv(rows, rows_per_block)), 2);
    qk_rms_vec_kernel<<<grid, kThreads, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
        static_cast<const __nv_bfloat16*>(q_weight), static_cast<const __nv_bfloat16*>(k_weight),
        static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_out), cos, sin,
        static_cast<uint32_t>(rows), make_fastdiv(static_cast<uint32_t>(heads)),
        make_fastdiv(static_cast<uint32_t>(seq)), static_cast<int>(width), group,
        RmsStrides{q_strides[0], q_strides[1], q_strides[2]},
        RmsStrides{k_strides[0], k_strides[1], k_strides[2]}, q_eps, k_eps, static_cast<int>(rotary));
    return launch_status();
  }
  dim3 grid(static_cast<unsigned>(cdiv(rows, kThreads / 32)), 2);
  qk_rms_kernel<<<grid, kThreads, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
      static_cast<const __nv_bfloat16*>(q_weight), static_cast<const __nv_bfloat16*>(k_weight),
      static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_out), cos, sin, rows, seq,
      heads, static_cast<int>(width), q_strides[0], q_strides[1], q_strides[2], k_strides[0],
      k_strides[1], k_strides[2], q_eps, k_eps, static_cast<int>(rotary));
  return launch_status();
}

XGB_API int xgb_indexed_affine(const void* x, const void* table, int64_t table_stride,
                               const void* addend, int64_t addend_stride,
                               const int64_t* indices, void* out, int64_t batch, int64_t seq,
                               int64_t width, int modulation, void* stream) {
  if (!x || !table || !addend || !indices || !out) return XGB_ERR_ARG;
  if (batch < 0 || seq < 0 || width <= 0) return XGB_ERR_SHAPE;
  const int64_t n = batch * seq * width;
  if (n == 0) return XGB_OK;
  const bool vec = width % 8 == 0 && table_stride % 8 == 0 &&
                   (!modulation || addend_stride % 8 == 0) && aligned16(x) && aligned16(table) &&
                   aligned16(addend) && aligned16(out);
  auto xb = static_cast<const __nv_bfloat16*>(x);
  auto tb = static_cast<const __nv_bfloat16*>(table);
  auto ab = static_cast<const __nv_bfloat16*>(addend);
  auto ob = static_cast<__nv_bfloat16*>(out);
  cudaStream_t st = as_stream(stream);
  const unsigned grid = static_cast<unsigned>(cdiv(vec ? n / 8 : n, kThreads));
  if (modulation) {
    if (vec)
      indexed_affine_kernel<true, true><<<grid, kThreads, 0, st>>>(xb, tb, ab, indices, ob, n, width, seq, table_stride, addend_stride);
    else
      indexed_affine_kernel<true, false><<<grid, kThreads, 0, st>>>(xb, tb, ab, indices, ob, n, width, seq, table_stride, addend_stride);
  } else {
    if (vec)
      indexed_affine_kernel<false, true><<<grid, kThreads, 0, st>>>(xb, tb, ab, indices, ob, n, width, seq, table_stride, addend_stride);
    else
      indexed_affine_kernel<false, false><<<grid, kThreads, 0, st>>>(xb, tb, ab, indices, ob, n, width, seq, table_stride, addend_stride);
  }
  return launch_status();
}

XGB_API int xgb_swiglu(const void* x, void* out, int64_t rows, int64_t width, float* amax_out,
                       void* stream) {
  if (!x || !out) return XGB_ERR_ARG;
  if (rows < 0 || width <= 0) return XGB_ERR_SHAPE;
  const int64_t n = rows * width;
  if (n == 0) return XGB_OK;
  const bool vec = width % 8 == 0 && aligned16(x) && aligned16(out);
  auto xb = static_cast<const __nv_bfloat16*>(x);
  auto ob = static_cast<__nv_bfloat16*>(out);
  cudaStream_t st = as_stream(stream);
  const unsigned grid = static_cast<unsigned>(cdiv(vec ? n / 8 : n, kThreads));
  if (vec)
    swiglu_kernel<true><<<grid, kThreads, 0, st>>>(xb, ob, n, width, amax_out);
  else
    swiglu_kernel<false><<<grid, kThreads, 0, st>>>(xb, ob, n, width, amax_out);
  return launch_status();
}
