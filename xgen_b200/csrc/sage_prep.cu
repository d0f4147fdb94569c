// Sage-style quantisation of post-A2A Q/K/V ahead of the tcgen05 attention
// (the step `sageattn` performs internally on the reference's CUDA path,
// x_base/x_base/operator/attention.py:363-375; algorithm from SageAttention2,
// Zhang et al. 2024, with the block sizes of BASELINE config 3):
//
//   Q: x * sm_scale * log2(e), per 64-token block INT8, scale = amax/127
//   K: x - mean_seq(K) (per head and channel), per 64-token block INT8
//   V: per-channel e4m3, scale[c] = max(amax_seq(|V[:,c]|)/448, FLT_MIN)
//
// Output layout (the attention kernel's TMA source): [B*H][S_pad][128] with
// S_pad = roundup(S, 128); rows >= S are zero. Scales fp32: q/k
// [B*H][S_pad/64], v [B*H][128].
//
// Three launches: per-chunk K sums and V abs-max (partials in the caller's
// workspace), a per-head finalize (mean, V scale), and the block quantiser.
#include <cfloat>

#include "xgb_common.cuh"

namespace xgb {
namespace {

constexpr int kD = 128;
constexpr int kStatsRows = 512;  // rows per stats CTA
constexpr int kThreads = 256;
constexpr float kLog2e = 1.4426950408889634f;

template <typename T>
__device__ __forceinline__ float tf(T v);
template <>
__device__ __forceinline__ float tf<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float tf<__half>(__half v) { return __half2float(v); }

struct Strides {
  int64_t b, h, s;  // element strides; channel stride is 1
};

// Workspace: ksum partials [BH][chunks][128] fp32, vmax [BH][128] int,
// kmean [BH][128] fp32.
struct Workspace {
  float* ksum;
  int* vmax;
  float* kmean;
};

inline int64_t stats_chunks(int64_t seq) { return (seq + kStatsRows - 1) / kStatsRows; }

inline Workspace carve(void* ws, int64_t bh, int64_t chunks) {
  char* p = static_cast<char*>(ws);
  Workspace w;
  w.ksum = reinterpret_cast<float*>(p);
  p += bh * chunks * kD * sizeof(float);
  w.vmax = reinterpret_cast<int*>(p);
  p += bh * kD * sizeof(int);
  w.kmean = reinterpret_cast<float*>(p);
  return w;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) stats_kernel(const T* __restrict__ k, Strides ks,
                                                         const T* __restrict__ v, Strides vs,
                                                         int64_t heads, int64_t seq,
                                                         Workspace w, int64_t chunks) {
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / heads, h = bh % heads;
  const int c = threadIdx.x % kD;
  const int r0 = threadIdx.x / kD;  // 0 or 1
  const int64_t row_begin = static_cast<int64_t>(blockIdx.x) * kStatsRows;
  const int64_t row_end = min(row_begin + kStatsRows, seq);
  const T* kp = k + b * ks.b + h * ks.h + c;
  const T* vp = v + b * vs.b + h * vs.h + c;
  float sum = 0.f;
  int vmax = 0;
  for (int64_t r = row_begin + r0; r < row_end; r += 2) {
    sum += tf<T>(kp[r * ks.s]);
    vmax = max(vmax, __float_as_int(fabsf(tf<T>(vp[r * vs.s]))));
  }
  __shared__ float part[kThreads];
  part[threadIdx.x] = sum;
  __syncthreads();
  if (r0 == 0) {
    w.ksum[(bh * chunks + blockIdx.x) * kD + c] = part[c] + part[c + kD];
  }
  atomicMax(&w.vmax[bh * kD + c], vmax);
}

__global__ void __launch_bounds__(kD) finalize_kernel(Workspace w, int64_t chunks, int64_t seq,
                                                      float* __restrict__ v_scale) {
  const int64_t bh = blockIdx.x;
  const int c = threadIdx.x;
  float sum = 0.f;
  for (int64_t i = 0; i < chunks; ++i) sum += w.ksum[(bh * chunks + i) * kD + c];
  w.kmean[bh * kD + c] = __fdiv_rn(sum, static_cast<float>(seq));
  const float s = __fdiv_rn(__int_as_float(w.vmax[bh * kD + c]), 448.0f);
  v_scale[bh * kD + c] = fmaxf(s, FLT_MIN);
}

// One CTA per (64-row block, head); thread t owns channels 8*(t%16)..+8 of
// rows t/16 + 16*i, i < 4.
template <typename T>
__global__ void __launch_bounds__(kThreads) quant_kernel(
    const T* __restrict__ q, Strides qs, const T* __restrict__ k, Strides ks,
    const T* __restrict__ v, Strides vs, int64_t heads, int64_t seq, int64_t s_pad,
    float q_mult, Workspace w, const float* __restrict__ v_scale, int8_t* __restrict__ q8,
    float* __restrict__ q_scale, int8_t* __restrict__ k8, float* __restrict__ k_scale,
    uint8_t* __restrict__ v8) {
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / heads, h = bh % heads;
  const int64_t blk = blockIdx.x;
  const int cg = threadIdx.x % 16;
  const int rr = threadIdx.x / 16;
  const int c0 = cg * 8;
  __shared__ float red[2][kThreads / 32];

  float qv[4][8], kv[4][8], vv[4][8];
  float qa = 0.f, ka = 0.f;
  float mean[8], vsc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    mean[j] = w.kmean[bh * kD + c0 + j];
    vsc[j] = v_scale[bh * kD + c0 + j];
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = blk * 64 + rr + 16 * i;
    const bool live = row < seq;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      qv[i][j] = 0.f;
      kv[i][j] = 0.f;
      vv[i][j] = 0.f;
    }
    if (live) {
      const T* qp = q + b * qs.b + h * qs.h + row * qs.s + c0;
      const T* kp = k + b * ks.b + h * ks.h + row * ks.s + c0;
      const T* vp = v + b * vs.b + h * vs.h + row * vs.s + c0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        qv[i][j] = __fmul_rn(tf<T>(qp[j]), q_mult);
        kv[i][j] = __fsub_rn(tf<T>(kp[j]), mean[j]);
        vv[i][j] = tf<T>(vp[j]);
        qa = fmaxf(qa, fabsf(qv[i][j]));
        ka = fmaxf(ka, fabsf(kv[i][j]));
      }
    }
  }
  qa = warp_max(qa);
  ka = warp_max(ka);
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = qa;
    red[1][threadIdx.x >> 5] = ka;
  }
  __syncthreads();
  qa = 0.f;
  ka = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) {
    qa = fmaxf(qa, red[0][i]);
    ka = fmaxf(ka, red[1][i]);
  }
  const float qsc = qa > 0.f ? __fdiv_rn(qa, 127.0f) : 1.0f;
  const float ksc = ka > 0.f ? __fdiv_rn(ka, 127.0f) : 1.0f;
  if (threadIdx.x == 0) {
    q_scale[bh * (s_pad / 64) + blk] = qsc;
    k_scale[bh * (s_pad / 64) + blk] = ksc;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = blk * 64 + rr + 16 * i;
    const int64_t off = (bh * s_pad + row) * kD + c0;
    uint32_t qw[2], kw[2], vw[2];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t qb = 0, kb = 0, vb = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int jj = half * 4 + j;
        const int qi = __float2int_rn(__fdiv_rn(qv[i][jj], qsc));
        const int ki = __float2int_rn(__fdiv_rn(kv[i][jj], ksc));
        qb |= (static_cast<uint32_t>(max(-127, min(127, qi))) & 0xFFu) << (8 * j);
        kb |= (static_cast<uint32_t>(max(-127, min(127, ki))) & 0xFFu) << (8 * j);
        vb |= static_cast<uint32_t>(f32_to_e4m3(__fdiv_rn(vv[i][jj], vsc[jj]))) << (8 * j);
      }
      qw[half] = qb;
      kw[half] = kb;
      vw[half] = vb;
    }
    *reinterpret_cast<uint2*>(q8 + off) = make_uint2(qw[0], qw[1]);
    *reinterpret_cast<uint2*>(k8 + off) = make_uint2(kw[0], kw[1]);
    *reinterpret_cast<uint2*>(v8 + off) = make_uint2(vw[0], vw[1]);
  }
}

}  // namespace
}  // namespace xgb

using namespace xgb;

XGB_API int64_t xgb_sage_prepare_workspace(int64_t batch, int64_t heads, int64_t seq) {
  if (batch <= 0 || heads <= 0 || seq <= 0) return 0;
  const int64_t bh = batch * heads;
  return bh * stats_chunks(seq) * kD * 4 + bh * kD * 4 + bh * kD * 4;
}

XGB_API int xgb_sage_prepare(const void* q, const int64_t* q_strides, const void* k,
                             const int64_t* k_strides, const void* v, const int64_t* v_strides,
                             int dtype, int64_t batch, int64_t heads, int64_t seq,
                             int64_t head_dim, float sm_scale, int8_t* q8, float* q_scale,
                             int8_t* k8, float* k_scale, uint8_t* v8, float* v_scale,
                             void* workspace, int64_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !q_strides || !k_strides || !v_strides) return XGB_ERR_ARG;
  if (!q8 || !q_scale || !k8 || !k_scale || !v8 || !v_scale) return XGB_ERR_ARG;
  if (dtype != XGB_BF16 && dtype != XGB_F16) return XGB_ERR_ARG;
  if (head_dim != kD) return XGB_ERR_SHAPE;
  if (batch <= 0 || heads <= 0 || seq <= 0) return XGB_ERR_SHAPE;
  if (!(sm_scale > 0.f)) return XGB_ERR_ARG;
  if (q_strides[3] != 1 || k_strides[3] != 1 || v_strides[3] != 1) return XGB_ERR_STRIDE;
  if ((reinterpret_cast<uintptr_t>(q8) | reinterpret_cast<uintptr_t>(k8) |
       reinterpret_cast<uintptr_t>(v8)) & 15u)
    return XGB_ERR_ALIGN;
  const int64_t need = xgb_sage_prepare_workspace(batch, heads, seq);
  if (!workspace || workspace_bytes < need) return XGB_ERR_WORKSPACE;
  const int64_t bh = batch * heads;
  const int64_t chunks = stats_chunks(seq);
  const int64_t s_pad = (seq + 127) / 128 * 128;
  Workspace w = carve(workspace, bh, chunks);
  cudaStream_t st = as_stream(stream);
  if (cudaMemsetAsync(w.vmax, 0, bh * kD * sizeof(int), st) != cudaSuccess) return XGB_ERR_LAUNCH;
  const Strides qs{q_strides[0], q_strides[1], q_strides[2]};
  const Strides ks{k_strides[0], k_strides[1], k_strides[2]};
  const Strides vs{v_strides[0], v_strides[1], v_strides[2]};
  const float q_mult = sm_scale * kLog2e;
  dim3 sgrid(static_cast<unsigned>(chunks), static_cast<unsigned>(bh));
  dim3 qgrid(static_cast<unsigned>(s_pad / 64), static_cast<unsigned>(bh));
  if (dtype == XGB_BF16) {
    auto qb = static_cast<const __nv_bfloat16*>(q);
    auto kb = static_cast<const __nv_bfloat16*>(k);
    auto vb = static_cast<const __nv_bfloat16*>(v);
    stats_kernel<<<sgrid, kThreads, 0, st>>>(kb, ks, vb, vs, heads, seq, w, chunks);
    finalize_kernel<<<static_cast<unsigned>(bh), kD, 0, st>>>(w, chunks, seq, v_scale);
    quant_kernel<<<qgrid, kThreads, 0, st>>>(qb, qs, kb, ks, vb, vs, heads, seq, s_pad, q_mult,
                                              w, v_scale, q8, q_scale, k8, k_scale, v8);
  } else {
    auto qh = static_cast<const __half*>(q);
    auto kh = static_cast<const __half*>(k);
    auto vh = static_cast<const __half*>(v);
    stats_kernel<<<sgrid, kThreads, 0, st>>>(kh, ks, vh, vs, heads, seq, w, chunks);
    finalize_kernel<<<static_cast<unsigned>(bh), kD, 0, st>>>(w, chunks, seq, v_scale);
    quant_kernel<<<qgrid, kThreads, 0, st>>>(qh, qs, kh, ks, vh, vs, heads, seq, s_pad, q_mult,
                                              w, v_scale, q8, q_scale, k8, k_scale, v8);
  }
  return launch_status();
}
