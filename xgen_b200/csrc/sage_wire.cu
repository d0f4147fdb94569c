// Sage quantisation before the sequence-parallel A2A ("INT8 on the wire").
//
// Each SP rank holds S_loc tokens of every head. Instead of sending bf16 (or
// the FP8 wire format) and quantising after the exchange, the sender
// quantises its own rows the way the attention kernel consumes them:
//
//   Q: RoPE, x * sm_scale * log2(e), int8 per (head, group of 16 tokens)
//   K: RoPE, x - mean over the whole sequence (per head and channel), int8
//      per (head, group of 16 tokens)
//   V: e4m3 per channel, scale = max(amax over the whole sequence / 448, FLT_MIN)
//
// The sequence-wide K means and V maxima come from per-rank sums and maxima
// (xgb_sage_wire_stats) all-reduced by the caller. Groups of 16 tokens align
// with every rank's span (S_loc is a multiple of 16), so the receiver's
// attention reads the exchanged buffers in place: Q/K/V rows
// [peer][S_loc][batch][head][128] and scales [peer][S_loc/16][batch][head][2]
// are, for one (batch, head), rows of a uniform stride. This is the
// SageAttention2 recipe (Zhang et al. 2024) with 16-token Q/K groups
// instead of the attention-side prepare step (sage_prep.cu), and the partial
// RoPE of x_base/x_base/operator/h3_partial_rope.py:9-47 fused in with its
// bf16 rounding.
//
// Sources are [peer, seq, batch, head] views of 128-channel rows (element
// strides, channel stride 1), as for the FP8 wire encode.
#include <cfloat>

#include "xgb_common.cuh"

namespace xgb {
namespace {

constexpr int kD = 128;
constexpr int kThreads = 256;     // 16 rows x 16 lanes of 8 channels
constexpr int kStatsRows = 256;   // rows per stats CTA

struct View {
  const __nv_bfloat16* p;
  int64_t st[4];  // peer, seq, batch, head
};

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&x)[8]) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
  for (int j = 0; j < 8; ++j) x[j] = __bfloat162float(e[j]);
}

// Eight channels c0..c0+7 of one row, with the reference's partial RoPE
// (bf16 result) when they lie below `rotary` (rotary/2 a multiple of 8, so
// the 8 channels sit on one side of the half split).
__device__ __forceinline__ void load_rope8(const __nv_bfloat16* row, int c0, const float* cos_row,
                                           const float* sin_row, int rotary, float (&x)[8]) {
  load8(row + c0, x);
  if (c0 >= rotary) return;
  const int half = rotary / 2;
  const bool first = c0 < half;
  float p[8];
  load8(row + (first ? c0 + half : c0 - half), p);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float cb = bf16_round(cos_row[c0 + j]);
    const float sb = bf16_round(sin_row[c0 + j]);
    const float left = bf16_round(__fmul_rn(x[j], cb));
    const float right = bf16_round(__fmul_rn(first ? -p[j] : p[j], sb));
    x[j] = bf16_round(__fadd_rn(left, right));
  }
}

__device__ __forceinline__ const __nv_bfloat16* row_ptr(const View& v, int64_t peer, int64_t s,
                                                        int64_t b, int64_t h) {
  return v.p + peer * v.st[0] + s * v.st[1] + b * v.st[2] + h * v.st[3];
}

// Per (chunk of 256 rows, peer*batch*head): partial channel sums of RoPE'd K
// and abs-maxima of V.
__global__ void __launch_bounds__(kThreads) stats_kernel(View k, View v, int64_t seq, int64_t batch,
                                                         int64_t heads, const float* cos,
                                                         const float* sin, int rotary,
                                                         float* __restrict__ part_sum,
                                                         float* __restrict__ part_max) {
  const int64_t head_id = blockIdx.y;  // (peer, batch, head)
  const int64_t h = head_id % heads;
  const int64_t b = (head_id / heads) % batch;
  const int64_t peer = head_id / (heads * batch);
  const int cg = threadIdx.x % 16, rr = threadIdx.x / 16, c0 = cg * 8;
  float sum[8], mx[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    sum[j] = 0.f;
    mx[j] = 0.f;
  }
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kStatsRows;
  const int64_t r1 = min(r0 + kStatsRows, seq);
  for (int64_t s = r0 + rr; s < r1; s += 16) {
    float kx[8], vx[8];
    load_rope8(row_ptr(k, peer, s, b, h), c0, cos + s * rotary, sin + s * rotary, rotary, kx);
    load8(row_ptr(v, peer, s, b, h) + c0, vx);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sum[j] += kx[j];
      mx[j] = fmaxf(mx[j], fabsf(vx[j]));
    }
  }
  __shared__ float ssum[16][kD], smax[16][kD];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    ssum[rr][c0 + j] = sum[j];
    smax[rr][c0 + j] = mx[j];
  }
  __syncthreads();
  if (threadIdx.x < kD) {
    float t = 0.f, m = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      t += ssum[i][threadIdx.x];
      m = fmaxf(m, smax[i][threadIdx.x]);
    }
    const int64_t o = (static_cast<int64_t>(blockIdx.x) * gridDim.y + head_id) * kD + threadIdx.x;
    part_sum[o] = t;
    part_max[o] = m;
  }
}

// Chunk partials -> per (peer, batch, head) sums and maxima, in chunk order.
__global__ void __launch_bounds__(kD) stats_finalize_kernel(const float* __restrict__ part_sum,
                                                            const float* __restrict__ part_max,
                                                            int64_t chunks, int64_t head_ids,
                                                            float* __restrict__ ksum,
                                                            float* __restrict__ vmax) {
  const int64_t head_id = blockIdx.x;
  float t = 0.f, m = 0.f;
  for (int64_t c = 0; c < chunks; ++c) {
    const int64_t o = (c * head_ids + head_id) * kD + threadIdx.x;
    t += part_sum[o];
    m = fmaxf(m, part_max[o]);
  }
  ksum[head_id * kD + threadIdx.x] = t;
  vmax[head_id * kD + threadIdx.x] = m;
}

__device__ __forceinline__ float block_absmax(float a, float* red) {
  a = warp_max(a);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) r = fmaxf(r, red[i]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ uint2 int8x8(const float (&x)[8], float s, float y) {
  uint32_t w[2];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int code = __float2int_rn(div_by(x[half * 4 + j], s, y));
      word |= (static_cast<uint32_t>(max(-127, min(127, code))) & 0xFFu) << (8 * j);
    }
    w[half] = word;
  }
  return make_uint2(w[0], w[1]);
}

// One CTA per (peer, group of 16 rows) x (batch, head); thread t owns
// channels 8*(t%16)..+8 of row t/16 of the group.
__global__ void __launch_bounds__(kThreads) encode_kernel(
    View q, View k, View v, int64_t seq, int64_t batch, int64_t heads, const float* cos,
    const float* sin, int rotary, float q_mult, const float* __restrict__ ksum,
    const float* __restrict__ vmax, float seq_real, int8_t* __restrict__ q8, int8_t* __restrict__ k8,
    uint8_t* __restrict__ v8, float* __restrict__ qk_scale, float* __restrict__ v_scale) {
  __shared__ float red[kThreads / 32];
  const int64_t groups = seq / 16;
  const int64_t peer = blockIdx.x / groups, g = blockIdx.x % groups;
  const int64_t b = blockIdx.y / heads, h = blockIdx.y % heads;
  const int64_t head_id = (peer * batch + b) * heads + h;
  const int cg = threadIdx.x % 16, rr = threadIdx.x / 16, c0 = cg * 8;
  const int64_t s = g * 16 + rr;
  const float* cs = cos + s * rotary;
  const float* sn = sin + s * rotary;
  // destination row [peer][s][b][h]
  const int64_t out_row = ((peer * seq + s) * batch + b) * heads + h;
  const int64_t scale_at = (((peer * groups + g) * batch + b) * heads + h) * 2;

  float x[8];
  // Q
  load_rope8(row_ptr(q, peer, s, b, h), c0, cs, sn, rotary, x);
  float a = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    x[j] = __fmul_rn(x[j], q_mult);
    a = fmaxf(a, fabsf(x[j]));
  }
  a = block_absmax(a, red);
  float sc = a > 0.f ? __fdiv_rn(a, 127.0f) : 1.0f;
  *reinterpret_cast<uint2*>(q8 + out_row * kD + c0) = int8x8(x, sc, __frcp_rn(sc));
  if (threadIdx.x == 0) qk_scale[scale_at] = sc;

  // K - mean
  load_rope8(row_ptr(k, peer, s, b, h), c0, cs, sn, rotary, x);
  a = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float mean = __fdiv_rn(ksum[head_id * kD + c0 + j], seq_real);
    x[j] = __fsub_rn(x[j], mean);
    a = fmaxf(a, fabsf(x[j]));
  }
  a = block_absmax(a, red);
  sc = a > 0.f ? __fdiv_rn(a, 127.0f) : 1.0f;
  *reinterpret_cast<uint2*>(k8 + out_row * kD + c0) = int8x8(x, sc, __frcp_rn(sc));
  if (threadIdx.x == 0) qk_scale[scale_at + 1] = sc;

  // V per channel
  load8(row_ptr(v, peer, s, b, h) + c0, x);
  uint32_t w[2];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = c0 + half * 4 + j;
      const float vs = fmaxf(__fdiv_rn(vmax[head_id * kD + c], 448.0f), FLT_MIN);
      word |= static_cast<uint32_t>(f32_to_e4m3(div_by(x[half * 4 + j], vs, __frcp_rn(vs)))) << (8 * j);
      if (g == 0 && rr == 0) v_scale[head_id * kD + c] = vs;
    }
    w[half] = word;
  }
  *reinterpret_cast<uint2*>(v8 + out_row * kD + c0) = make_uint2(w[0], w[1]);
}

int check_views(const View (&vs)[3], int n) {
  for (int i = 0; i < n; ++i) {
    if (!vs[i].p) return XGB_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(vs[i].p) & 15u) return XGB_ERR_ALIGN;
    for (int d = 0; d < 4; ++d)
      if (vs[i].st[d] % 8) return XGB_ERR_STRIDE;  // 16-byte row loads
  }
  return XGB_OK;
}

View make_view(const void* p, const int64_t* st) {
  View v{static_cast<const __nv_bfloat16*>(p), {st[0], st[1], st[2], st[3]}};
  return v;
}

}  // namespace
}  // namespace xgb

using namespace xgb;

XGB_API int64_t xgb_sage_wire_stats_workspace(int64_t peers, int64_t seq, int64_t batch,
                                              int64_t heads) {
  if (peers <= 0 || seq <= 0 || batch <= 0 || heads <= 0) return 0;
  const int64_t chunks = (seq + kStatsRows - 1) / kStatsRows;
  return 2 * chunks * peers * batch * heads * kD * static_cast<int64_t>(sizeof(float));
}

XGB_API int xgb_sage_wire_stats(const void* k, const int64_t* k_strides, const void* v,
                                const int64_t* v_strides, int64_t peers, int64_t seq,
                                int64_t batch, int64_t heads, const float* cos, const float* sin,
                                int64_t rotary, float* ksum, float* vmax, void* workspace,
                                int64_t workspace_bytes, void* stream) {
  if (!k_strides || !v_strides || !ksum || !vmax) return XGB_ERR_ARG;
  if (peers <= 0 || seq <= 0 || batch <= 0 || heads <= 0) return XGB_ERR_SHAPE;
  if (rotary < 0 || rotary > kD || rotary % 16) return XGB_ERR_SHAPE;
  if (rotary > 0 && (!cos || !sin)) return XGB_ERR_ARG;
  const View views[3] = {make_view(k, k_strides), make_view(v, v_strides), make_view(k, k_strides)};
  int rc = check_views(views, 2);
  if (rc) return rc;
  if (!workspace || workspace_bytes < xgb_sage_wire_stats_workspace(peers, seq, batch, heads))
    return XGB_ERR_WORKSPACE;
  const int64_t chunks = (seq + kStatsRows - 1) / kStatsRows;
  const int64_t ids = peers * batch * heads;
  if (ids > 65535) return XGB_ERR_SHAPE;
  float* part_sum = static_cast<float*>(workspace);
  float* part_max = part_sum + chunks * ids * kD;
  cudaStream_t st = as_stream(stream);
  stats_kernel<<<dim3(static_cast<unsigned>(chunks), static_cast<unsigned>(ids)), kThreads, 0, st>>>(
      views[0], views[1], seq, batch, heads, cos, sin, static_cast<int>(rotary), part_sum, part_max);
  stats_finalize_kernel<<<static_cast<unsigned>(ids), kD, 0, st>>>(part_sum, part_max, chunks, ids,
                                                                   ksum, vmax);
  return launch_status();
}

XGB_API int xgb_sage_wire_encode(const void* q, const int64_t* q_strides, const void* k,
                                 const int64_t* k_strides, const void* v, const int64_t* v_strides,
                                 int64_t peers, int64_t seq, int64_t batch, int64_t heads,
                                 const float* cos, const float* sin, int64_t rotary, float sm_scale,
                                 const float* ksum, const float* vmax, int64_t seq_real,
                                 int8_t* q8, int8_t* k8, uint8_t* v8, float* qk_scale,
                                 float* v_scale, void* stream) {
  if (!q_strides || !k_strides || !v_strides || !ksum || !vmax) return XGB_ERR_ARG;
  if (!q8 || !k8 || !v8 || !qk_scale || !v_scale) return XGB_ERR_ARG;
  if (peers <= 0 || seq <= 0 || seq % 16 || batch <= 0 || heads <= 0) return XGB_ERR_SHAPE;
  if (seq_real <= 0 || seq_real > peers * seq) return XGB_ERR_SHAPE;
  if (rotary < 0 || rotary > kD || rotary % 16) return XGB_ERR_SHAPE;
  if (rotary > 0 && (!cos || !sin)) return XGB_ERR_ARG;
  if (!(sm_scale > 0.f)) return XGB_ERR_ARG;
  const View views[3] = {make_view(q, q_strides), make_view(k, k_strides), make_view(v, v_strides)};
  int rc = check_views(views, 3);
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(q8) | reinterpret_cast<uintptr_t>(k8) |
       reinterpret_cast<uintptr_t>(v8)) & 7u)
    return XGB_ERR_ALIGN;
  if (batch * heads > 65535 || peers * (seq / 16) > INT32_MAX) return XGB_ERR_SHAPE;
  const float q_mult = sm_scale * 1.4426950408889634f;
  dim3 grid(static_cast<unsigned>(peers * (seq / 16)), static_cast<unsigned>(batch * heads));
  encode_kernel<<<grid, kThreads, 0, as_stream(stream)>>>(
      views[0], views[1], views[2], seq, batch, heads, cos, sin, static_cast<int>(rotary), q_mult,
      ksum, vmax, static_cast<float>(seq_real), q8, k8, v8, qk_scale, v_scale);
  return launch_status();
}
