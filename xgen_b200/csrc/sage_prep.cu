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
// Two launches: per-chunk K sums and V abs-max (partials in the caller's
// workspace; the last chunk of a head to finish turns them into the K mean
// and the V scale), then the block quantiser. `xgb_sage_prepare_rope` also
// applies the rotate-half RoPE of Q and K (x_base/x_base/operator/
// h3_partial_rope.py:9-29) as it loads them, so the RoPE needs no pass of
// its own.
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
// done [BH] int (chunks of the head finished; zeroed with vmax per call),
// kmean [BH][128] fp32.
struct Workspace {
  float* ksum;
  int* vmax;
  int* done;
  float* kmean;
  float* vscale;  // the caller's v_scale output
};

inline int64_t stats_chunks(int64_t seq) { return (seq + kStatsRows - 1) / kStatsRows; }

inline Workspace carve(void* ws, int64_t bh, int64_t chunks) {
  char* p = static_cast<char*>(ws);
  Workspace w;
  w.ksum = reinterpret_cast<float*>(p);
  p += bh * chunks * kD * sizeof(float);
  w.vmax = reinterpret_cast<int*>(p);
  p += bh * kD * sizeof(int);
  w.done = reinterpret_cast<int*>(p);
  p += (bh + 3) / 4 * 4 * sizeof(int);
  w.kmean = reinterpret_cast<float*>(p);
  return w;
}

// Eight consecutive channels of one 16-byte load as fp32.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& raw, float (&x)[8]) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int j = 0; j < 8; ++j) x[j] = tf<T>(e[j]);
}

// Where the kernels read Q (stream 0), K (1) and V (2) rows of 128 channels
// of (batch b, head h, sequence row): `load` fetches the 8 channels from c0
// in a raw form, `unpack` turns them into fp32.
//
// StridedSource: bf16/fp16 [B, H, S, 128] views with element strides.
template <typename T>
struct StridedSource {
  const T* p[3];
  Strides st[3];
  using Raw = uint4;
  __device__ __forceinline__ Raw load(int stream, int64_t b, int64_t h, int64_t row, int c0) const {
    return __ldg(reinterpret_cast<const uint4*>(p[stream] + b * st[stream].b + h * st[stream].h +
                                                row * st[stream].s + c0));
  }
  __device__ __forceinline__ static Raw zero() { return make_uint4(0, 0, 0, 0); }
  __device__ __forceinline__ static void unpack(const Raw& r, float (&x)[8]) { unpack8<T>(r, x); }
};

// RopeSource: bf16 [B, H, S, 128] views like StridedSource, with the
// rotate-half RoPE of the first `rotary` channels applied to Q (stream 0)
// and K (stream 1) as they are loaded: channel c pairs with c +- rotary/2
// (the partner chunk is a second 16-byte load of the same row), and each
// product and the sum round to bf16, the reference's arithmetic (rope8_bf16).
// cos/sin: fp32 [S, rotary] rows of the attention's sequence positions.
struct RopeSource {
  StridedSource<__nv_bfloat16> base;
  const float* cos;
  const float* sin;
  int rotary;
  using Raw = uint4;
  __device__ __forceinline__ Raw load(int stream, int64_t b, int64_t h, int64_t row, int c0) const {
    const Raw x = base.load(stream, b, h, row, c0);
    if (stream == 2 || c0 >= rotary) return x;
    const int half = rotary / 2;
    const bool first = c0 < half;
    const Raw partner = base.load(stream, b, h, row, first ? c0 + half : c0 - half);
    const int64_t at = row * rotary + c0;
    return rope8_bf16(x, partner, first, cos + at, sin + at);
  }
  __device__ __forceinline__ static Raw zero() { return make_uint4(0, 0, 0, 0); }
  __device__ __forceinline__ static void unpack(const Raw& r, float (&x)[8]) { unpack8<__nv_bfloat16>(r, x); }
};

// WireSource: the received PHAA FP8 wire (x_base/x_base/phaa/fp8_transport.py
// :26-63): per source peer p, the Q, K and V sections of its rows
// [s, batch, head] (s < seq, the peer's shard), each row 128 e4m3 bytes and
// an fp32 scale. Sequence row g of the attention is row g % seq of peer
// g / seq. A value reads as bf16(e4m3 * scale), the wire decode's result,
// so the prepared operands equal those of decode + StridedSource.
struct WireSource {
  const uint8_t* payload;
  int64_t batch, heads, peer_rows, peer_bytes;
  FastDiv div_seq;
  struct Raw {
    uint32_t lo, hi;
    float scale;
  };
  __device__ __forceinline__ Raw load(int stream, int64_t b, int64_t h, int64_t row, int c0) const {
    const uint32_t peer = fast_div(static_cast<uint32_t>(row), div_seq);
    const int64_t s = row - static_cast<int64_t>(peer) * div_seq.d;
    const uint8_t* r = payload + peer * peer_bytes +
                       (stream * peer_rows + (s * batch + b) * heads + h) * (kD + 4);
    return Raw{__ldg(reinterpret_cast<const uint32_t*>(r + c0)),
               __ldg(reinterpret_cast<const uint32_t*>(r + c0 + 4)),
               __ldg(reinterpret_cast<const float*>(r + kD))};
  }
  __device__ __forceinline__ static Raw zero() { return Raw{0, 0, 0.f}; }
  __device__ __forceinline__ static void unpack(const Raw& r, float (&x)[8]) {
    const uint32_t w[2] = {r.lo, r.hi};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint16_t pair = static_cast<uint16_t>(w[k / 2] >> (16 * (k & 1)));
      const float2 f = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3)));
      const uint32_t b2 = round_bf16x2(__fmul_rn(f.x, r.scale), __fmul_rn(f.y, r.scale));
      x[2 * k] = __uint_as_float(b2 << 16);
      x[2 * k + 1] = __uint_as_float(b2 & 0xFFFF0000u);
    }
  }
};

// Per 512-row chunk of one head: channel sums of K and channel abs-max of V.
// Thread t owns channels 8*(t%16)..+8 of rows t/16 + 16*i.
// Grids of both kernels put (batch, head) fastest: consecutive CTAs read the
// same sequence rows of all heads (contiguous in [B, S, H, D] storage and on
// the wire, and sharing the RoPE table rows in L2).
template <typename Src>
__global__ void __launch_bounds__(kThreads) stats_kernel(Src src, int64_t heads, int64_t seq,
                                                         Workspace w, int64_t chunks) {
  const int64_t bh = blockIdx.x;
  const int64_t chunk = blockIdx.y;
  const int64_t b = bh / heads, h = bh % heads;
  const int cg = threadIdx.x % 16;
  const int rr = threadIdx.x / 16;
  const int c0 = cg * 8;
  const int64_t row_begin = chunk * kStatsRows;
  const int64_t row_end = min(row_begin + kStatsRows, seq);
  float sum[8], vmx[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    sum[j] = 0.f;
    vmx[j] = 0.f;
  }
  for (int64_t r = row_begin + rr; r < row_end; r += kThreads / 16) {
    float kx[8], vx[8];
    Src::unpack(src.load(1, b, h, r, c0), kx);
    Src::unpack(src.load(2, b, h, r, c0), vx);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sum[j] += kx[j];
      vmx[j] = fmaxf(vmx[j], fabsf(vx[j]));
    }
  }
  __shared__ float part[kThreads / 16][kD];
  __shared__ float vpart[kThreads / 16][kD];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    part[rr][c0 + j] = sum[j];
    vpart[rr][c0 + j] = vmx[j];
  }
  __syncthreads();
  if (threadIdx.x < kD) {
    const int c = threadIdx.x;
    float t = 0.f, m = 0.f;
#pragma unroll
    for (int i = 0; i < kThreads / 16; ++i) {
      t += part[i][c];
      m = fmaxf(m, vpart[i][c]);
    }
    w.ksum[(bh * chunks + chunk) * kD + c] = t;
    atomicMax(&w.vmax[bh * kD + c], __float_as_int(m));
  }
  // The last chunk of the head to finish turns the partials into the K
  // channel means and the V channel scales: eight slices each sum every
  // eighth chunk, then the slices are added in a fixed order, so the result
  // does not depend on which chunk finishes last.
  __threadfence();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = atomicAdd(&w.done[bh], 1) == chunks - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  constexpr int kSlices = 8;
  float* slices = &part[0][0];  // reuse: kSlices x kD floats fit in part
  static_assert(kSlices * kD <= (kThreads / 16) * kD, "slice scratch");
  for (int k = threadIdx.x; k < kSlices * kD; k += kThreads) {
    const int c = k % kD, slice = k / kD;
    float sum = 0.f;
    for (int64_t i = slice; i < chunks; i += kSlices) sum += __ldcg(&w.ksum[(bh * chunks + i) * kD + c]);
    slices[slice * kD + c] = sum;
  }
  __syncthreads();
  if (threadIdx.x < kD) {
    const int c = threadIdx.x;
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < kSlices; ++j) t += slices[j * kD + c];
    w.kmean[bh * kD + c] = __fdiv_rn(t, static_cast<float>(seq));
    const float sc = __fdiv_rn(__int_as_float(__ldcg(&w.vmax[bh * kD + c])), 448.0f);
    w.vscale[bh * kD + c] = fmaxf(sc, FLT_MIN);
  }
}

// Block abs-max over the CTA (kN threads).
template <int kN>
__device__ __forceinline__ float block_absmax(float a, float* red) {
  a = warp_max(a);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int i = 0; i < kN / 32; ++i) r = fmaxf(r, red[i]);
  __syncthreads();
  return r;
}

// R rows (64 / R apart) x 8 channels of int8 codes round(x / s) clamped to +-127.
template <int R>
__device__ __forceinline__ void store_int8(int8_t* dst, int64_t row_stride, const float (&x)[R][8],
                                           float s, float y) {
#pragma unroll
  for (int i = 0; i < R; ++i) {
    uint32_t w[2];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // clamp to +-127, then round to nearest even by adding 1.5 * 2^23:
        // the low byte of the sum's bits is the two's-complement code (the
        // same code as rounding first and clamping after; NaN gives -127)
        const float q = fminf(fmaxf(div_by(x[i][half * 4 + j], s, y), -127.0f), 127.0f);
        word |= (__float_as_uint(__fadd_rn(q, 12582912.0f)) & 0xFFu) << (8 * j);
      }
      w[half] = word;
    }
    *reinterpret_cast<uint2*>(dst + (64 / R) * i * row_stride) = make_uint2(w[0], w[1]);
  }
}

// One CTA of 512 threads per (64-row block, head); thread t owns channels
// 8*(t%16)..+8 of rows t/16 + 32*i, i < 2 (16-byte loads of 8 channels).
// All six loads of a thread (Q, K, V) are issued before any is used, kept as
// raw 16-byte words, and Q, K and V are then quantised one after another.
constexpr int kQuantThreads = 512;
constexpr int kQuantRows = 64 * 16 / kQuantThreads;  // rows per thread

template <typename Src>
__global__ void __launch_bounds__(kQuantThreads, 2) quant_kernel(
    Src src, int64_t heads, int64_t seq, int64_t s_pad, float q_mult, Workspace w,
    const float* __restrict__ v_scale, int8_t* __restrict__ q8, float* __restrict__ q_scale,
    int8_t* __restrict__ k8, float* __restrict__ k_scale, uint8_t* __restrict__ v8) {
  const int64_t bh = blockIdx.x;
  const int64_t b = bh / heads, h = bh % heads;
  const int64_t blk = blockIdx.y;
  const int cg = threadIdx.x % 16;
  const int rr = threadIdx.x / 16;
  const int c0 = cg * 8;
  const int64_t row0 = blk * 64 + rr;
  const int64_t off0 = (bh * s_pad + row0) * kD + c0;
  constexpr int R = kQuantRows;
  constexpr int kStep = 64 / R;
  __shared__ float red[kQuantThreads / 32];
  float x[R][8];
  typename Src::Raw rq[R], rk[R], rv[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int64_t row = row0 + kStep * i;
    const bool ok = row < seq;
    rq[i] = ok ? src.load(0, b, h, row, c0) : Src::zero();
    rk[i] = ok ? src.load(1, b, h, row, c0) : Src::zero();
    rv[i] = ok ? src.load(2, b, h, row, c0) : Src::zero();
  }

  // Values are recomputed from the raw words in each pass (the same
  // operations give the same bits), which keeps few registers live.
  bool ok[R];
#pragma unroll
  for (int i = 0; i < R; ++i) ok[i] = row0 + kStep * i < seq;

  // Q: x * sm_scale * log2(e), per-block int8.
  float a = 0.f;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    Src::unpack(rq[i], x[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) a = fmaxf(a, fabsf(__fmul_rn(x[i][j], q_mult)));
  }
  a = block_absmax<kQuantThreads>(a, red);
  float sc = a > 0.f ? __fdiv_rn(a, 127.0f) : 1.0f;
  if (threadIdx.x == 0) q_scale[bh * (s_pad / 64) + blk] = sc;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    Src::unpack(rq[i], x[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[i][j] = __fmul_rn(x[i][j], q_mult);  // rows >= seq: 0
  }
  store_int8(q8 + off0, kD, x, sc, __frcp_rn(sc));

  // K: x - mean over the sequence, per-block int8.
  float mean[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) mean[j] = w.kmean[bh * kD + c0 + j];
  a = 0.f;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    Src::unpack(rk[i], x[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) a = fmaxf(a, ok[i] ? fabsf(__fsub_rn(x[i][j], mean[j])) : 0.f);
  }
  a = block_absmax<kQuantThreads>(a, red);
  sc = a > 0.f ? __fdiv_rn(a, 127.0f) : 1.0f;
  if (threadIdx.x == 0) k_scale[bh * (s_pad / 64) + blk] = sc;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    Src::unpack(rk[i], x[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[i][j] = ok[i] ? __fsub_rn(x[i][j], mean[j]) : 0.f;
  }
  store_int8(k8 + off0, kD, x, sc, __frcp_rn(sc));

  // V: per-channel e4m3 (rows >= seq were loaded as zeros).
  float vsc[8], vrc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    vsc[j] = v_scale[bh * kD + c0 + j];
    vrc[j] = __frcp_rn(vsc[j]);
  }
#pragma unroll
  for (int i = 0; i < R; ++i) {
    Src::unpack(rv[i], x[i]);
    uint32_t q[4];
#pragma unroll
    for (int j = 0; j < 8; j += 2)
      q[j / 2] = e4m3x2(div_by(x[i][j], vsc[j], vrc[j]), div_by(x[i][j + 1], vsc[j + 1], vrc[j + 1]));
    *reinterpret_cast<uint2*>(v8 + off0 + kStep * i * kD) = make_uint2(q[0] | (q[1] << 16), q[2] | (q[3] << 16));
  }
}

struct Outputs {
  int8_t* q8;
  float* q_scale;
  int8_t* k8;
  float* k_scale;
  uint8_t* v8;
  float* v_scale;
};

inline int64_t stats_workspace(int64_t bh, int64_t seq) {
  return bh * stats_chunks(seq) * kD * 4 + bh * kD * 4 + (bh + 3) / 4 * 4 * 4 + bh * kD * 4;
}

// Statistics, finalize and quantisation of [batch, heads, seq] rows read from `src`.
template <typename Src>
int prepare(const Src& src, int64_t batch, int64_t heads, int64_t seq, float sm_scale,
            const Outputs& o, void* workspace, cudaStream_t st) {
  const int64_t bh = batch * heads;
  const int64_t chunks = stats_chunks(seq);
  const int64_t s_pad = (seq + 127) / 128 * 128;
  Workspace w = carve(workspace, bh, chunks);
  w.vscale = o.v_scale;
  // vmax and the per-head chunk counters, contiguous
  const size_t zero_bytes = bh * kD * sizeof(int) + (bh + 3) / 4 * 4 * sizeof(int);
  if (cudaMemsetAsync(w.vmax, 0, zero_bytes, st) != cudaSuccess) return XGB_ERR_LAUNCH;
  const float q_mult = sm_scale * kLog2e;
  if (chunks > 65535 || s_pad / 64 > 65535) return XGB_ERR_SHAPE;  // grid y
  const dim3 sgrid(static_cast<unsigned>(bh), static_cast<unsigned>(chunks));
  const dim3 qgrid(static_cast<unsigned>(bh), static_cast<unsigned>(s_pad / 64));
  stats_kernel<<<sgrid, kThreads, 0, st>>>(src, heads, seq, w, chunks);
  quant_kernel<<<qgrid, kQuantThreads, 0, st>>>(src, heads, seq, s_pad, q_mult, w, o.v_scale, o.q8,
                                                o.q_scale, o.k8, o.k_scale, o.v8);
  return launch_status();
}

}  // namespace
}  // namespace xgb

using namespace xgb;

XGB_API int64_t xgb_sage_prepare_workspace(int64_t batch, int64_t heads, int64_t seq) {
  if (batch <= 0 || heads <= 0 || seq <= 0) return 0;
  return stats_workspace(batch * heads, seq);
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
  // 16-byte loads of 8 channels: row starts and strides in multiples of 8.
  for (int d = 0; d < 3; ++d)
    if (q_strides[d] % 8 || k_strides[d] % 8 || v_strides[d] % 8) return XGB_ERR_STRIDE;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v)) & 15u)
    return XGB_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(q8) | reinterpret_cast<uintptr_t>(k8) |
       reinterpret_cast<uintptr_t>(v8)) & 15u)
    return XGB_ERR_ALIGN;
  const int64_t need = xgb_sage_prepare_workspace(batch, heads, seq);
  if (!workspace || workspace_bytes < need) return XGB_ERR_WORKSPACE;
  const Strides qs{q_strides[0], q_strides[1], q_strides[2]};
  const Strides ks{k_strides[0], k_strides[1], k_strides[2]};
  const Strides vs{v_strides[0], v_strides[1], v_strides[2]};
  const Outputs o{q8, q_scale, k8, k_scale, v8, v_scale};
  if (dtype == XGB_BF16) {
    using S = StridedSource<__nv_bfloat16>;
    const S src{{static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                 static_cast<const __nv_bfloat16*>(v)}, {qs, ks, vs}};
    return prepare(src, batch, heads, seq, sm_scale, o, workspace, as_stream(stream));
  }
  using S = StridedSource<__half>;
  const S src{{static_cast<const __half*>(q), static_cast<const __half*>(k), static_cast<const __half*>(v)},
              {qs, ks, vs}};
  return prepare(src, batch, heads, seq, sm_scale, o, workspace, as_stream(stream));
}

XGB_API int xgb_sage_prepare_rope(const void* q, const int64_t* q_strides, const void* k,
                                  const int64_t* k_strides, const void* v, const int64_t* v_strides,
                                  int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                                  float sm_scale, const float* cos, const float* sin, int64_t rotary,
                                  int8_t* q8, float* q_scale, int8_t* k8, float* k_scale, uint8_t* v8,
                                  float* v_scale, void* workspace, int64_t workspace_bytes,
                                  void* stream) {
  if (!q || !k || !v || !q_strides || !k_strides || !v_strides || !cos || !sin) return XGB_ERR_ARG;
  if (!q8 || !q_scale || !k8 || !k_scale || !v8 || !v_scale) return XGB_ERR_ARG;
  if (head_dim != kD) return XGB_ERR_SHAPE;
  if (batch <= 0 || heads <= 0 || seq <= 0) return XGB_ERR_SHAPE;
  // 8-channel chunks pair with chunks rotary/2 away: rotary/2 a multiple of 8
  if (rotary <= 0 || rotary > kD || rotary % 16) return XGB_ERR_SHAPE;
  if (!(sm_scale > 0.f)) return XGB_ERR_ARG;
  if (q_strides[3] != 1 || k_strides[3] != 1 || v_strides[3] != 1) return XGB_ERR_STRIDE;
  for (int d = 0; d < 3; ++d)
    if (q_strides[d] % 8 || k_strides[d] % 8 || v_strides[d] % 8) return XGB_ERR_STRIDE;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(cos) | reinterpret_cast<uintptr_t>(sin)) & 15u)
    return XGB_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(q8) | reinterpret_cast<uintptr_t>(k8) |
       reinterpret_cast<uintptr_t>(v8)) & 15u)
    return XGB_ERR_ALIGN;
  const int64_t need = xgb_sage_prepare_workspace(batch, heads, seq);
  if (!workspace || workspace_bytes < need) return XGB_ERR_WORKSPACE;
  using B = StridedSource<__nv_bfloat16>;
  RopeSource src{};
  src.base = B{{static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                static_cast<const __nv_bfloat16*>(v)},
               {Strides{q_strides[0], q_strides[1], q_strides[2]},
                Strides{k_strides[0], k_strides[1], k_strides[2]},
                Strides{v_strides[0], v_strides[1], v_strides[2]}}};
  src.cos = cos;
  src.sin = sin;
  src.rotary = static_cast<int>(rotary);
  const Outputs o{q8, q_scale, k8, k_scale, v8, v_scale};
  return prepare(src, batch, heads, seq, sm_scale, o, workspace, as_stream(stream));
}

XGB_API int xgb_sage_prepare_wire(const uint8_t* payload, int64_t peers, int64_t seq,
                                  int64_t batch, int64_t heads, int64_t valid_seq,
                                  int64_t peer_padding, float sm_scale, int8_t* q8, float* q_scale,
                                  int8_t* k8, float* k_scale, uint8_t* v8, float* v_scale,
                                  void* workspace, int64_t workspace_bytes, void* stream) {
  if (!payload || !q8 || !q_scale || !k8 || !k_scale || !v8 || !v_scale) return XGB_ERR_ARG;
  if (peers <= 0 || seq <= 0 || batch <= 0 || heads <= 0) return XGB_ERR_SHAPE;
  if (valid_seq <= 0 || valid_seq > peers * seq || peers * seq > INT32_MAX) return XGB_ERR_SHAPE;
  if (peer_padding < 0 || peer_padding % 4) return XGB_ERR_ARG;
  if (!(sm_scale > 0.f)) return XGB_ERR_ARG;
  // 4-byte loads of codes and scales: the wire rows start at 4-byte multiples
  if ((reinterpret_cast<uintptr_t>(payload) & 3u) ||
      ((reinterpret_cast<uintptr_t>(q8) | reinterpret_cast<uintptr_t>(k8) |
        reinterpret_cast<uintptr_t>(v8)) & 15u))
    return XGB_ERR_ALIGN;
  const int64_t need = xgb_sage_prepare_workspace(batch, heads, valid_seq);
  if (!workspace || workspace_bytes < need) return XGB_ERR_WORKSPACE;
  WireSource src{};
  src.payload = payload;
  src.batch = batch;
  src.heads = heads;
  src.peer_rows = seq * batch * heads;
  src.peer_bytes = 3 * src.peer_rows * (kD + 4) + peer_padding;
  src.div_seq = make_fastdiv(static_cast<uint32_t>(seq));
  const Outputs o{q8, q_scale, k8, k_scale, v8, v_scale};
  return prepare(src, batch, heads, valid_seq, sm_scale, o, workspace, as_stream(stream));
}
