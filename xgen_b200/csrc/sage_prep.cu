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
// One launch: a cooperative kernel of one or two CTAs per SM in three phases
// split by grid barriers (bounded waits): (A) read Q, K and V once; quantise
// Q and accumulate K column sums and V column abs-maxima; (B) per head, the K
// mean and the V scale; (C) quantise K and V, walking the sequence backwards
// so the rows phase A read last are still in L2. `xgb_sage_prepare_rope`
// also applies the rotate-half RoPE of Q and K (x_base/x_base/operator/
// h3_partial_rope.py:9-29) as it loads them, so the RoPE needs no pass of
// its own.
#include <cfloat>

#include "sm100.cuh"
#include "xgb_common.cuh"

namespace xgb {
namespace {

constexpr int kD = 128;
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

struct Outputs {
  int8_t* q8;
  float* q_scale;
  int8_t* k8;
  float* k_scale;
  uint8_t* v8;
  float* v_scale;
};

// The kernel: 512 threads per CTA; thread t owns channels 8*(t%16)..+8 of
// rows t/16 and t/16 + 32 of a 64-row block (16-byte loads of 8 channels).
constexpr int kPrepThreads = 512;
constexpr int kPrepRows = 64 * 16 / kPrepThreads;  // rows per thread and block
constexpr int kMaxPrepCtas = 296;                  // two per SM of a B200
constexpr uint64_t kBarrierLimitNs = 2000000000ull;

// Heads are taken in groups of G (the grid is P CTAs per head of a group):
// CTA c works on head g0 + c % G of group g0 and on the blocks c / G,
// c / G + P, ... of it.
struct PrepShape {
  int64_t heads, bh, seq, s_pad, n_blk;
  int G, P;
  float q_mult;
};

// Workspace: barrier counter (zeroed per call), then kmean [BH][128], then
// the per-CTA partial K column sums and V column abs-maxima [BH][P][128].
struct PrepWork {
  int* arrive;
  float* kmean;
  float* part_k;
  float* part_v;
  int* err;
};

constexpr int64_t kCounterBytes = 64;

// Partial rows per head: P <= kMaxPrepCtas / min(BH, kMaxPrepCtas), at least 1.
inline int64_t partials_per_head(int64_t bh) {
  return std::max<int64_t>(1, kMaxPrepCtas / std::min<int64_t>(bh, kMaxPrepCtas));
}

inline int64_t prep_workspace(int64_t bh) {
  return kCounterBytes + bh * kD * 4 + 2 * bh * partials_per_head(bh) * kD * 4;
}

inline PrepWork carve(void* ws, int64_t bh, int P, int* err) {
  char* p = static_cast<char*>(ws);
  PrepWork w;
  w.arrive = reinterpret_cast<int*>(p);
  p += kCounterBytes;
  w.kmean = reinterpret_cast<float*>(p);
  p += bh * kD * 4;
  w.part_k = reinterpret_cast<float*>(p);
  p += bh * P * kD * 4;
  w.part_v = reinterpret_cast<float*>(p);
  w.err = err;
  return w;
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier of a cooperative launch: every CTA's writes before it are
// visible to every CTA after it. The wait gives up after kBarrierLimitNs,
// records a timeout in *err and returns false (every thread of the CTA).
__device__ bool grid_barrier(int* arrive, int target, int* err, int* ok_smem) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = *ok_smem;
    __threadfence();
    atomicAdd(arrive, 1);
    if (ok) {
      const uint64_t t0 = sm100::global_timer_ns();
      while (ld_acquire(arrive) < target) {
        if (sm100::global_timer_ns() - t0 > kBarrierLimitNs) {
          if (err) atomicExch(err, sm100::kErrTimeout);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    __threadfence();
    *ok_smem = ok;
  }
  __syncthreads();
  return *ok_smem != 0;
}

template <typename Src>
__global__ void __launch_bounds__(kPrepThreads, 2) prepare_kernel(Src src, PrepShape sh, PrepWork w,
                                                                  Outputs o) {
  constexpr int R = kPrepRows;
  constexpr int kStep = 64 / R;
  const int cg = threadIdx.x % 16;
  const int rr = threadIdx.x / 16;
  const int c0 = cg * 8;
  const int grid = static_cast<int>(gridDim.x);
  const int hg = static_cast<int>(blockIdx.x) % sh.G;
  const int pidx = static_cast<int>(blockIdx.x) / sh.G;
  __shared__ float red[kPrepThreads / 32];
  __shared__ float part[kPrepThreads / 16][kD];
  __shared__ float vpart[kPrepThreads / 16][kD];
  __shared__ int ok_smem;
  if (threadIdx.x == 0) ok_smem = 1;
  float x[R][8];

  // ---- A: Q codes; K column sums and V column abs-maxima per CTA and head.
  for (int64_t g0 = 0; g0 < sh.bh; g0 += sh.G) {
    const int64_t bh = g0 + hg;
    const bool active = bh < sh.bh;  // the last group may hold fewer heads (uniform per CTA)
    const int64_t b = bh / sh.heads, h = bh % sh.heads;
    float ksum[8], vmx[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      ksum[j] = 0.f;
      vmx[j] = 0.f;
    }
    for (int64_t blk = pidx; active && blk < sh.n_blk; blk += sh.P) {
      const int64_t row0 = blk * 64 + rr;
      const int64_t off0 = (bh * sh.s_pad + row0) * kD + c0;
      typename Src::Raw rq[R], rk[R], rv[R];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int64_t row = row0 + kStep * i;
        const bool ok = row < sh.seq;
        rq[i] = ok ? src.load(0, b, h, row, c0) : Src::zero();
        rk[i] = ok ? src.load(1, b, h, row, c0) : Src::zero();
        rv[i] = ok ? src.load(2, b, h, row, c0) : Src::zero();
      }
      // K and V statistics (rows >= seq were loaded as zeros).
#pragma unroll
      for (int i = 0; i < R; ++i) {
        float kx[8], vx[8];
        Src::unpack(rk[i], kx);
        Src::unpack(rv[i], vx);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          ksum[j] += kx[j];
          vmx[j] = fmaxf(vmx[j], fabsf(vx[j]));
        }
      }
      // Q: x * sm_scale * log2(e), per-block int8.
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < R; ++i) {
        Src::unpack(rq[i], x[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          x[i][j] = __fmul_rn(x[i][j], sh.q_mult);  // rows >= seq: 0
          a = fmaxf(a, fabsf(x[i][j]));
        }
      }
      a = block_absmax<kPrepThreads>(a, red);
      const float sc = a > 0.f ? __fdiv_rn(a, 127.0f) : 1.0f;
      if (threadIdx.x == 0) o.q_scale[bh * (sh.s_pad / 64) + blk] = sc;
      store_int8(o.q8 + off0, kD, x, sc, __frcp_rn(sc));
    }
    if (active) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        part[rr][c0 + j] = ksum[j];
        vpart[rr][c0 + j] = vmx[j];
      }
    }
    __syncthreads();
    if (active && threadIdx.x < kD) {
      const int c = threadIdx.x;
      float t = 0.f, m = 0.f;
#pragma unroll 8
      for (int i = 0; i < kPrepThreads / 16; ++i) {
        t += part[i][c];
        m = fmaxf(m, vpart[i][c]);
      }
      w.part_k[(bh * sh.P + pidx) * kD + c] = t;
      w.part_v[(bh * sh.P + pidx) * kD + c] = m;
    }
    __syncthreads();
  }
  bool ok = grid_barrier(w.arrive, grid, w.err, &ok_smem);

  // ---- B: per head, K mean = sum / seq and V scale = max(amax / 448, FLT_MIN),
  // each from the head's P partial rows in a fixed order (four interleaved
  // slices, added in slice order), so the result does not depend on timing.
  for (int64_t bh = blockIdx.x; ok && bh < sh.bh; bh += grid) {
    const int slice = threadIdx.x / kD, c = threadIdx.x % kD;
    float t = 0.f, m = 0.f;
    for (int p = slice; p < sh.P; p += kPrepThreads / kD) {
      t += __ldcg(&w.part_k[(bh * sh.P + p) * kD + c]);
      m = fmaxf(m, __ldcg(&w.part_v[(bh * sh.P + p) * kD + c]));
    }
    part[slice][c] = t;
    vpart[slice][c] = m;
    __syncthreads();
    if (threadIdx.x < kD) {
      float ts = 0.f, ms = 0.f;
#pragma unroll
      for (int s = 0; s < kPrepThreads / kD; ++s) {
        ts += part[s][c];
        ms = fmaxf(ms, vpart[s][c]);
      }
      w.kmean[bh * kD + c] = __fdiv_rn(ts, static_cast<float>(sh.seq));
      o.v_scale[bh * kD + c] = fmaxf(__fdiv_rn(ms, 448.0f), FLT_MIN);
    }
    __syncthreads();
  }
  ok = grid_barrier(w.arrive, 2 * grid, w.err, &ok_smem) && ok;

  // ---- C: K codes (mean-smoothed, per-block int8) and V codes (per-channel
  // e4m3), groups and blocks in reverse order of phase A.
  const int64_t n_groups = (sh.bh + sh.G - 1) / sh.G;
  for (int64_t gi = n_groups - 1; ok && gi >= 0; --gi) {
    const int64_t bh = gi * sh.G + hg;
    if (bh >= sh.bh) continue;  // uniform per CTA
    const int64_t b = bh / sh.heads, h = bh % sh.heads;
    float mean[8], vsc[8], vrc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mean[j] = __ldcg(&w.kmean[bh * kD + c0 + j]);
      vsc[j] = __ldcg(&o.v_scale[bh * kD + c0 + j]);
      vrc[j] = __frcp_rn(vsc[j]);
    }
    for (int64_t k = pidx; k < sh.n_blk; k += sh.P) {
      const int64_t blk = sh.n_blk - 1 - k;
      const int64_t row0 = blk * 64 + rr;
      const int64_t off0 = (bh * sh.s_pad + row0) * kD + c0;
      typename Src::Raw rk[R], rv[R];
      bool valid[R];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int64_t row = row0 + kStep * i;
        valid[i] = row < sh.seq;
        rk[i] = valid[i] ? src.load(1, b, h, row, c0) : Src::zero();
        rv[i] = valid[i] ? src.load(2, b, h, row, c0) : Src::zero();
      }
      // K: x - mean over the sequence, per-block int8 (rows >= seq: 0).
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < R; ++i) {
        Src::unpack(rk[i], x[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          x[i][j] = valid[i] ? __fsub_rn(x[i][j], mean[j]) : 0.f;
          a = fmaxf(a, fabsf(x[i][j]));
        }
      }
      a = block_absmax<kPrepThreads>(a, red);
      const float sc = a > 0.f ? __fdiv_rn(a, 127.0f) : 1.0f;
      if (threadIdx.x == 0) o.k_scale[bh * (sh.s_pad / 64) + blk] = sc;
      store_int8(o.k8 + off0, kD, x, sc, __frcp_rn(sc));
      // V: per-channel e4m3 (rows >= seq were loaded as zeros).
#pragma unroll
      for (int i = 0; i < R; ++i) {
        Src::unpack(rv[i], x[i]);
        uint32_t q[4];
#pragma unroll
        for (int j = 0; j < 8; j += 2)
          q[j / 2] = e4m3x2(div_by(x[i][j], vsc[j], vrc[j]), div_by(x[i][j + 1], vsc[j + 1], vrc[j + 1]));
        *reinterpret_cast<uint2*>(o.v8 + off0 + kStep * i * kD) = make_uint2(q[0] | (q[1] << 16), q[2] | (q[3] << 16));
      }
    }
  }
}

// Cooperative launch of prepare_kernel over [BH, seq] rows read from `src`.
template <typename Src>
int prepare(const Src& src, int64_t batch, int64_t heads, int64_t seq, float sm_scale, const Outputs& o, void* workspace,
            int64_t workspace_bytes, int* err, cudaStream_t st) {
  if (!workspace || workspace_bytes < prep_workspace(batch * heads)) return XGB_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 15u) return XGB_ERR_ALIGN;
  static int occupancy[64] = {};  // per device; the kernel's static shape fixes it
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return XGB_ERR_DEVICE;
  if (occupancy[dev] == 0) {
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, prepare_kernel<Src>, kPrepThreads, 0) !=
        cudaSuccess)
      return XGB_ERR_LAUNCH;
    occupancy[dev] = occ;
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return XGB_ERR_DEVICE;
  const int64_t cap = std::min<int64_t>(kMaxPrepCtas, static_cast<int64_t>(occupancy[dev]) * sms);
  if (cap <= 0) return XGB_ERR_LAUNCH;
  const int64_t bh = batch * heads;
  PrepShape sh;
  sh.heads = heads;
  sh.bh = bh;
  sh.seq = seq;
  sh.s_pad = (seq + 127) / 128 * 128;
  sh.n_blk = sh.s_pad / 64;
  sh.G = static_cast<int>(std::min<int64_t>(bh, cap));
  sh.P = static_cast<int>(cap / sh.G);
  sh.q_mult = sm_scale * kLog2e;
  PrepWork w = carve(workspace, bh, sh.P, err);
  if (cudaMemsetAsync(w.arrive, 0, sizeof(int), st) != cudaSuccess) return XGB_ERR_LAUNCH;
  Src s = src;
  Outputs out = o;
  void* args[] = {&s, &sh, &w, &out};
  const unsigned grid = static_cast<unsigned>(sh.G) * static_cast<unsigned>(sh.P);
  if (cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(&prepare_kernel<Src>), dim3(grid),
                                  dim3(kPrepThreads), args, 0, st) != cudaSuccess)
    return XGB_ERR_LAUNCH;
  return XGB_OK;
}

}  // namespace
}  // namespace xgb

using namespace xgb;

XGB_API int64_t xgb_sage_prepare_workspace(int64_t batch, int64_t heads, int64_t seq) {
  if (batch <= 0 || heads <= 0 || seq <= 0) return 0;
  return prep_workspace(batch * heads);
}

XGB_API int xgb_sage_prepare(const void* q, const int64_t* q_strides, const void* k,
                             const int64_t* k_strides, const void* v, const int64_t* v_strides,
                             int dtype, int64_t batch, int64_t heads, int64_t seq,
                             int64_t head_dim, float sm_scale, int8_t* q8, float* q_scale,
                             int8_t* k8, float* k_scale, uint8_t* v8, float* v_scale,
                             void* workspace, int64_t workspace_bytes, int* error_flag,
                             void* stream) {
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
  const Strides qs{q_strides[0], q_strides[1], q_strides[2]};
  const Strides ks{k_strides[0], k_strides[1], k_strides[2]};
  const Strides vs{v_strides[0], v_strides[1], v_strides[2]};
  const Outputs o{q8, q_scale, k8, k_scale, v8, v_scale};
  if (dtype == XGB_BF16) {
    using S = StridedSource<__nv_bfloat16>;
    const S src{{static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                 static_cast<const __nv_bfloat16*>(v)}, {qs, ks, vs}};
    return prepare(src, batch, heads, seq, sm_scale, o, workspace, workspace_bytes, error_flag,
                 as_stream(stream));
  }
  using S = StridedSource<__half>;
  const S src{{static_cast<const __half*>(q), static_cast<const __half*>(k), static_cast<const __half*>(v)},
              {qs, ks, vs}};
  return prepare(src, batch, heads, seq, sm_scale, o, workspace, workspace_bytes, error_flag,
                 as_stream(stream));
}

XGB_API int xgb_sage_prepare_rope(const void* q, const int64_t* q_strides, const void* k,
                                  const int64_t* k_strides, const void* v, const int64_t* v_strides,
                                  int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                                  float sm_scale, const float* cos, const float* sin, int64_t rotary,
                                  int8_t* q8, float* q_scale, int8_t* k8, float* k_scale, uint8_t* v8,
                                  float* v_scale, void* workspace, int64_t workspace_bytes,
                                  int* error_flag, void* stream) {
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
  return prepare(src, batch, heads, seq, sm_scale, o, workspace, workspace_bytes, error_flag,
                 as_stream(stream));
}

XGB_API int xgb_sage_prepare_wire(const uint8_t* payload, int64_t peers, int64_t seq,
                                  int64_t batch, int64_t heads, int64_t valid_seq,
                                  int64_t peer_padding, float sm_scale, int8_t* q8, float* q_scale,
                                  int8_t* k8, float* k_scale, uint8_t* v8, float* v_scale,
                                  void* workspace, int64_t workspace_bytes, int* error_flag,
                                  void* stream) {
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
  WireSource src{};
  src.payload = payload;
  src.batch = batch;
  src.heads = heads;
  src.peer_rows = seq * batch * heads;
  src.peer_bytes = 3 * src.peer_rows * (kD + 4) + peer_padding;
  src.div_seq = make_fastdiv(static_cast<uint32_t>(seq));
  const Outputs o{q8, q_scale, k8, k_scale, v8, v_scale};
  return prepare(src, batch, heads, valid_seq, sm_scale, o, workspace, workspace_bytes, error_flag,
                 as_stream(stream));
}
