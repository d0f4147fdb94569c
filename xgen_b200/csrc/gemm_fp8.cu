// FP8 (e4m3) GEMM on sm_100a tensor cores for the H3 FP8 Linear layers.
//
//   out[m, n] = bf16(acc[m, n] * (sa[m] * sb[n]) + bias[n])        (plain)
//   out[m, n] = bf16(bf16(y * gate[idx[m], n]) + residual[m, n])    (gated)
//       with y = the plain result, the AdaLN gate + residual of the block
//   out[m, j] = bf16(bf16(silu(yg)) * yv)                              (SwiGLU)
//       with yg, yv = bf16 plain results of the gate and value columns of
//       the gate-first SwiGLU (x_base/x_base/operator/h3_swiglu.py:15-29):
//       W rows interleaved in groups of 128, [gate j..j+127 | value
//       j..j+127] per 256-row tile, so one tile yields 128 outputs
//
// acc = sum_k A[m, k] * W[n, k] in fp32 (tcgen05 kind::f8f6f4), A [M, K] and
// W [N, K] e4m3 row-major (both K-major), sa/sb per-row/per-column scales
// or broadcast scalars (stride 0), bias optional. Replaces torch._scaled_mm
// in H3FP8Linear._local_forward (x_base/x_base/operator/h3_fp8.py:48-68) and,
// in the gated form, the `_apply(..., modulation=False)` that follows the
// attention/FFN output projections (x_base/x_base/operator/h3_indexed_affine.py
// :52-61), with the reference's rounding after each eager op.
//
// Persistent kernel, one CTA per SM, tiles of 128 x 256 (M x N), K blocks
// of 128 bytes:
//   warp 0     TMA producer (A 16 KB + W 32 KB per stage, 4 stages)
//   warp 1     TMEM allocator + MMA issuer (4 x M128 N256 K32 per stage)
//   warps 2-9  epilogue: one thread per output row (TMEM lane) and column
//              half (warps 2-5 columns 0-127, warps 6-9 columns 128-255),
//              fp32 read in chunks of 32 columns; per-column scales, bias,
//              AdaLN gate and residual move as 16-byte vectors
// Two TMEM accumulators (2 x 256 columns) let the epilogue of one tile run
// under the MMAs of the next. Every mbarrier wait is bounded.
#include <atomic>
#include <cstdlib>

#include "sm100.cuh"
#include "tma_host.h"

namespace xgb {
namespace gemm {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 128;  // bytes of K per stage (e4m3)
constexpr int kStages = 4;
constexpr int kThreads = 320;
constexpr int kEpiThreads = 256;
constexpr int kABytes = kBM * kBK;
constexpr int kBBytes = kBN * kBK;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kBarOff = kStages * kStageBytes;
constexpr int kSmem = kBarOff + 256 + 1024;
constexpr uint32_t kIdesc = instr_desc(1, 0, 0, false, false, kBM, kBN);

enum Epilogue : int { kPlain = 0, kGated = 1, kGeluErf = 2, kGeluTanh = 3, kSwiGLU = 4 };

// GELU of the FFN up projection: exact (erf) or the tanh approximation.
__device__ __forceinline__ float gelu_erf(float y) { return 0.5f * y * (1.0f + erff(y * 0.70710678118654752f)); }
__device__ __forceinline__ float gelu_tanh(float y) {
  return 0.5f * y * (1.0f + tanhf(0.79788456080286536f * (y + 0.044715f * y * y * y)));
}
// Gate-first SwiGLU of one bf16 gate/value pair with the reference's
// rounding: act = bf16(g / (1 + exp(-g))), out = bf16(act * v).
__device__ __forceinline__ float swiglu_pair(float g, float v) {
  const float act = bf16_round(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))));
  return bf16_round(__fmul_rn(act, v));
}

struct Params {
  int M, N, K;
  const float* sa;
  int64_t sa_stride;  // 0: per-tensor scalar, 1: per row
  const float* sb;
  int64_t sb_stride;  // 0: per-tensor scalar, 1: per column
  const __nv_bfloat16* bias;  // may be null
  __nv_bfloat16* out;
  int64_t ldo;
  // gated epilogue
  const __nv_bfloat16* gate;  // rows of the AdaLN table, row stride ldg
  int64_t ldg;
  const int64_t* idx;         // [M] table row of each output row
  const __nv_bfloat16* residual;
  int64_t ldr;
  int* err;
  bool vec;  // 16-byte aligned scale/bias/gate/residual columns (host-checked)
};

struct Barriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t end;
  uint32_t tmem_base;
};

// One accumulator tile's epilogue for the output row `m` this thread owns
// (its TMEM lane) and the column half `half`: reads the fp32 accumulators at
// TMEM address `acc` and writes the bf16 outputs with the kEpi epilogue.
template <int kEpi>
__device__ __forceinline__ void epilogue_tile(const Params& p, uint32_t acc, int m, int n0, int half) {
  const bool row_ok = m < p.M;
  const float sa = row_ok ? p.sa[m * p.sa_stride] : 0.f;
  const int64_t grow = (kEpi == kGated && row_ok) ? p.idx[m] : 0;
  if constexpr (kEpi == kSwiGLU) {
    // N % 256 == 0 (checked on the host): gate columns n0 + [0, 128),
    // value columns n0 + [128, 256), outputs n0/2 + [0, 128).
#pragma unroll 1
    for (int c = half * (kBN / 128); c < (half + 1) * (kBN / 128); ++c) {
      uint32_t rg[32], rv[32];
      tmem_ld32(acc + c * 32, rg);
      tmem_ld32(acc + kBN / 2 + c * 32, rv);
      tmem_ld_wait();
      if (row_ok) {
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float y[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int ng = n0 + c * 32 + e + u, nv = ng + kBN / 2;
            const float bg = p.bias ? __bfloat162float(p.bias[ng]) : 0.f;
            const float bv = p.bias ? __bfloat162float(p.bias[nv]) : 0.f;
            const float g = bf16_round(fmaf(__uint_as_float(rg[e + u]), sa * p.sb[ng * p.sb_stride], bg));
            const float v = bf16_round(fmaf(__uint_as_float(rv[e + u]), sa * p.sb[nv * p.sb_stride], bv));
            y[u] = swiglu_pair(g, v);
          }
          w[e / 2] = pack_bf16x2(y[0], y[1]);
        }
        uint4* d4 = reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(m) * p.ldo + n0 / 2 + c * 32);
#pragma unroll
        for (int v = 0; v < 4; ++v) d4[v] = make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
      }
    }
  } else {
#pragma unroll 1
    for (int c = half * (kBN / 64); c < (half + 1) * (kBN / 64); ++c) {
      uint32_t r[32];
      tmem_ld32(acc + c * 32, r);
      tmem_ld_wait();
      const int nb = n0 + c * 32;
      if (row_ok && p.vec && nb + 32 <= p.N) {
        // 8 columns at a time: scales, bias, gate row and residual as vectors
        __nv_bfloat16* dst = p.out + static_cast<int64_t>(m) * p.ldo + nb;
#pragma unroll
        for (int g8 = 0; g8 < 4; ++g8) {
          const int n = nb + g8 * 8;
          float alpha[8], bias[8], y[8];
          if (p.sb_stride) {
            const float4 b0 = __ldg(reinterpret_cast<const float4*>(p.sb + n));
            const float4 b1 = __ldg(reinterpret_cast<const float4*>(p.sb + n + 4));
            alpha[0] = sa * b0.x; alpha[1] = sa * b0.y; alpha[2] = sa * b0.z; alpha[3] = sa * b0.w;
            alpha[4] = sa * b1.x; alpha[5] = sa * b1.y; alpha[6] = sa * b1.z; alpha[7] = sa * b1.w;
          } else {
            const float al = sa * p.sb[0];
#pragma unroll
            for (int i = 0; i < 8; ++i) alpha[i] = al;
          }
          if (p.bias) {
            unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(p.bias + n)), bias);
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) bias[i] = 0.f;
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            y[i] = fmaf(__uint_as_float(r[g8 * 8 + i]), alpha[i], bias[i]);
            if constexpr (kEpi == kGeluErf) y[i] = gelu_erf(y[i]);
            if constexpr (kEpi == kGeluTanh) y[i] = gelu_tanh(y[i]);
          }
          if constexpr (kEpi == kGated) {
            // reference: attn = bf16(GEMM); x = bf16(bf16(attn*gate) + res)
            float gt[8], res[8];
            unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(p.gate + grow * p.ldg + n)), gt);
            unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(p.residual + static_cast<int64_t>(m) * p.ldr + n)), res);
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = __fadd_rn(bf16_round(__fmul_rn(bf16_round(y[i]), gt[i])), res[i]);
          }
          reinterpret_cast<uint4*>(dst)[g8] =
              make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                         pack_bf16x2(y[6], y[7]));
        }
      } else if (row_ok && nb < p.N) {
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float y[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int n = min(nb + e + u, p.N - 1);
            const float alpha = sa * p.sb[n * p.sb_stride];
            const float bias = p.bias ? __bfloat162float(p.bias[n]) : 0.f;
            y[u] = fmaf(__uint_as_float(r[e + u]), alpha, bias);
            if constexpr (kEpi == kGeluErf) y[u] = gelu_erf(y[u]);
            if constexpr (kEpi == kGeluTanh) y[u] = gelu_tanh(y[u]);
            if constexpr (kEpi == kGated) {
              // reference: attn = bf16(GEMM); x = bf16(bf16(attn*gate) + res)
              const float g = __bfloat162float(p.gate[grow * p.ldg + n]);
              const float res = __bfloat162float(p.residual[static_cast<int64_t>(m) * p.ldr + n]);
              y[u] = __fadd_rn(bf16_round(__fmul_rn(bf16_round(y[u]), g)), res);
            }
          }
          w[e / 2] = pack_bf16x2(y[0], y[1]);
        }
        __nv_bfloat16* dst = p.out + static_cast<int64_t>(m) * p.ldo + nb;
        if (nb + 32 <= p.N) {
          uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
          for (int v = 0; v < 4; ++v) d4[v] = make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
        } else {
          const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(w);
          for (int e = 0; e < p.N - nb; ++e) dst[e] = wb[e];
        }
      }
    }
  }
}

template <int kEpi>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap a_map,
                    const __grid_constant__ CUtensorMap b_map, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kBarOff);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (p.M + kBM - 1) / kBM;
  const int n_tiles = (p.N + kBN - 1) / kBN;
  const int tiles = m_tiles * n_tiles;
  const int k_blocks = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->acc_full[a], 1);
      mbar_init(&bars->acc_empty[a], kEpiThreads);
    }
    mbar_init(&bars->end, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc<512>(&bars->tmem_base);
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&a_map);
    prefetch_tmap(&b_map);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      bool ok = true;
      int it = 0;  // global k-block counter of this CTA
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int m0 = (t / n_tiles) * kBM;
        const int n0 = (t % n_tiles) * kBN;
        for (int kb = 0; kb < k_blocks && ok; ++kb, ++it) {
          const int s = it % kStages;
          if (it >= kStages) ok = mbar_wait(&bars->empty[s], ((it / kStages) - 1) & 1, p.err);
          if (!ok) break;
          uint8_t* st = smem + s * kStageBytes;
          mbar_arrive_expect_tx(&bars->full[s], kStageBytes);
          tma_load_2d(st, &a_map, &bars->full[s], kb * kBK, m0);
          tma_load_2d(st + kABytes, &b_map, &bars->full[s], kb * kBK, n0);
        }
      }
      // drain: the last stages' copies must land before the CTA exits
      for (int j = max(0, it - kStages); j < it; ++j)
        mbar_wait(&bars->full[j % kStages], (j / kStages) & 1, p.err, 100000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = true;
      int it = 0, lt = 0;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++lt) {
        const int a = lt & 1;
        if (lt >= 2) ok = mbar_wait(&bars->acc_empty[a], ((lt >> 1) - 1) & 1, p.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + a * kBN;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          ok = mbar_wait(&bars->full[s], (it / kStages) & 1, p.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t as = smem_u32(smem + s * kStageBytes);
          const uint32_t bs = as + kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k)
            mma_ss<Kind::kF8F6F4>(d, smem_desc_sw128(as + k * 32, 16, 1024),
                                  smem_desc_sw128(bs + k * 32, 16, 1024), kIdesc, kb > 0 || k > 0);
          tc_commit(&bars->empty[s]);
        }
        if (!ok) break;
        tc_commit(&bars->acc_full[a]);
      }
      tc_commit(&bars->end);
      mbar_wait(&bars->end, 0, p.err, 100000000ull);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;       // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;   // column half of the tile
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    int lt = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++lt) {
      const int a = lt & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&bars->acc_full[a], (lt >> 1) & 1, p.err));
      if (!ok) break;
      tc_fence_after();
      const int m = (t / n_tiles) * kBM + quarter * 32 + lane;
      const int n0 = (t % n_tiles) * kBN;
      epilogue_tile<kEpi>(p, lane_addr + a * kBN, m, n0, half);
      tc_fence_before();
      mbar_arrive(&bars->acc_empty[a]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

// ---------------------------------------------------------------- CTA pairs
// The same GEMM on CTA pairs (cta_group::2): a pair computes a 256 x 256
// tile with M256 N256 K32 MMAs issued by rank 0. Each CTA loads its own 128
// rows of A and its own 128 of the tile's 256 W rows per stage (32 KB), so
// a pair moves 64 KB per k-block for twice the work of one 1-CTA stage
// (48 KB): per SM a third less L2-to-SM traffic, and 7 stages (224 KB) in flight.
// Each CTA's TMEM holds its 128 output rows x 256 columns, so the epilogue
// is the 1-CTA one on rows m0 + 128 * rank.
//
// Pair protocol (every wait bounded):
//   full[s]      rank 0 only: rank 0's producer expects 64 KB, both CTAs'
//                TMA loads count their bytes on it
//   empty[s]     per CTA: the MMA commits to both CTAs' barriers
//   acc_full[a]  per CTA: the MMA commits to both
//   acc_empty[a] rank 0: 16 arrivals, one per epilogue warp of both CTAs
//   end          per CTA: the MMA's last commit; TMEM is freed after it
// A cluster barrier after the barrier inits and one before exit keep both
// CTAs alive while the other may still signal them.
constexpr int kPairStages = 7;
constexpr int kPairRows = 128;                      // A rows and W rows per CTA
constexpr int kPairABytes = kPairRows * kBK;        // 16 KB
constexpr int kPairStageBytes = 2 * kPairRows * kBK;  // 32 KB
constexpr int kPairBarOff = kPairStages * kPairStageBytes;
constexpr int kPairSmem = kPairBarOff + 256 + 1024;
constexpr uint32_t kPairIdesc = instr_desc(1, 0, 0, false, false, 2 * kPairRows, kBN);

struct PairBarriers {
  uint64_t full[kPairStages];
  uint64_t empty[kPairStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t end;
  uint32_t tmem_base;
};

template <int kEpi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_fp8_pair_kernel(const __grid_constant__ CUtensorMap a_map,
                         const __grid_constant__ CUtensorMap b_map, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  PairBarriers* bars = reinterpret_cast<PairBarriers*>(smem + kPairBarOff);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;
  const int m_tiles = (p.M + 2 * kPairRows - 1) / (2 * kPairRows);
  const int n_tiles = (p.N + kBN - 1) / kBN;
  const int tiles = m_tiles * n_tiles;
  const int k_blocks = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->acc_full[a], 1);
      mbar_init(&bars->acc_empty[a], 2 * (kEpiThreads / 32));
    }
    mbar_init(&bars->end, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair<512>(&bars->tmem_base);
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&a_map);
    prefetch_tmap(&b_map);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producers (both CTAs)
    if (lane == 0) {
      bool ok = true;
      int it = 0;
      for (int t = pair; t < tiles && ok; t += pairs) {
        const int m0 = (t / n_tiles) * 2 * kPairRows + static_cast<int>(rank) * kPairRows;
        const int n0 = (t % n_tiles) * kBN + static_cast<int>(rank) * kPairRows;
        for (int kb = 0; kb < k_blocks && ok; ++kb, ++it) {
          const int s = it % kPairStages;
          if (it >= kPairStages) ok = mbar_wait(&bars->empty[s], ((it / kPairStages) - 1) & 1, p.err);
          if (!ok) break;
          uint8_t* st = smem + s * kPairStageBytes;
          const uint32_t full0 = map_to_rank(&bars->full[s], 0);
          if (rank == 0) mbar_arrive_expect_tx(&bars->full[s], 2 * kPairStageBytes);
          tma_load_2d_pair(st, &a_map, full0, kb * kBK, m0);
          tma_load_2d_pair(st + kPairABytes, &b_map, full0, kb * kBK, n0);
        }
      }
      // After a timed-out wait, rank 0 drains the stages it armed before the
      // CTAs leave: their full barrier completes only once both CTAs' loads
      // have landed (bounded, like every wait). On the normal path the MMA
      // issuer has consumed every stage, so these waits return at once.
      if (!ok && rank == 0) {
        for (int i = max(0, it - kPairStages); i < it; ++i)
          mbar_wait(&bars->full[i % kPairStages], (i / kPairStages) & 1, nullptr, 100000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (rank 0)
    if (lane == 0 && rank == 0) {
      bool ok = true;
      int it = 0, lt = 0;
      for (int t = pair; t < tiles && ok; t += pairs, ++lt) {
        const int a = lt & 1;
        if (lt >= 2) ok = mbar_wait(&bars->acc_empty[a], ((lt >> 1) - 1) & 1, p.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + a * kBN;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % kPairStages;
          ok = mbar_wait(&bars->full[s], (it / kPairStages) & 1, p.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t as = smem_u32(smem + s * kPairStageBytes);
          const uint32_t bs = as + kPairABytes;
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k)
            mma_pair_f8f6f4(d, smem_desc_sw128(as + k * 32, 16, 1024),
                            smem_desc_sw128(bs + k * 32, 16, 1024), kPairIdesc, kb > 0 || k > 0);
          tc_commit_pair(map_to_rank(&bars->empty[s], 0));
          tc_commit_pair(map_to_rank(&bars->empty[s], 1));
        }
        if (!ok) break;
        tc_commit_pair(map_to_rank(&bars->acc_full[a], 0));
        tc_commit_pair(map_to_rank(&bars->acc_full[a], 1));
      }
      tc_commit_pair(map_to_rank(&bars->end, 0));
      tc_commit_pair(map_to_rank(&bars->end, 1));
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    int lt = 0;
    for (int t = pair; t < tiles; t += pairs, ++lt) {
      const int a = lt & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&bars->acc_full[a], (lt >> 1) & 1, p.err));
      if (!ok) break;
      tc_fence_after();
      const int m = (t / n_tiles) * 2 * kPairRows + static_cast<int>(rank) * kPairRows + quarter * 32 + lane;
      const int n0 = (t % n_tiles) * kBN;
      epilogue_tile<kEpi>(p, lane_addr + a * kBN, m, n0, half);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_rank(&bars->acc_empty[a], 0));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // every pair MMA (which reads both CTAs' shared memory) has ended
    mbar_wait(&bars->end, 0, p.err, 100000000ull);
    tc_fence_after();
    tmem_dealloc_pair<512>(tmem);
  }
  cluster_sync();
}

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// CTA pairs are used for M > 128 unless XGB_GEMM_CTA_PAIRS=0 (read per call).
bool pairs_enabled() {
  const char* v = std::getenv("XGB_GEMM_CTA_PAIRS");
  return !(v && v[0] == '0');
}

// Pairs of this kernel that can be resident at once (0 if the pair launch is
// unavailable): the persistent grid is sized to it so no pair waits for
// another to finish.
template <int kEpi>
int pair_slots() {
  auto kernel = gemm_fp8_pair_kernel<kEpi>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmem) != cudaSuccess)
    return 0;
  // Measured once per epilogue instantiation and device (its register and
  // shared-memory use set the occupancy); stored as clusters + 1, 0 = not yet.
  constexpr int kMaxDevices = 64;
  static std::atomic<int> cached[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  const int known = cached[dev].load(std::memory_order_relaxed);
  if (known > 0) return known - 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * static_cast<unsigned>(sm_count()));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPairSmem;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    clusters = 0;
  }
  cached[dev].store(clusters + 1, std::memory_order_relaxed);
  return clusters;
}

template <int kEpi>
int launch(const void* a, const void* w, const Params& p, cudaStream_t st) {
  CUtensorMap am, bm;
  const uint64_t adims[2] = {static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.M)};
  const uint64_t astr[1] = {static_cast<uint64_t>(p.K)};
  const uint32_t abox[2] = {kBK, kBM};
  const uint64_t bdims[2] = {static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.N)};
  const uint32_t bbox[2] = {kBK, kBN};
  if (!make_tensor_map(&am, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a, adims, astr, abox) ||
      !make_tensor_map(&bm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w, bdims, astr, bbox))
    return XGB_ERR_ALIGN;
  if (p.M > kBM && pairs_enabled()) {
    // CTA pairs: W tiles of 128 rows per CTA
    CUtensorMap bm2;
    const uint32_t bbox2[2] = {kBK, kPairRows};
    if (!make_tensor_map(&bm2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w, bdims, astr, bbox2))
      return XGB_ERR_ALIGN;
    auto kernel = gemm_fp8_pair_kernel<kEpi>;
    const int max_pairs = pair_slots<kEpi>();
    if (max_pairs > 0) {
      const int tiles = ((p.M + 2 * kPairRows - 1) / (2 * kPairRows)) * ((p.N + kBN - 1) / kBN);
      const int grid = 2 * std::min(tiles, max_pairs);
      kernel<<<grid, kThreads, kPairSmem, st>>>(am, bm2, p);
      return launch_status();
    }
  }
  auto kernel = gemm_fp8_kernel<kEpi>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
    return XGB_ERR_LAUNCH;
  const int tiles = ((p.M + kBM - 1) / kBM) * ((p.N + kBN - 1) / kBN);
  const int grid = std::min(tiles, sm_count());
  kernel<<<grid, kThreads, kSmem, st>>>(am, bm, p);
  return launch_status();
}

}  // namespace gemm
}  // namespace xgb

using namespace xgb;

XGB_API int xgb_fp8_gemm(const uint8_t* a, const uint8_t* w, int64_t M, int64_t N, int64_t K,
                         const float* scale_a, int64_t scale_a_stride, const float* scale_w,
                         int64_t scale_w_stride, const void* bias, int activation, void* out,
                         int64_t ldo,
                         const void* gate, int64_t ldg, const int64_t* gate_index,
                         const void* residual, int64_t ldr, int* error_flag, void* stream) {
  if (!a || !w || !scale_a || !scale_w || !out) return XGB_ERR_ARG;
  if (M <= 0 || N <= 0 || K <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return XGB_ERR_SHAPE;
  if (K % 16 || N % 16) return XGB_ERR_SHAPE;  // 16-byte TMA rows, as the reference requires
  if ((scale_a_stride != 0 && scale_a_stride != 1) || (scale_w_stride != 0 && scale_w_stride != 1))
    return XGB_ERR_STRIDE;
  const bool swiglu = activation == 3;
  if (swiglu && N % 256) return XGB_ERR_SHAPE;  // whole gate/value groups per tile
  if (ldo < (swiglu ? N / 2 : N) || ldo % 8) return XGB_ERR_STRIDE;
  const bool gated = gate != nullptr;
  if (gated && (!gate_index || !residual || ldr < N || ldg < N)) return XGB_ERR_ARG;
  if (activation < 0 || activation > 3 || (gated && activation != 0)) return XGB_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w) |
       reinterpret_cast<uintptr_t>(out)) & 15u)
    return XGB_ERR_ALIGN;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      major != 10)
    return XGB_ERR_DEVICE;
  gemm::Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.sa = scale_a;
  p.sa_stride = scale_a_stride;
  p.sb = scale_w;
  p.sb_stride = scale_w_stride;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.gate = static_cast<const __nv_bfloat16*>(gate);
  p.ldg = ldg;
  p.idx = gate_index;
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.ldr = ldr;
  p.err = error_flag;
  const auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  p.vec = (scale_w_stride == 0 || a16(scale_w)) && (!bias || a16(bias)) &&
          (!gated || (a16(gate) && a16(residual) && ldg % 8 == 0 && ldr % 8 == 0));
  cudaStream_t st = as_stream(stream);
  if (gated) return gemm::launch<gemm::kGated>(a, w, p, st);
  if (activation == 1) return gemm::launch<gemm::kGeluErf>(a, w, p, st);
  if (activation == 2) return gemm::launch<gemm::kGeluTanh>(a, w, p, st);
  if (activation == 3) return gemm::launch<gemm::kSwiGLU>(a, w, p, st);
  return gemm::launch<gemm::kPlain>(a, w, p, st);
}
