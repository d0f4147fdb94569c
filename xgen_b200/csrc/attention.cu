// Non-causal flash attention on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the attention call of the H3 processor: `sageattn(q, k, v,
// tensor_layout="HND", is_causal=False)` for the Sage-FP8 recipe and cuDNN
// SDPA for the BF16 recipe (x_base/x_base/operator/attention.py:357-375,
// h3_sage_cuda.py:21-25, h3_dense_cuda.py:11-15).
//
// CTA = two 128-row Q tiles of one (batch, head); KV tiles of 128 keys.
//   warps 0-3  softmax for Q tile 0 (TMEM lanes 0-127)
//   warps 4-7  softmax for Q tile 1
//   warp  8    TMA producer (Q once, then a K/V ring of kStages stages)
//   warp  9    TMEM allocator + single-thread tcgen05.mma issuer
// TMEM (512 columns): S0 | S1 | O0 | O1, 128 fp32 columns each. P_i is
// written over the first columns of S_i and read by the P.V MMA straight from
// TMEM (A operand in TMEM), so P never touches shared memory.
//
// Sage variant: S = int8 Q . int8 K^T (kind::i8, s32 accumulate), scores
// dequantised per 64-row Q block x 64-key K block (sm_scale*log2e folded into
// the Q scale), P in e4m3 (x kPScale), O += P.V with e4m3 V (kind::f8f6f4,
// fp32 accumulate), per-channel V scale applied in the epilogue.
// BF16 variant: kind::f16 for both products, P in bf16.
//
// Online softmax in the exp2 domain with lazy rescaling: a row's running max
// only moves (and O is rescaled in TMEM) when a tile raises it by more than
// kTau (log2 units), so P <= 2^kTau.
//
// Ordering relies on tcgen05.mma ops issued by one thread executing in
// issue order: S_i(j+1) is issued after PV_i(j), which reads P_i(j) from the
// same TMEM columns. The commit that publishes S_i(j+1) therefore also
// certifies PV_i(j) complete, so the softmax warps may rescale O_i then.
#include <climits>

#include "sm100.cuh"
#include "tma_host.h"

namespace xgb {
namespace attn {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kQT = 2;
constexpr int kBN = 128;
constexpr int kD = 128;
constexpr int kThreads = 320;
constexpr int kTmaWarp = 8;
constexpr int kMmaWarp = 9;
constexpr float kNegInf = -__builtin_huge_valf();
// log2(448 / 2^4): e4m3 P = exp2(x + kLog2PScale) spans up to 448 under kTau = 4.
constexpr float kLog2PScale = 4.807354922057604f;

template <bool kSage>
struct Cfg {
  static constexpr int kElem = kSage ? 1 : 2;
  static constexpr int kTileBytes = kBM * kD * kElem;  // one 128x128 tile
  static constexpr int kSubTiles = kSage ? 1 : 2;      // 128-byte wide TMA boxes per tile
  static constexpr int kStages = kSage ? 4 : 2;
  static constexpr int kKSteps = kSage ? 4 : 8;        // MMA K steps over D (and over keys)
  static constexpr float kTau = kSage ? 4.0f : 8.0f;
  static constexpr float kPScale = kSage ? 448.0f / 16.0f : 1.0f;  // 448 / 2^kTau for e4m3
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQT * kTileBytes;
  static constexpr int kVOff = kKOff + kStages * kTileBytes;
  static constexpr int kBarOff = kVOff + kStages * kTileBytes;
  static constexpr int kSmem = kBarOff + 256 + 1024;  // + barriers + alignment slack
  static constexpr uint32_t kIdescQK =
      kSage ? instr_desc(2, 1, 1, false, false, kBM, kBN) : instr_desc(1, 1, 1, false, false, kBM, kBN);
  static constexpr uint32_t kIdescPV =
      kSage ? instr_desc(1, 0, 0, false, true, kBM, kD) : instr_desc(1, 1, 1, false, true, kBM, kD);
};

struct Params {
  // Sage
  const float* q_scale;
  const float* k_scale;
  const float* v_scale;
  int64_t scale_stride;  // per-head stride of q/k scale rows (= S_pad / 64)
  // common
  int heads;
  int seq_q;
  int seq_kv;
  float scale_log2;  // bf16: sm_scale * log2(e)
  __nv_bfloat16* out;
  int64_t osb, osh, oss;
  int* err;
};

struct Barriers {
  uint64_t q_full;
  uint64_t k_full[4];
  uint64_t v_full[4];
  uint64_t kv_empty[4];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_full[2];
  uint64_t end;
  uint32_t tmem_base;
};

template <bool kSage>
__device__ __forceinline__ void load_tile(const CUtensorMap* map, uint8_t* dst, uint64_t* bar,
                                          int row, int bh, int heads) {
  if constexpr (kSage) {
    tma_load_3d(dst, map, bar, 0, row, bh);
  } else {
    const int b = bh / heads, h = bh % heads;
    tma_load_4d(dst, map, bar, 0, row, h, b);
    tma_load_4d(dst + 16384, map, bar, 64, row, h, b);
  }
}

// K-major SW128 descriptor of MMA K-step `k` within a 128x128 tile.
template <bool kSage>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_saddr, int k) {
  // 32 bytes of K per step; bf16 tiles hold d 0-63 and d 64-127 in two
  // 16 KB sub-tiles.
  const uint32_t sub = kSage ? 0u : static_cast<uint32_t>(k >> 2) * 16384u;
  const uint32_t off = static_cast<uint32_t>(kSage ? k : (k & 3)) * 32u;
  return smem_desc_sw128(tile_saddr + sub + off, 16, 1024);
}

// MN-major SW128 descriptor of the V tile for MMA K-step `k` (keys).
template <bool kSage>
__device__ __forceinline__ uint64_t vdesc(uint32_t tile_saddr, int k) {
  // keys per step: 32 (e4m3) or 16 (bf16); each key row is 128 B per sub-tile.
  const uint32_t off = static_cast<uint32_t>(k) * (kSage ? 32u : 16u) * 128u;
  return smem_desc_sw128(tile_saddr + off, 16384, 1024);
}

template <bool kSage>
__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap q_map,
                     const __grid_constant__ CUtensorMap k_map,
                     const __grid_constant__ CUtensorMap v_map, const Params p) {
  using C = Cfg<kSage>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + C::kBarOff);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int m0 = blockIdx.x * (kQT * kBM);
  const int n_kv = (p.seq_kv + kBN - 1) / kBN;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], kBM);
      mbar_init(&bars->o_full[i], 1);
    }
    mbar_init(&bars->end, 1);
    fence_barrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc<512>(&bars->tmem_base);
  if (warp == kTmaWarp && lane == 0) {
    prefetch_tmap(&q_map);
    prefetch_tmap(&k_map);
    prefetch_tmap(&v_map);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == kTmaWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      bool ok = true;
      mbar_arrive_expect_tx(&bars->q_full, kQT * C::kTileBytes);
      for (int i = 0; i < kQT; ++i)
        load_tile<kSage>(&q_map, smem + C::kQOff + i * C::kTileBytes, &bars->q_full, m0 + i * kBM,
                         bh, p.heads);
      int issued = 0;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j % C::kStages;
        if (j >= C::kStages) ok = mbar_wait(&bars->kv_empty[s], ((j / C::kStages) - 1) & 1, p.err);
        if (!ok) break;
        mbar_arrive_expect_tx(&bars->k_full[s], C::kTileBytes);
        load_tile<kSage>(&k_map, smem + C::kKOff + s * C::kTileBytes, &bars->k_full[s], j * kBN, bh,
                         p.heads);
        mbar_arrive_expect_tx(&bars->v_full[s], C::kTileBytes);
        load_tile<kSage>(&v_map, smem + C::kVOff + s * C::kTileBytes, &bars->v_full[s], j * kBN, bh,
                         p.heads);
        issued = j + 1;
      }
      // Never leave with copies in flight: wait (bounded) for the last ones.
      for (int j = max(0, issued - C::kStages); j < issued; ++j) {
        const int s = j % C::kStages;
        mbar_wait(&bars->k_full[s], (j / C::kStages) & 1, p.err, 100000000ull);
        mbar_wait(&bars->v_full[s], (j / C::kStages) & 1, p.err, 100000000ull);
      }
      mbar_wait(&bars->q_full, 0, p.err, 100000000ull);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t q_saddr = smem_u32(smem + C::kQOff);
      const uint32_t k_saddr = smem_u32(smem + C::kKOff);
      const uint32_t v_saddr = smem_u32(smem + C::kVOff);
      constexpr Kind kQK = kSage ? Kind::kI8 : Kind::kF16;
      constexpr Kind kPV = kSage ? Kind::kF8F6F4 : Kind::kF16;
      bool ok = mbar_wait(&bars->q_full, 0, p.err);
      auto issue_s = [&](int i, int stage) {
        const uint32_t qa = q_saddr + i * C::kTileBytes;
        const uint32_t ka = k_saddr + stage * C::kTileBytes;
#pragma unroll
        for (int k = 0; k < C::kKSteps; ++k)
          mma_ss<kQK>(tmem + i * 128, kmajor_desc<kSage>(qa, k), kmajor_desc<kSage>(ka, k),
                      C::kIdescQK, k > 0);
        tc_commit(&bars->s_full[i]);
      };
      auto issue_pv = [&](int i, int stage, bool acc) {
        const uint32_t va = v_saddr + stage * C::kTileBytes;
#pragma unroll
        for (int k = 0; k < C::kKSteps; ++k)
          mma_ts<kPV>(tmem + 256 + i * 128, tmem + i * 128 + k * 8, vdesc<kSage>(va, k),
                      C::kIdescPV, acc || k > 0);
      };
      if (ok) {
        ok = mbar_wait(&bars->k_full[0], 0, p.err);
        if (ok) {
          tc_fence_after();
          issue_s(0, 0);
          issue_s(1, 0);
        }
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j % C::kStages;
        const uint32_t ph = (j / C::kStages) & 1;
        const int sn = (j + 1) % C::kStages;
        const uint32_t phn = ((j + 1) / C::kStages) & 1;
        ok = mbar_wait(&bars->v_full[s], ph, p.err) && mbar_wait(&bars->p_full[0], j & 1, p.err);
        if (!ok) break;
        tc_fence_after();
        issue_pv(0, s, j > 0);
        if (j + 1 < n_kv) {
          ok = mbar_wait(&bars->k_full[sn], phn, p.err);
          if (!ok) break;
          tc_fence_after();
          issue_s(0, sn);
        }
        ok = mbar_wait(&bars->p_full[1], j & 1, p.err);
        if (!ok) break;
        tc_fence_after();
        issue_pv(1, s, j > 0);
        tc_commit(&bars->kv_empty[s]);
        if (j + 1 < n_kv) issue_s(1, sn);
      }
      tc_commit(&bars->o_full[0]);
      tc_commit(&bars->o_full[1]);
      tc_commit(&bars->end);
      mbar_wait(&bars->end, 0, p.err, 100000000ull);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int i = warp >> 2;               // Q tile of this warpgroup
    const int lane_base = (warp & 3) * 32;  // TMEM lane quarter of this warp
    const int row = m0 + i * kBM + lane_base + lane;
    const uint32_t s_addr = tmem + (static_cast<uint32_t>(lane_base) << 16) + i * 128;
    const uint32_t o_addr = tmem + (static_cast<uint32_t>(lane_base) << 16) + 256 + i * 128;
    float qs = 0.f;
    if constexpr (kSage) {
      if (row < p.scale_stride * 64) qs = p.q_scale[static_cast<int64_t>(bh) * p.scale_stride + row / 64];
    }
    float m_used = kNegInf;
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[i], j & 1, p.err));
      if (!ok) break;
      tc_fence_after();
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(s_addr + c * 32, r[c]);
      tmem_ld_wait();
      // Row max of this tile, on the raw accumulators: the score scale is
      // positive, so max(scale * s) = scale * max(s) (integer max for Sage).
      const int valid = p.seq_kv - j * kBN;  // keys >= valid are padding
      const bool tail = valid < kBN;
      float comb0 = p.scale_log2, comb1 = p.scale_log2;
      float mt;
      if constexpr (kSage) {
        comb0 = qs * p.k_scale[static_cast<int64_t>(bh) * p.scale_stride + 2 * j];
        comb1 = qs * p.k_scale[static_cast<int64_t>(bh) * p.scale_stride + 2 * j + 1];
        int mx0 = INT_MIN, mx1 = INT_MIN;
        if (!tail) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            mx0 = max(mx0, max(static_cast<int>(r[0][e]), static_cast<int>(r[1][e])));
            mx1 = max(mx1, max(static_cast<int>(r[2][e]), static_cast<int>(r[3][e])));
          }
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int col = c * 32 + e;
              if (col < valid) {
                if (c < 2) mx0 = max(mx0, static_cast<int>(r[c][e]));
                else mx1 = max(mx1, static_cast<int>(r[c][e]));
              }
            }
        }
        mt = fmaxf(mx0 == INT_MIN ? kNegInf : comb0 * static_cast<float>(mx0),
                   mx1 == INT_MIN ? kNegInf : comb1 * static_cast<float>(mx1));
      } else {
        float m0 = kNegInf, m1 = kNegInf;
        if (!tail) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            m0 = fmaxf(m0, fmaxf(__uint_as_float(r[0][e]), __uint_as_float(r[1][e])));
            m1 = fmaxf(m1, fmaxf(__uint_as_float(r[2][e]), __uint_as_float(r[3][e])));
          }
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (c * 32 + e < valid) m0 = fmaxf(m0, __uint_as_float(r[c][e]));
        }
        mt = fmaxf(m0, m1) * comb0;
      }
      // Lazy rescale decision (warp-uniform TMEM traffic).
      const float m_new = fmaxf(m_used, mt);
      const bool need = m_new > m_used + C::kTau;
      if (j == 0) {
        m_used = m_new;
      } else if (__any_sync(0xffffffffu, need)) {
        const float alpha = need ? ex2_approx(m_used - m_new) : 1.0f;
        if (need) m_used = m_new;
        l *= alpha;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(o_addr + c * 32, o);
        }
        tmem_st_wait();
      }
      // P = exp2(scale*s - m_used) (times kPScale for e4m3, folded into the
      // exponent), row sum, pack and store over S.
      float rs = 0.f;
      uint32_t packed[32];
      if constexpr (kSage) {
        // exp2 on packed halves: the f16 argument keeps ~1e-3 relative
        // accuracy for |x| < 16, finer than the e4m3 P it feeds.
        const float off = kLog2PScale - m_used;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float comb = c < 2 ? comb0 : comb1;
          // f16x2 partial sums over 8 pairs each (<= 8 * 448), then fp32.
          __half2 hsum0 = __float2half2_rn(0.f), hsum1 = hsum0;
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            float x[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              x[t] = fmaf(static_cast<float>(static_cast<int>(r[c][e + t])), comb, off);
              if (tail && c * 32 + e + t >= valid) x[t] = kNegInf;
            }
            const uint32_t e01 = ex2_f16x2(pack_f16x2(x[0], x[1]));
            const uint32_t e23 = ex2_f16x2(pack_f16x2(x[2], x[3]));
            hsum0 = __hadd2(hsum0, *reinterpret_cast<const __half2*>(&e01));
            hsum1 = __hadd2(hsum1, *reinterpret_cast<const __half2*>(&e23));
            packed[c * 8 + e / 4] = e4m3x2_from_f16x2(e01) | (e4m3x2_from_f16x2(e23) << 16);
          }
          const float2 f0 = __half22float2(hsum0), f1 = __half22float2(hsum1);
          rs += (f0.x + f0.y) + (f1.x + f1.y);
        }
        tmem_st32(s_addr, packed);
      } else {
        const float off = -m_used;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const int col = (half * 2 + c) * 32 + e;
              float xa = fmaf(__uint_as_float(r[half * 2 + c][e]), comb0, off);
              float xb = fmaf(__uint_as_float(r[half * 2 + c][e + 1]), comb0, off);
              if (tail) {
                if (col >= valid) xa = kNegInf;
                if (col + 1 >= valid) xb = kNegInf;
              }
              const float a = ex2_approx(xa);
              const float b = ex2_approx(xb);
              rs += a + b;
              packed[c * 16 + e / 2] = pack_bf16x2(a, b);
            }
          }
          tmem_st32(s_addr + half * 32, packed);
        }
      }
      l += rs;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars->p_full[i]);
    }
    // ------------------------------------------------------------ epilogue
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_full[i], 0, p.err));
    if (ok) {
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.0f / l : 0.f;
      const int b = bh / p.heads, h = bh % p.heads;
      __nv_bfloat16* dst = p.out + b * p.osb + h * p.osh + static_cast<int64_t>(row) * p.oss;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(o_addr + c * 32, o);
        tmem_ld_wait();
        if (row < p.seq_q) {
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float x0 = __uint_as_float(o[e]) * inv_l;
            float x1 = __uint_as_float(o[e + 1]) * inv_l;
            if constexpr (kSage) {  // l sums the same kPScale-scaled P
              x0 *= p.v_scale[static_cast<int64_t>(bh) * kD + c * 32 + e];
              x1 *= p.v_scale[static_cast<int64_t>(bh) * kD + c * 32 + e + 1];
            }
            w[e / 2] = pack_bf16x2(x0, x1);
          }
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) d4[v] = make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

inline bool aligned(const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; }

template <bool kSage>
int launch(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const Params& p,
           int64_t bh, cudaStream_t st) {
  using C = Cfg<kSage>;
  auto kernel = attention_kernel<kSage>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) !=
      cudaSuccess)
    return XGB_ERR_LAUNCH;
  dim3 grid(static_cast<unsigned>((p.seq_q + kQT * kBM - 1) / (kQT * kBM)),
            static_cast<unsigned>(bh));
  kernel<<<grid, kThreads, C::kSmem, st>>>(qm, km, vm, p);
  return launch_status();
}

int check_device() {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return XGB_ERR_DEVICE;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return XGB_ERR_DEVICE;
  return major == 10 ? XGB_OK : XGB_ERR_DEVICE;
}

}  // namespace attn
}  // namespace xgb

using namespace xgb;
using namespace xgb::attn;

XGB_API int xgb_attention_sage(const int8_t* q8, const float* q_scale, const int8_t* k8,
                               const float* k_scale, const uint8_t* v8, const float* v_scale,
                               int64_t batch, int64_t heads, int64_t seq, void* out,
                               const int64_t* out_strides, int* error_flag, void* stream) {
  if (!q8 || !q_scale || !k8 || !k_scale || !v8 || !v_scale || !out || !out_strides)
    return XGB_ERR_ARG;
  if (batch <= 0 || heads <= 0 || seq <= 0 || seq > (1 << 30) || batch * heads > 65535)
    return XGB_ERR_SHAPE;
  if (out_strides[3] != 1 || out_strides[2] % 8 || out_strides[1] % 8 || out_strides[0] % 8)
    return XGB_ERR_STRIDE;
  if (!aligned(q8, 16) || !aligned(k8, 16) || !aligned(v8, 16) || !aligned(out, 16))
    return XGB_ERR_ALIGN;
  int rc = check_device();
  if (rc) return rc;
  const int64_t s_pad = (seq + 127) / 128 * 128;
  const int64_t bh = batch * heads;
  CUtensorMap qm, km, vm;
  const uint64_t dims[3] = {static_cast<uint64_t>(kD), static_cast<uint64_t>(s_pad),
                            static_cast<uint64_t>(bh)};
  const uint64_t strides[2] = {static_cast<uint64_t>(kD), static_cast<uint64_t>(s_pad * kD)};
  const uint32_t box[3] = {128, 128, 1};
  if (!make_tensor_map(&qm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, q8, dims, strides, box) ||
      !make_tensor_map(&km, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, k8, dims, strides, box) ||
      !make_tensor_map(&vm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, v8, dims, strides, box))
    return XGB_ERR_ALIGN;
  Params p{};
  p.q_scale = q_scale;
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.scale_stride = s_pad / 64;
  p.heads = static_cast<int>(heads);
  p.seq_q = static_cast<int>(seq);
  p.seq_kv = static_cast<int>(seq);
  p.scale_log2 = 1.0f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.osb = out_strides[0];
  p.osh = out_strides[1];
  p.oss = out_strides[2];
  p.err = error_flag;
  return launch<true>(qm, km, vm, p, bh, as_stream(stream));
}

XGB_API int xgb_attention_bf16(const void* q, const int64_t* q_strides, const void* k,
                               const int64_t* k_strides, const void* v, const int64_t* v_strides,
                               int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_kv,
                               float sm_scale, void* out, const int64_t* out_strides,
                               int* error_flag, void* stream) {
  if (!q || !k || !v || !out || !q_strides || !k_strides || !v_strides || !out_strides)
    return XGB_ERR_ARG;
  if (batch <= 0 || heads <= 0 || seq_q <= 0 || seq_kv <= 0 || seq_q > (1 << 30) ||
      seq_kv > (1 << 30) || batch * heads > 65535)
    return XGB_ERR_SHAPE;
  if (!(sm_scale > 0.f)) return XGB_ERR_ARG;
  const int64_t* all[4] = {q_strides, k_strides, v_strides, out_strides};
  for (auto s : all) {
    if (s[3] != 1) return XGB_ERR_STRIDE;
    for (int d = 0; d < 3; ++d)
      if (s[d] % 8 || s[d] <= 0) return XGB_ERR_STRIDE;  // 16-byte TMA strides
  }
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16))
    return XGB_ERR_ALIGN;
  int rc = check_device();
  if (rc) return rc;
  CUtensorMap qm, km, vm;
  const uint32_t box[4] = {64, 128, 1, 1};
  auto make = [&](CUtensorMap* m, const void* base, const int64_t* s, int64_t seq) {
    const uint64_t dims[4] = {static_cast<uint64_t>(kD), static_cast<uint64_t>(seq),
                              static_cast<uint64_t>(heads), static_cast<uint64_t>(batch)};
    const uint64_t strides[3] = {static_cast<uint64_t>(s[2]) * 2, static_cast<uint64_t>(s[1]) * 2,
                                 static_cast<uint64_t>(s[0]) * 2};
    return make_tensor_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box);
  };
  if (!make(&qm, q, q_strides, seq_q) || !make(&km, k, k_strides, seq_kv) ||
      !make(&vm, v, v_strides, seq_kv))
    return XGB_ERR_ALIGN;
  Params p{};
  p.heads = static_cast<int>(heads);
  p.seq_q = static_cast<int>(seq_q);
  p.seq_kv = static_cast<int>(seq_kv);
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.osb = out_strides[0];
  p.osh = out_strides[1];
  p.oss = out_strides[2];
  p.err = error_flag;
  return launch<false>(qm, km, vm, p, batch * heads, as_stream(stream));
}
