// Non-causal flash attention on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the attention call of the H3 processor: `sageattn(q, k, v,
// tensor_layout="HND", is_causal=False)` for the Sage-FP8 recipe and cuDNN
// SDPA for the BF16 recipe (x_base/x_base/operator/attention.py:357-375,
// h3_sage_cuda.py:21-25, h3_dense_cuda.py:11-15).
//
// CTA = two 128-row Q tiles of one (batch, head); KV tiles of 64 keys.
//   warps 0-3  softmax for Q tile 0 (TMEM lanes 0-127)
//   warps 4-7  softmax for Q tile 1
//   warp  8    TMA producer (Q once, then a K/V ring of kStages stages)
//   warp  9    TMEM allocator + tcgen05.mma issuer for Q tile 0
//   warp 10    tcgen05.mma issuer for Q tile 1 (independent streams, so one
//              tile's S(t+2) never waits on the other tile's softmax)
// TMEM (512 columns): S0a | S0b | S1a | S1b (64 fp32 columns each) | O0 | O1
// (128 each). Each Q tile double-buffers S: while its softmax works on KV
// tile t (buffer t%2) the tensor core already holds S(t+1) in the other
// buffer and computes S(t+2) once PV(t) has consumed P(t). P(t) is written
// over the first columns of its S buffer and read by the P.V MMA straight
// from TMEM (A operand in TMEM), so P never touches shared memory.
//
// Sage variant: S = int8 Q . int8 K^T (kind::i8, s32 accumulate), scores
// dequantised per 64-row Q block x 64-key K block (sm_scale*log2e folded into
// the Q scale), P in e4m3 (x kPScale), O += P.V with e4m3 V (kind::f8f6f4,
// fp32 accumulate), per-channel V scale applied in the epilogue.
// BF16 variant: kind::f16 for both products, P in bf16.
//
// Online softmax in the exp2 domain with lazy rescaling: a row's running max
// only moves (and O is rescaled in TMEM) when a tile raises it by more than
// kTau (log2 units), so P <= 2^kTau. A rescale first waits for the previous
// tile's P.V (pv_done) so O is stable: when S(t) is visible, PV(t-2) has
// completed, so pv_done is at most one phase behind and its parity wait is
// exact.
//
// Ordering relies on tcgen05.mma ops issued by one thread executing in
// issue order: S_i(t+2) is issued by tile i's issuer after PV_i(t), which
// reads P_i(t) from the same TMEM columns.
#include <climits>

#include "sm100.cuh"
#include "tma_host.h"

namespace xgb {
namespace attn {

using namespace sm100;

constexpr int kBM = 128;  // rows per Q tile
constexpr int kQT = 2;    // Q tiles per CTA
constexpr int kBN = 64;   // keys per KV tile
constexpr int kD = 128;
constexpr int kThreads = 352;
constexpr int kTmaWarp = 8;
constexpr int kMmaWarp = 9;  // warps 9 and 10 issue the MMAs of Q tiles 0 and 1
constexpr float kNegInf = -__builtin_huge_valf();
// log2(448 / 2^4): e4m3 P = exp2(x + kLog2PScale) spans up to 448 under kTau = 4.
constexpr float kLog2PScale = 4.807354922057604f;
// One pair of exp2 in kPolyPairs runs as a packed fp32x2 polynomial
// (ex2_poly2) on the FMA pipe instead of two MUFU ops in the Sage kernel,
// easing the MUFU load of the exp section a little. Measured on B200
// (768P-5s, accumulator init on): 1 in 6 pairs is best (1,526 TFLOP/s at 24
// heads against 1,490 for 1 in 8, 1,491 for 1 in 4, 1,477 for 1 in 3);
// larger shares lose, because the exp section is bound by issue and
// dependency latency rather than by MUFU throughput. 0 disables it.
#ifndef XGB_ATTN_POLY_PAIRS
#define XGB_ATTN_POLY_PAIRS 6
#endif
constexpr int kPolyPairs = XGB_ATTN_POLY_PAIRS;
__device__ __forceinline__ bool poly_pair(int pair) {
  return kPolyPairs > 0 && pair % (kPolyPairs > 0 ? kPolyPairs : 1) == kPolyPairs - 1;
}
#ifndef XGB_ATTN_TURN
#define XGB_ATTN_TURN 1
#endif
constexpr bool kTurn = XGB_ATTN_TURN != 0;
// Sage S accumulators start at the bit pattern 0x4B400000 (the float
// 12582912.0) instead of 0: one kind::f8f6f4 MMA of two constant e5m2 tiles
// (every A byte 1536, every B byte 256: 32 * 1536 * 256 = 12582912, exact in
// fp32) writes it before the INT8 QK^T accumulates onto it in s32. The
// scores then arrive as the exact floats 12582912 + s (|s| < 2^21), with no
// per-score integer add in the softmax. The constant tiles cost 24 KB of
// shared memory and 1/16 more tensor work per S tile. 0 disables it (the
// softmax then adds the pattern itself).
#ifndef XGB_ATTN_INIT_MMA
#define XGB_ATTN_INIT_MMA 1
#endif
constexpr bool kInitMma = XGB_ATTN_INIT_MMA != 0;
constexpr uint32_t kInitAWord = 0x66666666u;  // e5m2 1536 in every byte
constexpr uint32_t kInitBWord = 0x5C5C5C5Cu;  // e5m2 256 in every byte
// Order of the Sage exp section: 0 works through the keys four at a time
// (arguments, exponentials, sums and packing of each group together); 1
// forms every argument of the tile, then every exponential, then the sums
// and packing.
#ifndef XGB_ATTN_EXP_ORDER
#define XGB_ATTN_EXP_ORDER 1
#endif
constexpr int kExpOrder = XGB_ATTN_EXP_ORDER;
// Packing of four e4m3 P values into one TMEM word: 0 joins the two
// converted pairs by shift and or; 1 by one 32-bit move of the two 16-bit
// halves.
#ifndef XGB_ATTN_PACK
#define XGB_ATTN_PACK 1
#endif
__device__ __forceinline__ uint32_t pack_p4(float a, float b, float c, float d) {
  if constexpr (XGB_ATTN_PACK == 1) {
    uint32_t w;
    asm("{\n\t.reg .b16 lo, hi;\n\t"
        "cvt.rn.satfinite.e4m3x2.f32 lo, %2, %1;\n\t"
        "cvt.rn.satfinite.e4m3x2.f32 hi, %4, %3;\n\t"
        "mov.b32 %0, {lo, hi};\n\t}"
        : "=r"(w)
        : "f"(a), "f"(b), "f"(c), "f"(d));
    return w;
  } else {
    return pack_e4m3x2(a, b) | (pack_e4m3x2(c, d) << 16);
  }
}
// Row sums: 0 adds each tile's partial sums to the row's total; 1 keeps the
// partials running across tiles (rescaled with O) and sums them at the end.
#ifndef XGB_ATTN_LSUM
#define XGB_ATTN_LSUM 1
#endif
constexpr bool kLsum = XGB_ATTN_LSUM != 0;
// S tile read from TMEM as one 64-column load (1) or two of 32 columns (0).
#ifndef XGB_ATTN_LD64
#define XGB_ATTN_LD64 1
#endif
constexpr bool kLd64 = XGB_ATTN_LD64 != 0;
constexpr int kTurnBar = 1;  // named barriers 1, 2: exp turn of WG0, WG1
constexpr int kEpiBar = 3;   // named barrier 3: the 256 softmax threads in the split epilogue
constexpr uint32_t kMagic = 0x4B400000u;
constexpr int kRevTiles = 148;  // Q-tile pairs per key-order group (BF16)

template <bool kSage>
struct Cfg {
  static constexpr int kElem = kSage ? 1 : 2;
  static constexpr int kQBytes = kBM * kD * kElem;   // one 128-row Q tile
  static constexpr int kKVBytes = kBN * kD * kElem;  // one 64-key K or V tile
  static constexpr int kSub = kBN * 128;             // bytes of one 128-byte-wide TMA box of K/V
  static constexpr int kStages = kSage ? 8 : 4;
  static constexpr int kKStepsD = kSage ? 4 : 8;     // QK^T MMA steps over D (32 B each)
  static constexpr int kKStepsN = kSage ? 2 : 4;     // P.V MMA steps over the 64 keys
  static constexpr float kTau = kSage ? 4.0f : 8.0f;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQT * kQBytes;
  static constexpr int kVOff = kKOff + kStages * kKVBytes;
  // Sage accumulator-init operands (XGB_ATTN_INIT_MMA): 128 and 64 rows of
  // 128 bytes, SW128 K-major like Q and K (all bytes equal, so the swizzle
  // does not matter).
  static constexpr bool kInit = kSage && kInitMma;
  static constexpr int kInitAOff = kVOff + kStages * kKVBytes;
  static constexpr int kInitBOff = kInitAOff + (kInit ? kBM * 128 : 0);
  static constexpr int kBarOff = kInitBOff + (kInit ? kBN * 128 : 0);
  static constexpr int kSmem = kBarOff + 512 + 1024;  // + barriers + alignment slack
  static constexpr uint32_t kIdescQK =
      kSage ? instr_desc(2, 1, 1, false, false, kBM, kBN) : instr_desc(1, 1, 1, false, false, kBM, kBN);
  static constexpr uint32_t kIdescPV =
      kSage ? instr_desc(1, 0, 0, false, true, kBM, kD) : instr_desc(1, 1, 1, false, true, kBM, kD);
  static constexpr uint32_t kIdescInit = instr_desc(1, 1, 1, false, false, kBM, kBN);  // e5m2 x e5m2 -> f32
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
  // Tail balancing. CTAs [0, n_full) each run one work item, a (batch*head,
  // Q-tile pair); CTA n_full + j runs part j % splits of the KV range of item
  // n_full + j / splits and leaves its unnormalised O and (max, sum) rows in
  // part_o / part_ml; the last part of an item to finish (counters) merges
  // them. splits = 1: no split.
  int n_qt;        // Q-tile pairs per (batch, head)
  int n_full;
  int splits;
  float* part_o;   // [tail CTAs][256][128]
  float* part_ml;  // [tail CTAs][256][2]
  int* counters;   // [tail items], zero at launch
  // Sage wire layout (kWire): Q/K scales per group of 16 tokens, strided:
  // the scale of (b, h, group g) sits at b*_b + h*_h + g*_g; the V scale row
  // of (b, h) at b*vs_b + h*vs_h; scale_rows = token rows the scales cover.
  int64_t qs_b, qs_h, qs_g, ks_b, ks_h, ks_g, vs_b, vs_h;
  int scale_rows;
};

struct Barriers {
  uint64_t q_full;
  uint64_t k_full[8];
  uint64_t v_full[8];
  uint64_t kv_empty[8];
  uint64_t s_full[2][2];  // [Q tile][S buffer]
  uint64_t p_full[2][2];
  uint64_t pv_done[2];
  uint64_t o_done[2];  // every P.V of Q tile i has landed in O_i
  uint64_t end[2];
  uint32_t tmem_base;
  int last;  // this CTA finished the last part of its item (split epilogue)
};

// TMEM column of S/P buffer `b` of Q tile `i`, and of O_i.
__device__ __forceinline__ uint32_t s_col(int i, int b) { return static_cast<uint32_t>(i * 128 + b * 64); }
__device__ __forceinline__ uint32_t o_col(int i) { return static_cast<uint32_t>(256 + i * 128); }

template <bool kSage, bool kWire>
__device__ __forceinline__ void load_rows(const CUtensorMap* map, uint8_t* dst, uint64_t* bar,
                                          int row, int bh, int heads, int sub_bytes) {
  if constexpr (kSage && kWire) {
    tma_load_4d(dst, map, bar, 0, row, bh % heads, bh / heads);
  } else if constexpr (kSage) {
    tma_load_3d(dst, map, bar, 0, row, bh);
  } else {
    const int b = bh / heads, h = bh % heads;
    tma_load_4d(dst, map, bar, 0, row, h, b);
    tma_load_4d(dst + sub_bytes, map, bar, 64, row, h, b);
  }
}

// K-major SW128 descriptor of MMA K-step `k` (32 bytes of D) within a tile
// whose 128-byte-wide sub-tiles (bf16: d 0-63, d 64-127) are `sub_bytes` apart.
template <bool kSage>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_saddr, int k, uint32_t sub_bytes) {
  const uint32_t sub = kSage ? 0u : static_cast<uint32_t>(k >> 2) * sub_bytes;
  const uint32_t off = static_cast<uint32_t>(kSage ? k : (k & 3)) * 32u;
  return smem_desc_sw128(tile_saddr + sub + off, 16, 1024);
}

// MN-major SW128 descriptor of the V tile for MMA K-step `k` (keys).
template <bool kSage>
__device__ __forceinline__ uint64_t vdesc(uint32_t tile_saddr, int k) {
  // keys per step: 32 (e4m3) or 16 (bf16); each key row is 128 B per sub-tile;
  // the bf16 d 64-127 sub-tile sits kSub bytes after d 0-63.
  const uint32_t off = static_cast<uint32_t>(k) * (kSage ? 32u : 16u) * 128u;
  return smem_desc_sw128(tile_saddr + off, Cfg<kSage>::kSub, 1024);
}

template <bool kSage, bool kWire = false>
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
  const int cta = blockIdx.x;
  const bool split = cta >= p.n_full;
  const int item = split ? p.n_full + (cta - p.n_full) / p.splits : cta;
  const int bh = item / p.n_qt;
  const int m0 = (item % p.n_qt) * (kQT * kBM);
  // KV tiles [kv0, kv0 + n_kv) of this CTA; the host keeps every part non-empty.
  const int n_all = (p.seq_kv + kBN - 1) / kBN;
  const int per = split ? (n_all + p.splits - 1) / p.splits : n_all;
  const int kv0 = split ? ((cta - p.n_full) % p.splits) * per : 0;
  const int n_kv = split ? min(per, n_all - kv0) : n_all;
  // BF16: consecutive groups of kRevTiles Q-tile pairs of a head (about one
  // wave of CTAs) walk the keys in opposite directions, so each group starts
  // on the K/V tiles the previous one read last, still in L2 (one head's bf16
  // K/V is about half the L2). Depends only on the item, so a result never
  // depends on how many heads a launch holds. Sage keeps the forward order:
  // its K/V stay in L2 anyway, and its P quantisation follows the key order.
  const bool rev = !kSage && (((item % p.n_qt) / kRevTiles) & 1);
  auto kv_at = [&](int t) { return kv0 + (rev ? n_kv - 1 - t : t); };

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->kv_empty[s], 2);  // released by both issuers
    }
    for (int i = 0; i < 2; ++i) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(&bars->s_full[i][b], 1);
        mbar_init(&bars->p_full[i][b], kBM);
      }
      mbar_init(&bars->pv_done[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->o_done[i], 1);
      mbar_init(&bars->end[i], 1);
    }
    fence_barrier_init();
  }
  if constexpr (C::kInit) {
    uint4* init = reinterpret_cast<uint4*>(smem + C::kInitAOff);
    for (int j = threadIdx.x; j < (kBM + kBN) * 128 / 16; j += kThreads) {
      const uint32_t w = j < kBM * 128 / 16 ? kInitAWord : kInitBWord;
      init[j] = make_uint4(w, w, w, w);
    }
    fence_proxy_async_smem();  // the tensor core reads them through the async proxy
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
      mbar_arrive_expect_tx(&bars->q_full, kQT * C::kQBytes);
      for (int i = 0; i < kQT; ++i)
        load_rows<kSage, kWire>(&q_map, smem + C::kQOff + i * C::kQBytes, &bars->q_full, m0 + i * kBM,
                         bh, p.heads, kBM * 128);
      int issued = 0;
      for (int t = 0; t < n_kv && ok; ++t) {
        const int s = t % C::kStages;
        if (t >= C::kStages) ok = mbar_wait(&bars->kv_empty[s], ((t / C::kStages) - 1) & 1, p.err);
        if (!ok) break;
        mbar_arrive_expect_tx(&bars->k_full[s], C::kKVBytes);
        load_rows<kSage, kWire>(&k_map, smem + C::kKOff + s * C::kKVBytes, &bars->k_full[s], kv_at(t) * kBN,
                         bh, p.heads, C::kSub);
        mbar_arrive_expect_tx(&bars->v_full[s], C::kKVBytes);
        load_rows<kSage, kWire>(&v_map, smem + C::kVOff + s * C::kKVBytes, &bars->v_full[s], kv_at(t) * kBN,
                         bh, p.heads, C::kSub);
        issued = t + 1;
      }
      // Never leave with copies in flight: wait (bounded) for the last ones.
      for (int t = max(0, issued - C::kStages); t < issued; ++t) {
        const int s = t % C::kStages;
        mbar_wait(&bars->k_full[s], (t / C::kStages) & 1, p.err, 100000000ull);
        mbar_wait(&bars->v_full[s], (t / C::kStages) & 1, p.err, 100000000ull);
      }
      mbar_wait(&bars->q_full, 0, p.err, 100000000ull);
    }
  } else if (warp == kMmaWarp || warp == kMmaWarp + 1) {
    // ------------------------------------------------------------ MMA issuers
    const int i = warp - kMmaWarp;  // Q tile served by this issuer
    if (lane == 0) {
      const uint32_t qa = smem_u32(smem + C::kQOff) + i * C::kQBytes;
      const uint32_t k_saddr = smem_u32(smem + C::kKOff);
      const uint32_t v_saddr = smem_u32(smem + C::kVOff);
      constexpr Kind kQK = kSage ? Kind::kI8 : Kind::kF16;
      constexpr Kind kPV = kSage ? Kind::kF8F6F4 : Kind::kF16;
      // S_i(t) -> buffer t%2 of Q tile i, publish on s_full[i][t%2].
      const uint64_t init_a = smem_desc_sw128(smem_u32(smem + C::kInitAOff), 16, 1024);
      const uint64_t init_b = smem_desc_sw128(smem_u32(smem + C::kInitBOff), 16, 1024);
      auto issue_s = [&](int t) {
        const uint32_t ka = k_saddr + (t % C::kStages) * C::kKVBytes;
        if constexpr (C::kInit)  // S = 0x4B400000 in every element, then += Q.K^T
          mma_ss<Kind::kF8F6F4>(tmem + s_col(i, t & 1), init_a, init_b, C::kIdescInit, false);
#pragma unroll
        for (int k = 0; k < C::kKStepsD; ++k)
          mma_ss<kQK>(tmem + s_col(i, t & 1), kmajor_desc<kSage>(qa, k, kBM * 128),
                      kmajor_desc<kSage>(ka, k, C::kSub), C::kIdescQK, C::kInit || k > 0);
        tc_commit(&bars->s_full[i][t & 1]);
      };
      bool ok = mbar_wait(&bars->q_full, 0, p.err);
      for (int t = 0; t < 2 && t < n_kv && ok; ++t) {
        ok = mbar_wait(&bars->k_full[t % C::kStages], (t / C::kStages) & 1, p.err);
        if (!ok) break;
        tc_fence_after();
        issue_s(t);
      }
      for (int t = 0; t < n_kv && ok; ++t) {
        const int s = t % C::kStages;
        ok = mbar_wait(&bars->v_full[s], (t / C::kStages) & 1, p.err) &&
             mbar_wait(&bars->p_full[i][t & 1], (t >> 1) & 1, p.err);
        if (!ok) break;
        tc_fence_after();
        // O_i += P_i(t) . V(t)
        const uint32_t va = v_saddr + s * C::kKVBytes;
#pragma unroll
        for (int k = 0; k < C::kKStepsN; ++k)
          mma_ts<kPV>(tmem + o_col(i), tmem + s_col(i, t & 1) + k * 8, vdesc<kSage>(va, k),
                      C::kIdescPV, t > 0 || k > 0);
        tc_commit(&bars->pv_done[i]);
        tc_commit(&bars->kv_empty[s]);
        const int t2 = t + 2;
        if (t2 < n_kv) {
          ok = mbar_wait(&bars->k_full[t2 % C::kStages], (t2 / C::kStages) & 1, p.err);
          if (!ok) break;
          tc_fence_after();
          issue_s(t2);
        }
      }
      tc_commit(&bars->o_done[i]);
      tc_commit(&bars->end[i]);
      mbar_wait(&bars->end[i], 0, p.err, 100000000ull);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int i = warp >> 2;                // Q tile of this warpgroup
    const int lane_base = (warp & 3) * 32;  // TMEM lane quarter of this warp
    const int row = m0 + i * kBM + lane_base + lane;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(lane_base) << 16);
    const uint32_t o_addr = lane_addr + o_col(i);
    const int hb = bh / p.heads, hh = bh % p.heads;
    float qs = 0.f;
    if constexpr (kSage && kWire) {
      if (row < p.scale_rows) qs = p.q_scale[hb * p.qs_b + hh * p.qs_h + (row / 16) * p.qs_g];
    } else if constexpr (kSage) {
      if (row < p.scale_stride * 64) qs = p.q_scale[static_cast<int64_t>(bh) * p.scale_stride + row / 64];
    }
    float m_used = kNegInf;
    float l = 0.f;
    // Row-sum partials (four packed chains). kLsum: they run across the tiles
    // and are summed once after the loop; otherwise each tile's are added to l.
    float rsa[4] = {0.f, 0.f, 0.f, 0.f}, rsb[4] = {0.f, 0.f, 0.f, 0.f};
    float ks = 0.f;  // K-block scale of the current tile (Sage)
    if constexpr (kSage && !kWire) ks = p.k_scale[static_cast<int64_t>(bh) * p.scale_stride + kv0];
    // Wire layout: the four 16-key group scales of the current and next tile
    // (groups past the last one read the last one; those keys are masked).
    float ks4[4] = {0.f, 0.f, 0.f, 0.f}, ks4n[4] = {0.f, 0.f, 0.f, 0.f};
    const float* ksp = kWire ? p.k_scale + hb * p.ks_b + hh * p.ks_h : nullptr;
    const int last_group = p.scale_rows / 16 - 1;
    const int ks_g = static_cast<int>(p.ks_g);
    auto load_ks4 = [&](int tile, float (&k)[4]) {
#pragma unroll
      for (int j = 0; j < 4; ++j) k[j] = __ldg(ksp + min(tile * 4 + j, last_group) * ks_g);
    };
    if constexpr (kSage && kWire) {
      if (n_kv > 0) load_ks4(kv0, ks4n);
    }
    bool ok = true;
    // The two warpgroups take turns in the MUFU-bound exp section so one's
    // exp overlaps the other's load/max/rescale work. The turn passes through
    // hardware named barriers (far cheaper to hand over than an mbarrier
    // poll): WG i waits on barrier kTurnBar + i, which completes when its 128
    // threads sync and the other WG's 128 arrive. WG1 hands the first turn to
    // WG0. Every iteration makes exactly one sync and one arrive per WG (WG1
    // skips its last arrive, which nothing would consume); a WG that stops
    // early on a failed wait still makes its remaining ones (below), so
    // neither WG can be left in bar.sync.
    const int turn_own = kTurnBar + i, turn_other = kTurnBar + (i ^ 1);
    int turns = 0;
    if (kTurn && i == 1 && n_kv > 0) named_arrive(turn_other, 2 * kBM);
    for (int t = 0; t < n_kv; ++t) {
      const uint32_t s_addr = lane_addr + s_col(i, t & 1);
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[i][t & 1], (t >> 1) & 1, p.err));
      if (!ok) break;
      tc_fence_after();
      uint32_t r[2][32];
      if constexpr (kLd64) {
        tmem_ld64(s_addr, r);
      } else {
        tmem_ld32(s_addr, r[0]);
        tmem_ld32(s_addr + 32, r[1]);
      }
      tmem_ld_wait();
      // Sage: the int32 scores s are read as the exact floats 12582912 + s:
      // their accumulator started at the bits 0x4B400000 (kInit), or the
      // pattern is added here (|s| < 2^22: 128 products of |int8| <= 127).
      // The map is monotone, so the max runs on floats and no conversion
      // instruction is needed. Padding keys (>= valid, last tile only) get a
      // sentinel far below any real score.
      const int valid = p.seq_kv - kv_at(t) * kBN;
      const float comb = kSage ? qs * ks : p.scale_log2;
      float comb4[4];
      if constexpr (kSage && kWire) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          ks4[j] = ks4n[j];
          comb4[j] = qs * ks4[j];
        }
        if (t + 1 < n_kv) load_ks4(kv0 + t + 1, ks4n);
      }
      if constexpr (kSage) {
        if (!kWire && t + 1 < n_kv) ks = p.k_scale[static_cast<int64_t>(bh) * p.scale_stride + kv0 + t + 1];
        if constexpr (!C::kInit) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) r[c][e] += kMagic;
        }
      }
      if (valid < kBN) {
        const uint32_t sentinel = kSage ? 0x4B000000u /* 12582912 - 2^22 */ : 0xFF800000u /* -inf */;
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c * 32 + e >= valid) r[c][e] = sentinel;
      }
      // Four independent 3-input max chains, then combined (wire layout: one
      // chain per 16-key scale group, scaled by its own group scale).
      float m4[4];
      float mt;
      if constexpr (kSage && kWire) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = j >> 1, e0 = (j & 1) * 16;
          float m = fmax3(__uint_as_float(r[c][e0]), __uint_as_float(r[c][e0 + 1]), __uint_as_float(r[c][e0 + 2]));
#pragma unroll
          for (int e = e0 + 3; e < e0 + 15; e += 2)
            m = fmax3(m, __uint_as_float(r[c][e]), __uint_as_float(r[c][e + 1]));
          m4[j] = comb4[j] * (fmaxf(m, __uint_as_float(r[c][e0 + 15])) - 12582912.0f);
        }
        mt = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      } else {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        m4[2 * c] = fmax3(__uint_as_float(r[c][0]), __uint_as_float(r[c][1]), __uint_as_float(r[c][2]));
        m4[2 * c + 1] = fmax3(__uint_as_float(r[c][3]), __uint_as_float(r[c][4]), __uint_as_float(r[c][5]));
#pragma unroll
        for (int e = 6; e < 30; e += 4) {
          m4[2 * c] = fmax3(m4[2 * c], __uint_as_float(r[c][e]), __uint_as_float(r[c][e + 1]));
          m4[2 * c + 1] = fmax3(m4[2 * c + 1], __uint_as_float(r[c][e + 2]), __uint_as_float(r[c][e + 3]));
        }
        m4[2 * c] = fmax3(m4[2 * c], __uint_as_float(r[c][30]), __uint_as_float(r[c][31]));
      }
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      mt = kSage ? comb * (mx - 12582912.0f) : mx * comb;
      }
      // Lazy rescale (warp-uniform TMEM traffic); O must hold PV(t-1).
      const float m_new = fmaxf(m_used, mt);
      const bool need = m_new > m_used + C::kTau;
      if (t == 0) {
        m_used = m_new;
      } else if (__any_sync(0xffffffffu, need)) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->pv_done[i], (t - 1) & 1, p.err));
        if (!ok) break;
        tc_fence_after();
        const float alpha = need ? ex2_approx(m_used - m_new) : 1.0f;
        if (need) m_used = m_new;
        if constexpr (kLsum) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            rsa[j] *= alpha;
            rsb[j] *= alpha;
          }
        } else {
          l *= alpha;
        }
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
      if constexpr (kTurn) named_sync(turn_own, 2 * kBM);
      // P = exp2(comb*s - m_used) (times kPScale for e4m3, folded into the
      // exponent), row sum, pack and store over the S buffer.
      // Row sums in four independent packed chains (short dependency chains).
      if constexpr (!kLsum) {
#pragma unroll
        for (int j = 0; j < 4; ++j) rsa[j] = rsb[j] = 0.f;
      }
      if constexpr (kSage) {
        const float off = (kLog2PScale - m_used) - 12582912.0f * comb;
        float offs[4];
        if constexpr (kWire) {
#pragma unroll
          for (int j = 0; j < 4; ++j) offs[j] = (kLog2PScale - m_used) - 12582912.0f * comb4[j];
        }
        uint32_t packed[16];  // 64 keys of e4m3 P = 16 TMEM columns
        if constexpr (kExpOrder == 1 && !kWire) {
          // every argument, then every exponential, then sums and packing
          float pv[2][32];
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; e += 2)
              ffma2(pv[c][e], pv[c][e + 1], __uint_as_float(r[c][e]), __uint_as_float(r[c][e + 1]), comb, comb,
                    off, off);
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              if (poly_pair((c * 32 + e) / 2)) {
                ex2_poly2<2>(pv[c][e], pv[c][e + 1], pv[c][e], pv[c][e + 1]);
              } else {
                pv[c][e] = ex2_approx(pv[c][e]);
                pv[c][e + 1] = ex2_approx(pv[c][e + 1]);
              }
            }
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              const int ch = (e / 4) & 1;
              fadd2(rsa[2 * ch], rsb[2 * ch], rsa[2 * ch], rsb[2 * ch], pv[c][e], pv[c][e + 1]);
              fadd2(rsa[2 * ch + 1], rsb[2 * ch + 1], rsa[2 * ch + 1], rsb[2 * ch + 1], pv[c][e + 2], pv[c][e + 3]);
              packed[c * 8 + e / 4] = pack_p4(pv[c][e], pv[c][e + 1], pv[c][e + 2], pv[c][e + 3]);
            }
        } else {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              float x[4], pv[4];
              const float cb = kWire ? comb4[c * 2 + e / 16] : comb;
              const float of = kWire ? offs[c * 2 + e / 16] : off;
              ffma2(x[0], x[1], __uint_as_float(r[c][e]), __uint_as_float(r[c][e + 1]), cb, cb, of, of);
              ffma2(x[2], x[3], __uint_as_float(r[c][e + 2]), __uint_as_float(r[c][e + 3]), cb, cb, of, of);
#pragma unroll
              for (int u = 0; u < 4; u += 2) {
                if (poly_pair((c * 32 + e + u) / 2)) {
                  ex2_poly2<2>(pv[u], pv[u + 1], x[u], x[u + 1]);
                } else {
                  pv[u] = ex2_approx(x[u]);
                  pv[u + 1] = ex2_approx(x[u + 1]);
                }
              }
              const int ch = (e / 4) & 1;
              fadd2(rsa[2 * ch], rsb[2 * ch], rsa[2 * ch], rsb[2 * ch], pv[0], pv[1]);
              fadd2(rsa[2 * ch + 1], rsb[2 * ch + 1], rsa[2 * ch + 1], rsb[2 * ch + 1], pv[2], pv[3]);
              packed[c * 8 + e / 4] = pack_p4(pv[0], pv[1], pv[2], pv[3]);
            }
          }
        }
        tmem_st16(s_addr, packed);
      } else {
        const float off = -m_used;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t packed[16];  // 32 keys of bf16 P = 16 TMEM columns
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float xa, xb;
            ffma2(xa, xb, __uint_as_float(r[c][e]), __uint_as_float(r[c][e + 1]), comb, comb, off, off);
            const float a = ex2_approx(xa);  // (the polynomial share does not pay for BF16)
            const float b = ex2_approx(xb);
            const int ch = (e / 2) & 3;
            fadd2(rsa[ch], rsb[ch], rsa[ch], rsb[ch], a, b);
            packed[e / 2] = pack_bf16x2(a, b);
          }
          tmem_st16(s_addr + c * 16, packed);
        }
      }
      if constexpr (kTurn) {
        if (!(i == 1 && t == n_kv - 1)) named_arrive(turn_other, 2 * kBM);
        turns = t + 1;
      }
      if constexpr (!kLsum) l += ((rsa[0] + rsb[0]) + (rsa[1] + rsb[1])) + ((rsa[2] + rsb[2]) + (rsa[3] + rsb[3]));
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars->p_full[i][t & 1]);
    }
    if constexpr (kTurn) {
      for (int t = turns; t < n_kv; ++t) {  // after a failed wait: keep the turn protocol
        named_sync(turn_own, 2 * kBM);
        if (!(i == 1 && t == n_kv - 1)) named_arrive(turn_other, 2 * kBM);
      }
    }
    if constexpr (kLsum) l = ((rsa[0] + rsb[0]) + (rsa[1] + rsb[1])) + ((rsa[2] + rsb[2]) + (rsa[3] + rsb[3]));
    // ------------------------------------------------------------ epilogue
    // pv_done may trail the last tile by two phases here, so a parity wait
    // on it would be ambiguous; o_done completes exactly once.
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_done[i], 0, p.err));
    __nv_bfloat16* dst = p.out + hb * p.osb + hh * p.osh + static_cast<int64_t>(row) * p.oss;
    const float* vsc = !kSage ? nullptr
                       : kWire ? p.v_scale + hb * p.vs_b + hh * p.vs_h
                               : p.v_scale + static_cast<int64_t>(bh) * kD;
    // out row = o / l (times the per-channel V scale for Sage), as bf16.
    auto store_row = [&](int c, const float* o, float inv_l) {
      uint32_t w[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float x0 = o[e] * inv_l;
        float x1 = o[e + 1] * inv_l;
        if constexpr (kSage) {  // l sums the same kPScale-scaled P
          x0 *= vsc[c * 32 + e];
          x1 *= vsc[c * 32 + e + 1];
        }
        w[e / 2] = pack_bf16x2(x0, x1);
      }
      uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
      for (int v = 0; v < 4; ++v) d4[v] = make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
    };
    if (!split) {
      if (ok) {
        tc_fence_after();
        const float inv_l = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + c * 32, o);
          tmem_ld_wait();
          if (row < p.seq_q) store_row(c, reinterpret_cast<const float*>(o), inv_l);
        }
      }
    } else {
      // Leave this part's rows, then the last part of the item merges:
      // M = max m_q, O = sum 2^(m_q - M) O_q, L = sum 2^(m_q - M) l_q.
      const int slot = cta - p.n_full;
      const int first = slot - slot % p.splits;
      const int r = i * kBM + lane_base + lane;  // row within the CTA
      if (ok) {
        tc_fence_after();
        float4* po = reinterpret_cast<float4*>(p.part_o + (static_cast<int64_t>(slot) * 256 + r) * kD);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int v = 0; v < 8; ++v)
            po[c * 8 + v] = make_float4(__uint_as_float(o[4 * v]), __uint_as_float(o[4 * v + 1]),
                                        __uint_as_float(o[4 * v + 2]), __uint_as_float(o[4 * v + 3]));
        }
        reinterpret_cast<float2*>(p.part_ml)[static_cast<int64_t>(slot) * 256 + r] = make_float2(m_used, l);
      }
      __threadfence();
      named_sync(kEpiBar, 2 * kBM);
      if (threadIdx.x == 0) {
        const int done = atomicAdd(&p.counters[slot / p.splits], 1);
        bars->last = done == p.splits - 1;
        if (bars->last) p.counters[slot / p.splits] = 0;  // ready for the next launch
      }
      named_sync(kEpiBar, 2 * kBM);
      if (bars->last && ok && row < p.seq_q) {
        __threadfence();
        const float2* ml = reinterpret_cast<const float2*>(p.part_ml);
        float mx = kNegInf;
        for (int q = 0; q < p.splits; ++q) mx = fmaxf(mx, __ldcg(&ml[static_cast<int64_t>(first + q) * 256 + r]).x);
        float lsum = 0.f;
        for (int q = 0; q < p.splits; ++q) {
          const float2 v = __ldcg(&ml[static_cast<int64_t>(first + q) * 256 + r]);
          lsum += ex2_approx(v.x - mx) * v.y;
        }
        const float inv_l = lsum > 0.f ? 1.0f / lsum : 0.f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float acc[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[e] = 0.f;
          for (int q = 0; q < p.splits; ++q) {
            const int64_t base = static_cast<int64_t>(first + q) * 256 + r;
            const float w = ex2_approx(__ldcg(&ml[base]).x - mx);
            const float4* po = reinterpret_cast<const float4*>(p.part_o + base * kD) + c * 8;
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              const float4 o4 = __ldcg(po + v);
              acc[4 * v] = fmaf(w, o4.x, acc[4 * v]);
              acc[4 * v + 1] = fmaf(w, o4.y, acc[4 * v + 1]);
              acc[4 * v + 2] = fmaf(w, o4.z, acc[4 * v + 2]);
              acc[4 * v + 3] = fmaf(w, o4.w, acc[4 * v + 3]);
            }
          }
          store_row(c, acc, inv_l);
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

// Workspace of the tail split: counters, then (max, sum) rows, then O rows,
// sized for one part per SM.
constexpr int64_t kCounterBytes = 1024;
inline int64_t split_bytes(int sms) {
  return kCounterBytes + static_cast<int64_t>(sms) * 256 * (2 + kD) * sizeof(float);
}

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <bool kSage, bool kWire = false>
int launch(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, Params p,
           int64_t bh, void* ws, int64_t ws_bytes, cudaStream_t st) {
  using C = Cfg<kSage>;
  auto kernel = attention_kernel<kSage, kWire>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) !=
      cudaSuccess)
    return XGB_ERR_LAUNCH;
  // Work items: (batch*head, pair of 128-row Q tiles), one CTA each, one CTA
  // per SM. The last, partial wave leaves SMs idle; its items are split
  // along the KV range so that wave fills the SMs with shorter CTAs.
  const int64_t n_qt = (p.seq_q + kQT * kBM - 1) / (kQT * kBM);
  const int64_t items = n_qt * bh;
  if (items > INT32_MAX / 2) return XGB_ERR_SHAPE;
  const int sms = sm_count();
  const int n_all = (p.seq_kv + kBN - 1) / kBN;
  const int tail = static_cast<int>(items % sms);
  int splits = 1;
  if (ws && tail > 0 && ws_bytes >= split_bytes(sms) && tail * (int64_t)sizeof(int) <= kCounterBytes) {
    splits = std::min(sms / tail, n_all);
    if (splits > 1) {
      const int per = (n_all + splits - 1) / splits;
      splits = (n_all + per - 1) / per;  // no empty part
    }
  }
  p.n_qt = static_cast<int>(n_qt);
  p.splits = 1;
  p.n_full = static_cast<int>(items);
  if (splits > 1) {
    char* w = static_cast<char*>(ws);
    p.counters = reinterpret_cast<int*>(w);
    p.part_ml = reinterpret_cast<float*>(w + kCounterBytes);
    p.part_o = p.part_ml + static_cast<int64_t>(sms) * 256 * 2;
    p.splits = splits;
    p.n_full = static_cast<int>(items - tail);
    if (cudaMemsetAsync(p.counters, 0, tail * sizeof(int), st) != cudaSuccess) return XGB_ERR_LAUNCH;
  }
  const int64_t grid = p.n_full + static_cast<int64_t>(items - p.n_full) * p.splits;
  kernel<<<static_cast<unsigned>(grid), kThreads, C::kSmem, st>>>(qm, km, vm, p);
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
                               const int64_t* out_strides, void* split_workspace,
                               int64_t split_workspace_bytes, int* error_flag, void* stream) {
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
  const uint32_t qbox[3] = {128, kBM, 1};
  const uint32_t kvbox[3] = {128, kBN, 1};
  if (!make_tensor_map(&qm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, q8, dims, strides, qbox) ||
      !make_tensor_map(&km, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, k8, dims, strides, kvbox) ||
      !make_tensor_map(&vm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, v8, dims, strides, kvbox))
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
  return launch<true>(qm, km, vm, p, bh, split_workspace, split_workspace_bytes, as_stream(stream));
}

XGB_API int xgb_attention_bf16(const void* q, const int64_t* q_strides, const void* k,
                               const int64_t* k_strides, const void* v, const int64_t* v_strides,
                               int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_kv,
                               float sm_scale, void* out, const int64_t* out_strides,
                               void* split_workspace, int64_t split_workspace_bytes,
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
  auto make = [&](CUtensorMap* m, const void* base, const int64_t* s, int64_t seq, uint32_t rows) {
    const uint32_t box[4] = {64, rows, 1, 1};
    const uint64_t dims[4] = {static_cast<uint64_t>(kD), static_cast<uint64_t>(seq),
                              static_cast<uint64_t>(heads), static_cast<uint64_t>(batch)};
    const uint64_t strides[3] = {static_cast<uint64_t>(s[2]) * 2, static_cast<uint64_t>(s[1]) * 2,
                                 static_cast<uint64_t>(s[0]) * 2};
    return make_tensor_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box);
  };
  if (!make(&qm, q, q_strides, seq_q, kBM) || !make(&km, k, k_strides, seq_kv, kBN) ||
      !make(&vm, v, v_strides, seq_kv, kBN))
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
  return launch<false>(qm, km, vm, p, batch * heads, split_workspace, split_workspace_bytes,
                       as_stream(stream));
}

XGB_API int64_t xgb_attention_split_workspace_bytes(void) { return split_bytes(sm_count()); }

XGB_API int xgb_attention_sage_strided(
    const int8_t* q8, const int64_t* q_strides, const float* q_scale, const int64_t* q_scale_strides,
    const int8_t* k8, const int64_t* k_strides, const float* k_scale, const int64_t* k_scale_strides,
    const uint8_t* v8, const int64_t* v_strides, const float* v_scale,
    const int64_t* v_scale_strides, int64_t batch, int64_t heads, int64_t seq, int64_t scale_rows,
    void* out, const int64_t* out_strides, void* split_workspace, int64_t split_workspace_bytes,
    int* error_flag, void* stream) {
  if (!q8 || !k8 || !v8 || !q_scale || !k_scale || !v_scale || !out) return XGB_ERR_ARG;
  if (!q_strides || !k_strides || !v_strides || !q_scale_strides || !k_scale_strides ||
      !v_scale_strides || !out_strides)
    return XGB_ERR_ARG;
  if (batch <= 0 || heads <= 0 || seq <= 0 || seq > (1 << 30) || scale_rows < seq ||
      scale_rows % 16 || scale_rows > (1 << 30))
    return XGB_ERR_SHAPE;
  if (out_strides[3] != 1 || out_strides[2] % 8 || out_strides[1] % 8 || out_strides[0] % 8)
    return XGB_ERR_STRIDE;
  const int64_t* in[3] = {q_strides, k_strides, v_strides};
  for (auto st : in)
    for (int d = 0; d < 3; ++d)
      if (st[d] % 16 || st[d] <= 0) return XGB_ERR_STRIDE;  // 16-byte TMA strides (1-byte elements)
  if (!aligned(q8, 16) || !aligned(k8, 16) || !aligned(v8, 16) || !aligned(out, 16))
    return XGB_ERR_ALIGN;
  int rc = check_device();
  if (rc) return rc;
  CUtensorMap qm, km, vm;
  auto make = [&](CUtensorMap* m, const void* base, const int64_t* s, uint32_t rows) {
    const uint32_t box[4] = {128, rows, 1, 1};
    const uint64_t dims[4] = {static_cast<uint64_t>(kD), static_cast<uint64_t>(scale_rows),
                              static_cast<uint64_t>(heads), static_cast<uint64_t>(batch)};
    const uint64_t strides[3] = {static_cast<uint64_t>(s[2]), static_cast<uint64_t>(s[1]),
                                 static_cast<uint64_t>(s[0])};
    return make_tensor_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, base, dims, strides, box);
  };
  if (!make(&qm, q8, q_strides, kBM) || !make(&km, k8, k_strides, kBN) || !make(&vm, v8, v_strides, kBN))
    return XGB_ERR_ALIGN;
  Params p{};
  p.q_scale = q_scale;
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.heads = static_cast<int>(heads);
  p.seq_q = static_cast<int>(seq);
  p.seq_kv = static_cast<int>(seq);
  p.scale_log2 = 1.0f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.osb = out_strides[0];
  p.osh = out_strides[1];
  p.oss = out_strides[2];
  p.err = error_flag;
  p.qs_b = q_scale_strides[0];
  p.qs_h = q_scale_strides[1];
  p.qs_g = q_scale_strides[2];
  p.ks_b = k_scale_strides[0];
  p.ks_h = k_scale_strides[1];
  p.ks_g = k_scale_strides[2];
  p.vs_b = v_scale_strides[0];
  p.vs_h = v_scale_strides[1];
  p.scale_rows = static_cast<int>(scale_rows);
  return launch<true, true>(qm, km, vm, p, batch * heads, split_workspace, split_workspace_bytes,
                            as_stream(stream));
}
