// PHAA FP8 wire codec: one byte A2A payload carrying per-row e4m3 values and
// an fp32 row scale, optionally with the pre-A2A rotate-half RoPE fused in.
//
// Wire layout (x_base/x_base/phaa/fp8_transport.py:26-63, :103-112):
//   per peer p: [stream0 rows][stream1 rows][stream2 rows][peer_padding zeros]
//   row:        width e4m3 bytes, then the fp32 scale
//   scale       = max(max|x| / 448, 1e-12); byte = e4m3(clamp(x/scale, +-448))
// The division is IEEE (__fdiv_rn), matching the reference algorithm as the
// Triton interpreter evaluates it.
//
// Rows are addressed through [peer, seq, batch, head] views with any element
// strides (unit channel stride) on both sides, so the async exchange's
// direct layouts (x_base/x_base/phaa/fp8_async_transport.py:14-81) need no
// copies: the return pack reads the attention output [batch, head, seq, D]
// and the direct gather / direct return decodes write the attention input
// [batch, head, seq, D] and the final [batch, seq, heads*D] in place. A row
// whose global sequence index peer*seq + s is >= valid_seq encodes as zeros
// (scale 1e-12) without a load and is skipped by the decode.
//
// Work split: a group of G = next_pow2(width/8) lanes owns one row, each lane
// 8 channels; 32/G rows per warp, so width=128 uses full warps (2 rows each).
#include <climits>
#include <type_traits>

#include "xgb_common.cuh"

namespace xgb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxStreams = 3;

struct EncodeArgs {
  const void* src[kMaxStreams];
  int64_t st[kMaxStreams][4];  // element strides: peer, seq, batch, head
  int64_t peers, seq, batch, heads, width, rows, peer_rows, peer_padding, valid_seq;
  FastDiv div_heads, div_batch, div_seq;  // row -> (peer, seq, batch, head)
  int streams;
  const float* cos;
  const float* sin;
  int64_t rotary;
  uint8_t* payload;
};

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

template <typename T, bool kVec>
__device__ __forceinline__ void load_row8(const T* p, int valid, float (&out)[8]) {
  if (kVec && valid == 8) {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
    const T* v = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = to_f<T>(v[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = i < valid ? to_f<T>(p[i]) : 0.f;
  }
}

// Row index -> (peer, seq, batch, head) of the [peer, seq, batch, head] order.
__device__ __forceinline__ void split_row(uint32_t r, FastDiv dh, FastDiv db, FastDiv ds,
                                          uint32_t& peer, uint32_t& s, uint32_t& bat,
                                          uint32_t& head) {
  const uint32_t q1 = fast_div(r, dh);
  head = r - q1 * dh.d;
  const uint32_t q2 = fast_div(q1, db);
  bat = q1 - q2 * db.d;
  peer = fast_div(q2, ds);
  s = q2 - peer * ds.d;
}

template <typename T, bool kVec>
__global__ void __launch_bounds__(kThreads) wire_encode_kernel(EncodeArgs a, int group) {
  const int slot = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int sub = lane & (group - 1);             // lane within the row group
  const int rows_per_warp = 32 / group;
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5)) *
                          rows_per_warp + lane / group;
  const bool live = row < a.rows;
  uint32_t peer, s, bat, head;
  split_row(live ? static_cast<uint32_t>(row) : 0u, a.div_heads, a.div_batch, a.div_seq, peer, s,
            bat, head);
  const bool inside = static_cast<int64_t>(peer) * a.seq + s < a.valid_seq;
  const T* src = static_cast<const T*>(a.src[slot]);
  if (inside) src += peer * a.st[slot][0] + s * a.st[slot][1] + bat * a.st[slot][2] + head * a.st[slot][3];
  const int c0 = sub * 8;
  const int valid = live ? max(0, min(8, static_cast<int>(a.width) - c0)) : 0;
  const int loaded = inside ? valid : 0;

  float x[8];
  load_row8<T, kVec>(src + c0, loaded, x);
  if (inside && a.rotary > 0 && slot < 2 && c0 < a.rotary) {
    // Fused pre-A2A RoPE (h3_partial_rope.py:9-29): bf16 result, then encode.
    const int64_t half = a.rotary / 2;
    const float* cs = a.cos + static_cast<int64_t>(s) * a.rotary;
    const float* sn = a.sin + static_cast<int64_t>(s) * a.rotary;
    float p[8], cv[8], sv[8];
    if (kVec && valid == 8 && c0 + 8 <= a.rotary && half % 8 == 0 && a.rotary % 4 == 0) {
      // The 8 channels sit on one side of the half split: the partner
      // channels and the cos/sin entries are contiguous vectors.
      const bool first = c0 < half;
      load_row8<T, true>(src + (first ? c0 + half : c0 - half), 8, p);
      const float4 c_lo = __ldg(reinterpret_cast<const float4*>(cs + c0));
      const float4 c_hi = __ldg(reinterpret_cast<const float4*>(cs + c0 + 4));
      const float4 s_lo = __ldg(reinterpret_cast<const float4*>(sn + c0));
      const float4 s_hi = __ldg(reinterpret_cast<const float4*>(sn + c0 + 4));
      cv[0] = c_lo.x; cv[1] = c_lo.y; cv[2] = c_lo.z; cv[3] = c_lo.w;
      cv[4] = c_hi.x; cv[5] = c_hi.y; cv[6] = c_hi.z; cv[7] = c_hi.w;
      sv[0] = s_lo.x; sv[1] = s_lo.y; sv[2] = s_lo.z; sv[3] = s_lo.w;
      sv[4] = s_hi.x; sv[5] = s_hi.y; sv[6] = s_hi.z; sv[7] = s_hi.w;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float left = bf16_round(__fmul_rn(x[i], bf16_round(cv[i])));
        const float right = bf16_round(__fmul_rn(first ? -p[i] : p[i], bf16_round(sv[i])));
        x[i] = to_f<T>(from_f<T>(__fadd_rn(left, right)));
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t c = c0 + i;
        if (i < valid && c < a.rotary) {
          const bool first = c < half;
          p[i] = to_f<T>(src[first ? c + half : c - half]);
          const float cb = bf16_round(cs[c]);
          const float sb = bf16_round(sn[c]);
          const float left = bf16_round(__fmul_rn(x[i], cb));
          const float right = bf16_round(__fmul_rn(first ? -p[i] : p[i], sb));
          x[i] = to_f<T>(from_f<T>(__fadd_rn(left, right)));
        }
      }
    }
  }
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(x[i]));
  for (int o = group / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float scale = fmaxf(__fdiv_rn(m, 448.0f), 1.0e-12f);
  if (!live) return;

  const int64_t wire_row = row + (static_cast<int64_t>(peer) * (a.streams - 1) + slot) * a.peer_rows;
  const int64_t offset = wire_row * (a.width + 4) + static_cast<int64_t>(peer) * a.peer_padding;
  uint8_t* dst = a.payload + offset;
  // x / scale, correctly rounded as the reference's division, then e4m3.
  const float y = __frcp_rn(scale);
  uint32_t w[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float q = fminf(fmaxf(div_by(x[4 * h + j], scale, y), -448.0f), 448.0f);
      word |= static_cast<uint32_t>(f32_to_e4m3(q)) << (8 * j);
    }
    w[h] = word;
  }
  if (valid == 8) {
    // Rows start at 4-byte multiples (width % 4 == 0), so two u32 stores.
    reinterpret_cast<uint32_t*>(dst + c0)[0] = w[0];
    reinterpret_cast<uint32_t*>(dst + c0)[1] = w[1];
  } else {
    const uint8_t* b = reinterpret_cast<const uint8_t*>(w);
    for (int i = 0; i < valid; ++i) dst[c0 + i] = b[i];
  }
  if (sub == 0) *reinterpret_cast<float*>(dst + a.width) = scale;
  if (a.peer_padding && sub == 0 && slot == 0 && row % a.peer_rows == 0) {
    const int64_t packet = a.peer_rows * a.streams * (a.width + 4);
    uint8_t* tail = a.payload + static_cast<int64_t>(peer) * (packet + a.peer_padding) + packet;
    for (int64_t i = 0; i < a.peer_padding; ++i) tail[i] = 0;
  }
}

// bf16 rows with width % (8V) == 0 and (rotary == 0 or rotary % (16V) == 0):
// the same bytes as wire_encode_kernel with fewer instructions and fewer L2
// reads. A group of G lanes owns one (peer, seq, batch) position and walks
// its heads kHeadBlock at a time, each lane 8V channels (V 16-byte words),
// so the position's cos/sin are read once for all heads, the per-row index
// and scale work is shared by 8V channels, and each lane has several row
// loads in flight; the RoPE partner channels come from the partner lane by
// shuffle. The row stays packed bf16x2: the RoPE products and sum
// are bf16x2 operations (rope8_bf16), the row scale's division by 448 and
// the per-element x / scale are Markstein-corrected reciprocal multiplies
// (the correctly rounded quotient; below 448e-12 the 1e-12 floor decides),
// and the saturating e4m3x2 conversion replaces the clamp to +-448 (values
// beyond 448 round to 448 either way).
constexpr int kHeadBlock = 3;  // H3 has 24 heads: 3, 6, 12 or 24 per rank

template <int V>
__global__ void __launch_bounds__(kThreads) wire_encode_bf16_kernel(EncodeArgs a, int group) {
  const int slot = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int sub = lane & (group - 1);
  const int64_t positions = a.rows / a.heads;
  const int64_t pos = (static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5)) *
                          (32 / group) + lane / group;
  const bool live = pos < positions;
  const uint32_t pr = live ? static_cast<uint32_t>(pos) : 0u;
  const uint32_t q2 = fast_div(pr, a.div_batch);  // peer * seq + s
  const uint32_t bat = pr - q2 * a.div_batch.d;
  const uint32_t peer = fast_div(q2, a.div_seq);
  const uint32_t s = q2 - peer * a.div_seq.d;
  const int c0 = sub * 8 * V;
  const bool has = live && c0 < a.width && static_cast<int64_t>(peer) * a.seq + s < a.valid_seq;
  const bool rope = has && slot < 2 && c0 < a.rotary;
  const int half = static_cast<int>(a.rotary / 2);
  const bool first = c0 < half;
  uint32_t cw[V][4], sw[V][4];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    if (rope) {
      load_cos_sin8(a.cos + static_cast<int64_t>(s) * a.rotary + c0 + 8 * v,
                    a.sin + static_cast<int64_t>(s) * a.rotary + c0 + 8 * v, cw[v], sw[v]);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) cw[v][k] = sw[v][k] = 0;
    }
  }
  const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(a.src[slot]) + peer * a.st[slot][0] +
                              s * a.st[slot][1] + bat * a.st[slot][2] + c0;
  // The partner channels c -/+ rotary/2 sit in the lane rotary/(16V) away
  // within the row group (rotary % (16V) == 0); they come by shuffle.
  const int plane = (lane & ~(group - 1)) | (c0 >= a.rotary ? sub : (first ? sub + half / (8 * V) : sub - half / (8 * V)));
  const int64_t hstride = a.st[slot][3];
  constexpr float kRcp448 = 1.0f / 448.0f;  // RN(1/448)
  const int64_t row_bytes = a.width + 4;
  uint8_t* dst0 = a.payload + ((static_cast<int64_t>(peer) * (a.streams - 1) + slot) * a.peer_rows + pos * a.heads) * row_bytes +
                  static_cast<int64_t>(peer) * a.peer_padding;
  const int heads = static_cast<int>(a.heads);
  for (int h0 = 0; h0 < heads; h0 += kHeadBlock) {
    uint4 raw[kHeadBlock][V];
#pragma unroll
    for (int j = 0; j < kHeadBlock; ++j) {
      const bool hj = has && h0 + j < heads;
      const __nv_bfloat16* src = base + (h0 + j) * hstride;
#pragma unroll
      for (int v = 0; v < V; ++v)
        raw[j][v] = hj ? __ldg(reinterpret_cast<const uint4*>(src) + v) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < kHeadBlock; ++j) {
      if (h0 + j >= heads) break;  // uniform across the warp
      float x[V][8];
      float m = 0.f;
#pragma unroll
      for (int v = 0; v < V; ++v) {
        if (slot < 2 && a.rotary > 0) {  // uniform: every lane of the group shuffles
          uint4 par;
          par.x = __shfl_sync(0xffffffffu, raw[j][v].x, plane);
          par.y = __shfl_sync(0xffffffffu, raw[j][v].y, plane);
          par.z = __shfl_sync(0xffffffffu, raw[j][v].z, plane);
          par.w = __shfl_sync(0xffffffffu, raw[j][v].w, plane);
          if (rope) raw[j][v] = rope8_bf16(raw[j][v], par, first, cw[v], sw[v]);
        }
        unpack_bf16x8(raw[j][v], x[v]);
        m = fmaxf(fmaxf(m, fabsf(x[v][0])), fabsf(x[v][1]));
        m = fmaxf(fmaxf(m, fabsf(x[v][2])), fabsf(x[v][3]));
        m = fmaxf(fmaxf(m, fabsf(x[v][4])), fabsf(x[v][5]));
        m = fmaxf(fmaxf(m, fabsf(x[v][6])), fabsf(x[v][7]));
      }
      for (int o = group / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float scale = fmaxf(div_by(m, 448.0f, kRcp448), 1.0e-12f);
      if (!live) continue;
      uint8_t* dst = dst0 + (h0 + j) * row_bytes;
      if (c0 < a.width) {
        const float y = __frcp_rn(scale);
#pragma unroll
        for (int v = 0; v < V; ++v) {
          const uint32_t e0 = e4m3x2(div_by(x[v][0], scale, y), div_by(x[v][1], scale, y));
          const uint32_t e1 = e4m3x2(div_by(x[v][2], scale, y), div_by(x[v][3], scale, y));
          const uint32_t e2 = e4m3x2(div_by(x[v][4], scale, y), div_by(x[v][5], scale, y));
          const uint32_t e3 = e4m3x2(div_by(x[v][6], scale, y), div_by(x[v][7], scale, y));
          // Rows start at 4-byte multiples (width % 4 == 0), so u32 stores.
          reinterpret_cast<uint32_t*>(dst + c0 + 8 * v)[0] = e0 | (e1 << 16);
          reinterpret_cast<uint32_t*>(dst + c0 + 8 * v)[1] = e2 | (e3 << 16);
        }
      }
      if (sub == 0) *reinterpret_cast<float*>(dst + a.width) = scale;
      if (a.peer_padding && sub == 0 && slot == 0) {
        const int64_t row = pos * a.heads + h0 + j;
        if (row % a.peer_rows == 0) {
          const int64_t packet = a.peer_rows * a.streams * row_bytes;
          uint8_t* tail = a.payload + static_cast<int64_t>(peer) * (packet + a.peer_padding) + packet;
          for (int64_t i = 0; i < a.peer_padding; ++i) tail[i] = 0;
        }
      }
    }
  }
}

// Peer form of wire_encode_bf16_kernel<2> (bf16 Q/K/V, 128 channels, the
// same bytes): the encoded rows go straight into each destination rank's
// receive buffer over NVLink instead of a local send buffer that an
// all-to-all then moves. dst[p] is where this rank's section starts in peer
// p's receive buffer (the offset an all_to_all_single would deliver it to).
// A warp owns 4 consecutive (seq, batch) positions of one peer; their rows
// for all heads are one contiguous span of the section, 16-byte aligned when
// a peer holds a multiple of 4 positions. The warp encodes the span into
// shared memory and then writes it out with 16-byte stores, so the link
// carries full sectors rather than the 4-byte pieces the row encoder makes.
constexpr int kMaxPeers = 8;
constexpr int kPeerPositions = 4;  // per warp: 8 lanes x 16 channels per position

struct PeerDst {
  uint8_t* dst[kMaxPeers];
};

__global__ void __launch_bounds__(kThreads) wire_encode_peers_kernel(EncodeArgs a, PeerDst pd) {
  extern __shared__ __align__(16) uint8_t stage[];
  constexpr int V = 2;
  constexpr int G = 8;
  constexpr int64_t kRowBytes = 132;
  const int slot = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int sub = lane & (G - 1);
  const int heads = static_cast<int>(a.heads);
  const int64_t span = kPeerPositions * heads * kRowBytes;
  uint8_t* st = stage + warp * span;
  const int64_t positions = a.rows / a.heads;
  const int64_t pos0 = (static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + warp) * kPeerPositions;
  if (pos0 >= positions) return;  // whole warps: positions % 4 == 0
  const int local = lane / G;
  const uint32_t pr = static_cast<uint32_t>(pos0 + local);
  const uint32_t q2 = fast_div(pr, a.div_batch);  // peer * seq + s
  const uint32_t bat = pr - q2 * a.div_batch.d;
  const uint32_t peer = fast_div(q2, a.div_seq);
  const uint32_t s = q2 - peer * a.div_seq.d;
  const int c0 = sub * 8 * V;
  const bool has = static_cast<int64_t>(peer) * a.seq + s < a.valid_seq;
  const bool rope = has && slot < 2 && c0 < a.rotary;
  const int half = static_cast<int>(a.rotary / 2);
  const bool first = c0 < half;
  uint32_t cw[V][4], sw[V][4];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    if (rope) {
      load_cos_sin8(a.cos + static_cast<int64_t>(s) * a.rotary + c0 + 8 * v,
                    a.sin + static_cast<int64_t>(s) * a.rotary + c0 + 8 * v, cw[v], sw[v]);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) cw[v][k] = sw[v][k] = 0;
    }
  }
  const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(a.src[slot]) + peer * a.st[slot][0] +
                              s * a.st[slot][1] + bat * a.st[slot][2] + c0;
  const int plane = (lane & ~(G - 1)) | (c0 >= a.rotary ? sub : (first ? sub + half / (8 * V) : sub - half / (8 * V)));
  const int64_t hstride = a.st[slot][3];
  constexpr float kRcp448 = 1.0f / 448.0f;  // RN(1/448)
  uint8_t* row0 = st + local * heads * kRowBytes;
  for (int h0 = 0; h0 < heads; h0 += kHeadBlock) {
    uint4 raw[kHeadBlock][V];
#pragma unroll
    for (int j = 0; j < kHeadBlock; ++j) {
      const bool hj = has && h0 + j < heads;
      const __nv_bfloat16* src = base + (h0 + j) * hstride;
#pragma unroll
      for (int v = 0; v < V; ++v)
        raw[j][v] = hj ? __ldg(reinterpret_cast<const uint4*>(src) + v) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < kHeadBlock; ++j) {
      if (h0 + j >= heads) break;  // uniform across the warp
      float x[V][8];
      float m = 0.f;
#pragma unroll
      for (int v = 0; v < V; ++v) {
        if (slot < 2 && a.rotary > 0) {  // uniform: every lane of the group shuffles
          uint4 par;
          par.x = __shfl_sync(0xffffffffu, raw[j][v].x, plane);
          par.y = __shfl_sync(0xffffffffu, raw[j][v].y, plane);
          par.z = __shfl_sync(0xffffffffu, raw[j][v].z, plane);
          par.w = __shfl_sync(0xffffffffu, raw[j][v].w, plane);
          if (rope) raw[j][v] = rope8_bf16(raw[j][v], par, first, cw[v], sw[v]);
        }
        unpack_bf16x8(raw[j][v], x[v]);
        m = fmaxf(fmaxf(m, fabsf(x[v][0])), fabsf(x[v][1]));
        m = fmaxf(fmaxf(m, fabsf(x[v][2])), fabsf(x[v][3]));
        m = fmaxf(fmaxf(m, fabsf(x[v][4])), fabsf(x[v][5]));
        m = fmaxf(fmaxf(m, fabsf(x[v][6])), fabsf(x[v][7]));
      }
      for (int o = G / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float scale = fmaxf(div_by(m, 448.0f, kRcp448), 1.0e-12f);
      uint8_t* row = row0 + (h0 + j) * kRowBytes;
      const float y = __frcp_rn(scale);
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const uint32_t e0 = e4m3x2(div_by(x[v][0], scale, y), div_by(x[v][1], scale, y));
        const uint32_t e1 = e4m3x2(div_by(x[v][2], scale, y), div_by(x[v][3], scale, y));
        const uint32_t e2 = e4m3x2(div_by(x[v][4], scale, y), div_by(x[v][5], scale, y));
        const uint32_t e3 = e4m3x2(div_by(x[v][6], scale, y), div_by(x[v][7], scale, y));
        reinterpret_cast<uint32_t*>(row + c0 + 8 * v)[0] = e0 | (e1 << 16);
        reinterpret_cast<uint32_t*>(row + c0 + 8 * v)[1] = e2 | (e3 << 16);
      }
      if (sub == 0) *reinterpret_cast<float*>(row + 128) = scale;
    }
  }
  __syncwarp();
  // The span's place in the destination section: [slot][seq, batch, head] rows.
  const uint32_t dpeer = __shfl_sync(0xffffffffu, peer, 0);
  const int64_t pos_in_peer = pos0 - static_cast<int64_t>(dpeer) * a.seq * a.batch;
  uint4* out = reinterpret_cast<uint4*>(pd.dst[dpeer] + (slot * a.peer_rows + pos_in_peer * heads) * kRowBytes);
  const uint4* in = reinterpret_cast<const uint4*>(st);
  for (int64_t i = lane; i < span / 16; i += 32) out[i] = in[i];
  __threadfence_system();  // these stores before anything this thread's stream does next
}

struct DecodeArgs {
  const uint8_t* payload;
  void* dst[kMaxStreams];
  int64_t st[kMaxStreams][4];  // element strides of the destination: peer, seq, batch, head
  int64_t seq, batch, heads, width, rows, peer_rows, peer_padding, valid_seq;
  FastDiv div_heads, div_batch, div_seq;
  int streams;
};

template <typename T>
__global__ void __launch_bounds__(kThreads) wire_decode_kernel(DecodeArgs a, int group) {
  const int slot = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int sub = lane & (group - 1);
  const int rows_per_warp = 32 / group;
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5)) *
                          rows_per_warp + lane / group;
  if (row >= a.rows) return;
  const int c0 = sub * 8;
  const int valid = max(0, min(8, static_cast<int>(a.width) - c0));
  if (valid == 0) return;
  uint32_t peer, s, bat, head;
  split_row(static_cast<uint32_t>(row), a.div_heads, a.div_batch, a.div_seq, peer, s, bat, head);
  if (static_cast<int64_t>(peer) * a.seq + s >= a.valid_seq) return;
  const int64_t wire_row = row + (peer * (a.streams - 1) + slot) * a.peer_rows;
  const uint8_t* src = a.payload + wire_row * (a.width + 4) + peer * a.peer_padding;
  const float scale = __ldg(reinterpret_cast<const float*>(src + a.width));
  T* dst = static_cast<T*>(a.dst[slot]) + peer * a.st[slot][0] + s * a.st[slot][1] +
           bat * a.st[slot][2] + head * a.st[slot][3] + c0;
  uint8_t b[8];
  if (valid == 8) {
    *reinterpret_cast<uint32_t*>(b) = __ldg(reinterpret_cast<const uint32_t*>(src + c0));
    *reinterpret_cast<uint32_t*>(b + 4) = __ldg(reinterpret_cast<const uint32_t*>(src + c0 + 4));
  } else {
    for (int i = 0; i < valid; ++i) b[i] = src[c0 + i];
  }
  T out[8];
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    // pairs: e4m3x2 -> f16x2 (exact) -> fp32, times the scale, one bf16x2 rounding
    uint32_t* o = reinterpret_cast<uint32_t*>(out);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint16_t pair = static_cast<uint16_t>(b[2 * k]) | (static_cast<uint16_t>(b[2 * k + 1]) << 8);
      const float2 f = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3)));
      o[k] = round_bf16x2(__fmul_rn(f.x, scale), __fmul_rn(f.y, scale));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = from_f<T>(__fmul_rn(e4m3_to_f32(b[i]), scale));
  }
  if (valid == 8 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<uint4*>(out);
  } else {
    for (int i = 0; i < valid; ++i) dst[i] = out[i];
  }
}

int group_for(int64_t width) {
  int lanes = static_cast<int>((width + 7) / 8);
  int g = 1;
  while (g < lanes) g <<= 1;
  return g;
}

}  // namespace
}  // namespace xgb

using namespace xgb;

XGB_API int xgb_fp8_wire_encode_view(const void* const* sources, const int64_t* strides,
                                     int streams, int64_t peers, int64_t seq, int64_t batch,
                                     int64_t heads, int64_t width, int dtype, const float* cos,
                                     const float* sin, int64_t rotary, int64_t valid_seq,
                                     int64_t peer_padding, uint8_t* payload, void* stream) {
  if (!sources || !strides || !payload) return XGB_ERR_ARG;
  if (streams != 1 && streams != 3) return XGB_ERR_ARG;
  if (dtype != XGB_BF16 && dtype != XGB_F16) return XGB_ERR_ARG;
  if (peers <= 0 || seq < 0 || batch < 0 || heads < 0) return XGB_ERR_SHAPE;
  if (valid_seq < 0 || valid_seq > peers * seq) return XGB_ERR_SHAPE;
  if (width <= 0 || width % 4 || width > 256) return XGB_ERR_SHAPE;
  if (peer_padding < 0 || peer_padding >= 16 || peer_padding % 4) return XGB_ERR_ARG;
  if (rotary < 0 || rotary % 2 || rotary > width) return XGB_ERR_SHAPE;
  if (rotary > 0 && (!cos || !sin || dtype != XGB_BF16)) return XGB_ERR_ARG;
  EncodeArgs a{};
  a.rows = peers * seq * batch * heads;
  if (a.rows == 0) return XGB_OK;
  bool vec = true;
  for (int s = 0; s < streams; ++s) {
    if (!sources[s]) return XGB_ERR_ARG;
    a.src[s] = sources[s];
    for (int d = 0; d < 4; ++d) {
      a.st[s][d] = strides[4 * s + d];
      if (a.st[s][d] % 8) vec = false;
    }
    if (reinterpret_cast<uintptr_t>(sources[s]) & 15u) vec = false;
  }
  if (width % 8) vec = false;
  // the vector RoPE reads cos/sin rows as float4
  if (rotary > 0 && ((reinterpret_cast<uintptr_t>(cos) | reinterpret_cast<uintptr_t>(sin)) & 15u))
    vec = false;
  if (a.rows > INT32_MAX) return XGB_ERR_SHAPE;
  a.peers = peers; a.seq = seq; a.batch = batch; a.heads = heads; a.width = width;
  a.peer_rows = a.rows / peers;
  a.peer_padding = peer_padding; a.streams = streams; a.valid_seq = valid_seq;
  a.div_heads = make_fastdiv(static_cast<uint32_t>(heads));
  a.div_batch = make_fastdiv(static_cast<uint32_t>(batch));
  a.div_seq = make_fastdiv(static_cast<uint32_t>(seq));
  a.cos = cos; a.sin = sin; a.rotary = rotary; a.payload = payload;
  const int group = group_for(width);
  const int64_t rows_per_block = (kThreads / 32) * (32 / group);
  dim3 grid(static_cast<unsigned>(cdiv(a.rows, rows_per_block)), streams);
  cudaStream_t st = as_stream(stream);
  if (dtype == XGB_BF16) {
    if (vec && width % 16 == 0 && rotary % 32 == 0 && heads <= INT32_MAX) {
      int g2 = 1;  // lanes per row at 16 channels per lane
      while (g2 < width / 16) g2 <<= 1;
      const dim3 pgrid(static_cast<unsigned>(cdiv(a.rows / heads, (kThreads / 32) * (32 / g2))), streams);
      wire_encode_bf16_kernel<2><<<pgrid, kThreads, 0, st>>>(a, g2);
    } else if (vec && rotary % 16 == 0 && heads <= INT32_MAX) {
      const dim3 pgrid(static_cast<unsigned>(cdiv(a.rows / heads, rows_per_block)), streams);
      wire_encode_bf16_kernel<1><<<pgrid, kThreads, 0, st>>>(a, group);
    }
    else if (vec) wire_encode_kernel<__nv_bfloat16, true><<<grid, kThreads, 0, st>>>(a, group);
    else wire_encode_kernel<__nv_bfloat16, false><<<grid, kThreads, 0, st>>>(a, group);
  } else {
    if (vec) wire_encode_kernel<__half, true><<<grid, kThreads, 0, st>>>(a, group);
    else wire_encode_kernel<__half, false><<<grid, kThreads, 0, st>>>(a, group);
  }
  return launch_status();
}

XGB_API int xgb_fp8_wire_encode(const void* const* sources, const int64_t* strides, int streams,
                                int64_t peers, int64_t seq, int64_t batch, int64_t heads,
                                int64_t width, int dtype, const float* cos, const float* sin,
                                int64_t rotary, int64_t peer_padding, uint8_t* payload,
                                void* stream) {
  if (peers <= 0 || seq < 0) return XGB_ERR_SHAPE;
  return xgb_fp8_wire_encode_view(sources, strides, streams, peers, seq, batch, heads, width,
                                  dtype, cos, sin, rotary, peers * seq, peer_padding, payload,
                                  stream);
}

XGB_API int xgb_fp8_wire_decode_view(const uint8_t* payload, void* const* dests,
                                     const int64_t* strides, int streams, int64_t peers,
                                     int64_t seq, int64_t batch, int64_t heads, int64_t width,
                                     int64_t valid_seq, int64_t peer_padding, int dtype,
                                     void* stream) {
  if (!payload || !dests || !strides) return XGB_ERR_ARG;
  if (streams != 1 && streams != 3) return XGB_ERR_ARG;
  if (dtype != XGB_BF16 && dtype != XGB_F16) return XGB_ERR_ARG;
  if (peers <= 0 || seq < 0 || batch < 0 || heads < 0) return XGB_ERR_SHAPE;
  if (valid_seq < 0 || valid_seq > peers * seq) return XGB_ERR_SHAPE;
  if (width <= 0 || width % 4 || width > 256) return XGB_ERR_SHAPE;
  if (peer_padding < 0 || peer_padding >= 16 || peer_padding % 4) return XGB_ERR_ARG;
  DecodeArgs a{};
  a.rows = peers * seq * batch * heads;
  if (a.rows == 0) return XGB_OK;
  a.payload = payload;
  for (int s = 0; s < streams; ++s) {
    if (!dests[s]) return XGB_ERR_ARG;
    a.dst[s] = dests[s];
    for (int d = 0; d < 4; ++d) a.st[s][d] = strides[4 * s + d];
  }
  if (a.rows > INT32_MAX) return XGB_ERR_SHAPE;
  a.seq = seq; a.batch = batch; a.heads = heads; a.width = width;
  a.peer_rows = a.rows / peers;
  a.peer_padding = peer_padding; a.streams = streams; a.valid_seq = valid_seq;
  a.div_heads = make_fastdiv(static_cast<uint32_t>(heads));
  a.div_batch = make_fastdiv(static_cast<uint32_t>(batch));
  a.div_seq = make_fastdiv(static_cast<uint32_t>(seq));
  const int group = group_for(width);
  const int64_t rows_per_block = (kThreads / 32) * (32 / group);
  dim3 grid(static_cast<unsigned>(cdiv(a.rows, rows_per_block)), streams);
  cudaStream_t st = as_stream(stream);
  if (dtype == XGB_BF16) wire_decode_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(a, group);
  else wire_decode_kernel<__half><<<grid, kThreads, 0, st>>>(a, group);
  return launch_status();
}

XGB_API int xgb_fp8_wire_decode(const uint8_t* payload, void* const* dests, int streams,
                                int64_t rows, int64_t peers, int64_t width, int64_t peer_padding,
                                int dtype, void* stream) {
  if (rows < 0 || peers <= 0 || rows % peers) return XGB_ERR_SHAPE;
  if (width <= 0) return XGB_ERR_SHAPE;
  const int64_t peer_rows = rows / peers;
  // Contiguous destinations: [peer, row, 1, 1] with row stride `width`.
  int64_t strides[4 * kMaxStreams];
  for (int s = 0; s < kMaxStreams; ++s) {
    strides[4 * s + 0] = peer_rows * width;
    strides[4 * s + 1] = width;
    strides[4 * s + 2] = 0;
    strides[4 * s + 3] = 0;
  }
  return xgb_fp8_wire_decode_view(payload, dests, strides, streams, peers, peer_rows, 1, 1, width,
                                  rows, peer_padding, dtype, stream);
}

XGB_API int xgb_fp8_wire_encode_peers(const void* const* sources, const int64_t* strides, int streams,
                                      int64_t peers, int64_t seq, int64_t batch, int64_t heads,
                                      const float* cos, const float* sin, int64_t rotary,
                                      int64_t valid_seq, uint8_t* const* peer_dst, void* stream) {
  if (!sources || !strides || !peer_dst) return XGB_ERR_ARG;
  if (streams != 1 && streams != 3) return XGB_ERR_ARG;
  if (streams == 1 && rotary != 0) return XGB_ERR_ARG;  // the RoPE is for Q and K
  if (peers <= 0 || peers > kMaxPeers || seq <= 0 || batch <= 0 || heads <= 0) return XGB_ERR_SHAPE;
  if (valid_seq <= 0 || valid_seq > peers * seq) return XGB_ERR_SHAPE;
  // whole warps of 4 positions inside one peer; shared-memory span per warp
  if ((seq * batch) % kPeerPositions || heads > 12) return XGB_ERR_SHAPE;
  if (rotary < 0 || rotary % 32 || rotary > 128) return XGB_ERR_SHAPE;
  if (rotary > 0 && (!cos || !sin)) return XGB_ERR_ARG;
  if (rotary > 0 && ((reinterpret_cast<uintptr_t>(cos) | reinterpret_cast<uintptr_t>(sin)) & 15u))
    return XGB_ERR_ALIGN;
  EncodeArgs a{};
  a.rows = peers * seq * batch * heads;
  if (a.rows > INT32_MAX) return XGB_ERR_SHAPE;
  for (int s = 0; s < streams; ++s) {
    if (!sources[s]) return XGB_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(sources[s]) & 15u) return XGB_ERR_ALIGN;
    a.src[s] = sources[s];
    for (int d = 0; d < 4; ++d) {
      a.st[s][d] = strides[4 * s + d];
      if (a.st[s][d] % 8) return XGB_ERR_STRIDE;
    }
  }
  PeerDst pd{};
  for (int p = 0; p < peers; ++p) {
    if (!peer_dst[p]) return XGB_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(peer_dst[p]) & 15u) return XGB_ERR_ALIGN;
    pd.dst[p] = peer_dst[p];
  }
  a.peers = peers; a.seq = seq; a.batch = batch; a.heads = heads; a.width = 128;
  a.peer_rows = a.rows / peers;
  a.peer_padding = 0; a.streams = streams; a.valid_seq = valid_seq;
  a.div_heads = make_fastdiv(static_cast<uint32_t>(heads));
  a.div_batch = make_fastdiv(static_cast<uint32_t>(batch));
  a.div_seq = make_fastdiv(static_cast<uint32_t>(seq));
  a.cos = cos; a.sin = sin; a.rotary = rotary; a.payload = nullptr;
  const int smem = (kThreads / 32) * kPeerPositions * static_cast<int>(heads) * 132;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(wire_encode_peers_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
          cudaSuccess)
    return XGB_ERR_LAUNCH;
  const int64_t positions = a.rows / heads;
  const dim3 grid(static_cast<unsigned>(cdiv(positions, (kThreads / 32) * kPeerPositions)), streams);
  wire_encode_peers_kernel<<<grid, kThreads, smem, as_stream(stream)>>>(a, pd);
  return launch_status();
}
