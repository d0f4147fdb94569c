// Dynamic e4m3 activation quantisation for the FP8 Linear.
//
// Per-tensor (the reference's scheme, x_base/x_base/operator/h3_fp8.py:9-12,
// h3_fp8_quant.py:9-25, h3_abs_peak.py:14-25):
//   peaks[b] = max |x| over block b            (NaN-propagating)
//   scale    = max(max(peaks) * fp32(1/448), FLT_MIN)   (torch CUDA scalar division)
//   out      = e4m3(clamp(x / scale, +-448))   (IEEE division, RNE)
// The max is order-independent, so the result is bit-exact with the
// reference whatever the block split; the per-block peaks live in a
// caller-provided workspace, as the reference's `peaks` tensor does.
//
// Per-token (the B200 FP8 Linear's activation scheme): the same formula per
// row, computed by one CTA per row from registers (rows up to 16,384 wide,
// vector-aligned) or one warp per row.
#include <cfloat>
#include <mutex>

#include "xgb_common.cuh"

namespace xgb {
namespace {

constexpr int kThreads = 256;
constexpr int64_t kPeakBlock = 8192;  // elements per peak, as the reference

template <typename T>
__device__ __forceinline__ float to_float(T v);
template <>
__device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_float<__half>(__half v) { return __half2float(v); }

__device__ __forceinline__ int abs_bits(float v) { return __float_as_int(fabsf(v)); }

// Block peaks: |x| bit images compared as integers (NaN sorts above +inf).
template <typename T>
__global__ void __launch_bounds__(kThreads) abs_peak_kernel(const T* __restrict__ x, int64_t n,
                                                            int* __restrict__ peaks) {
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kPeakBlock;
  const int64_t end = min(base + kPeakBlock, n);
  int m = 0;
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (end - base) % 8 == 0;
  if (vec) {
    for (int64_t i = base + threadIdx.x * 8; i < end; i += kThreads * 8) {
      uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + i));
      const T* v = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) m = max(m, abs_bits(to_float<T>(v[j])));
    }
  } else {
    for (int64_t i = base + threadIdx.x; i < end; i += kThreads) m = max(m, abs_bits(to_float<T>(x[i])));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ int warp_peak[kThreads / 32];
  if ((threadIdx.x & 31) == 0) warp_peak[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    int r = 0;
    for (int w = 0; w < kThreads / 32; ++w) r = max(r, warp_peak[w]);
    peaks[blockIdx.x] = r;
  }
}

__global__ void __launch_bounds__(kThreads) peak_to_scale_kernel(const int* __restrict__ peaks,
                                                                 int64_t blocks,
                                                                 float* __restrict__ scale) {
  int m = 0;
  for (int64_t i = threadIdx.x; i < blocks; i += kThreads) m = max(m, peaks[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ int warp_peak[kThreads / 32];
  if ((threadIdx.x & 31) == 0) warp_peak[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    int r = 0;
    for (int w = 0; w < kThreads / 32; ++w) r = max(r, warp_peak[w]);
    // torch evaluates `amax / 448.0` on a CUDA tensor as amax * fp32(1/448)
    // (a CPU-scalar divisor is turned into a reciprocal multiply), which is
    // what the reference's GPU path and its bit-equality test see.
    const float s = __fmul_rn(__int_as_float(r), 1.0f / 448.0f);
    *scale = isnan(s) ? s : fmaxf(s, FLT_MIN);  // clamp_min keeps NaN
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) pack_kernel(const T* __restrict__ x, int64_t n,
                                                        const float* __restrict__ scale_ptr,
                                                        uint8_t* __restrict__ out) {
  const float scale = __ldg(scale_ptr);
  const float y = __frcp_rn(scale);
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) * 8;
  if (i >= n) return;
  if (i + 8 <= n && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
      (reinterpret_cast<uintptr_t>(out) & 7u) == 0) {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + i));
    const T* v = reinterpret_cast<const T*>(&raw);
    uint8_t b[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      b[j] = f32_to_e4m3(fminf(fmaxf(div_by(to_float<T>(v[j]), scale, y), -448.f), 448.f));
    *reinterpret_cast<uint2*>(out + i) = *reinterpret_cast<uint2*>(b);
  } else {
    for (int64_t j = i; j < min(i + 8, n); ++j)
      out[j] = f32_to_e4m3(fminf(fmaxf(div_by(to_float<T>(x[j]), scale, y), -448.f), 448.f));
  }
}

// One warp per row: amax, scale, pack.
template <typename T>
__global__ void __launch_bounds__(kThreads) per_token_kernel(const T* __restrict__ x, int64_t rows,
                                                             int64_t cols, int64_t row_stride,
                                                             uint8_t* __restrict__ out,
                                                             float* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* src = x + row * row_stride;
  uint8_t* dst = out + row * cols;
  // 16-byte loads and 8-byte stores need both x and out aligned for them.
  const bool vec = cols % 8 == 0 && row_stride % 8 == 0 &&
                   (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 7u) == 0;
  int m = 0;
  if (vec) {
    for (int64_t c = lane * 8; c < cols; c += 256) {
      uint4 raw = __ldg(reinterpret_cast<const uint4*>(src + c));
      const T* v = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) m = max(m, abs_bits(to_float<T>(v[j])));
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) m = max(m, abs_bits(to_float<T>(src[c])));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float amax_scale = __fdiv_rn(__int_as_float(m), 448.0f);
  const float scale = isnan(amax_scale) ? amax_scale : fmaxf(amax_scale, FLT_MIN);
  if (lane == 0) scales[row] = scale;
  const float y = __frcp_rn(scale);
  if (vec) {
    for (int64_t c = lane * 8; c < cols; c += 256) {
      uint4 raw = __ldg(reinterpret_cast<const uint4*>(src + c));
      const T* v = reinterpret_cast<const T*>(&raw);
      uint8_t b[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        b[j] = f32_to_e4m3(fminf(fmaxf(div_by(to_float<T>(v[j]), scale, y), -448.f), 448.f));
      *reinterpret_cast<uint2*>(dst + c) = *reinterpret_cast<uint2*>(b);
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32)
      dst[c] = f32_to_e4m3(fminf(fmaxf(div_by(to_float<T>(src[c]), scale, y), -448.f), 448.f));
  }
}

// One CTA per row for rows of up to 16,384 channels: the row is read once
// into registers (P 16-byte chunks per thread), reduced, and packed from the
// registers, so it crosses HBM once (a warp-per-row pass re-reads rows that
// no longer fit L2 at FFN widths). Same values as per_token_kernel.
constexpr int kRowThreads = 256;

template <typename T, int P>
__global__ void __launch_bounds__(kRowThreads) per_token_row_kernel(
    const T* __restrict__ x, int64_t cols, int64_t row_stride, uint8_t* __restrict__ out,
    float* __restrict__ scales) {
  __shared__ int red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const int chunks = static_cast<int>(cols / 8);
  const uint4* src = reinterpret_cast<const uint4*>(x + row * row_stride);
  uint4 raw[P];
#pragma unroll
  for (int j = 0; j < P; ++j) {
    const int c = threadIdx.x + j * kRowThreads;
    raw[j] = c < chunks ? __ldg(src + c) : make_uint4(0, 0, 0, 0);
  }
  int m = 0;
#pragma unroll
  for (int j = 0; j < P; ++j) {
    const T* v = reinterpret_cast<const T*>(&raw[j]);
#pragma unroll
    for (int e = 0; e < 8; ++e) m = max(m, abs_bits(to_float<T>(v[e])));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kRowThreads / 32; ++i) m = max(m, red[i]);
  const float amax_scale = __fdiv_rn(__int_as_float(m), 448.0f);
  const float scale = isnan(amax_scale) ? amax_scale : fmaxf(amax_scale, FLT_MIN);
  if (threadIdx.x == 0) scales[row] = scale;
  const float y = __frcp_rn(scale);
  uint2* dst = reinterpret_cast<uint2*>(out + row * cols);
#pragma unroll
  for (int j = 0; j < P; ++j) {
    const int c = threadIdx.x + j * kRowThreads;
    if (c < chunks) {
      const T* v = reinterpret_cast<const T*>(&raw[j]);
      uint32_t q[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2)
        q[e / 2] = e4m3x2(fminf(fmaxf(div_by(to_float<T>(v[e]), scale, y), -448.f), 448.f),
                          fminf(fmaxf(div_by(to_float<T>(v[e + 1]), scale, y), -448.f), 448.f));
      dst[c] = make_uint2(q[0] | (q[1] << 16), q[2] | (q[3] << 16));
    }
  }
}

template <typename T>
bool launch_per_token_rows(const T* x, int64_t rows, int64_t cols, int64_t row_stride,
                           uint8_t* out, float* scales, cudaStream_t st) {
  const int64_t per_thread = cdiv(cols / 8, kRowThreads);
  if (cols % 8 || row_stride % 8 || per_thread > 8 || rows > INT32_MAX ||
      (reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(out) & 7u))
    return false;
  const dim3 grid(static_cast<unsigned>(rows));
  if (per_thread <= 1) per_token_row_kernel<T, 1><<<grid, kRowThreads, 0, st>>>(x, cols, row_stride, out, scales);
  else if (per_thread <= 2) per_token_row_kernel<T, 2><<<grid, kRowThreads, 0, st>>>(x, cols, row_stride, out, scales);
  else if (per_thread <= 4) per_token_row_kernel<T, 4><<<grid, kRowThreads, 0, st>>>(x, cols, row_stride, out, scales);
  else if (per_thread <= 6) per_token_row_kernel<T, 6><<<grid, kRowThreads, 0, st>>>(x, cols, row_stride, out, scales);
  else per_token_row_kernel<T, 8><<<grid, kRowThreads, 0, st>>>(x, cols, row_stride, out, scales);
  return true;
}

}  // namespace
}  // namespace xgb

using namespace xgb;

XGB_API int64_t xgb_fp8_quantize_per_tensor_workspace(int64_t n) {
  if (n <= 0) return 0;
  return cdiv(n, kPeakBlock) * static_cast<int64_t>(sizeof(int));
}

XGB_API int xgb_fp8_quantize_per_tensor(const void* x, int dtype, int64_t n, uint8_t* out,
                                        float* scale_out, void* workspace,
                                        int64_t workspace_bytes, void* stream) {
  if (!x || !out || !scale_out) return XGB_ERR_ARG;
  if (dtype != XGB_BF16 && dtype != XGB_F16) return XGB_ERR_ARG;
  if (n <= 0) return XGB_ERR_SHAPE;
  const int64_t blocks = cdiv(n, kPeakBlock);
  if (!workspace || workspace_bytes < xgb_fp8_quantize_per_tensor_workspace(n))
    return XGB_ERR_WORKSPACE;
  int* peaks = static_cast<int*>(workspace);
  cudaStream_t st = as_stream(stream);
  const unsigned pack_grid = static_cast<unsigned>(cdiv(cdiv(n, 8), kThreads));
  if (dtype == XGB_BF16) {
    auto xb = static_cast<const __nv_bfloat16*>(x);
    abs_peak_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(xb, n, peaks);
    peak_to_scale_kernel<<<1, kThreads, 0, st>>>(peaks, blocks, scale_out);
    pack_kernel<<<pack_grid, kThreads, 0, st>>>(xb, n, scale_out, out);
  } else {
    auto xh = static_cast<const __half*>(x);
    abs_peak_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(xh, n, peaks);
    peak_to_scale_kernel<<<1, kThreads, 0, st>>>(peaks, blocks, scale_out);
    pack_kernel<<<pack_grid, kThreads, 0, st>>>(xh, n, scale_out, out);
  }
  return launch_status();
}

XGB_API int xgb_fp8_abs_peak_scale(const void* x, int dtype, int64_t n, float* scale_out,
                                   void* workspace, int64_t workspace_bytes, void* stream) {
  if (!x || !scale_out) return XGB_ERR_ARG;
  if (dtype != XGB_BF16 && dtype != XGB_F16) return XGB_ERR_ARG;
  if (n <= 0) return XGB_ERR_SHAPE;
  const int64_t blocks = cdiv(n, kPeakBlock);
  if (!workspace || workspace_bytes < xgb_fp8_quantize_per_tensor_workspace(n))
    return XGB_ERR_WORKSPACE;
  int* peaks = static_cast<int*>(workspace);
  cudaStream_t st = as_stream(stream);
  if (dtype == XGB_BF16)
    abs_peak_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), n, peaks);
  else
    abs_peak_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(
        static_cast<const __half*>(x), n, peaks);
  peak_to_scale_kernel<<<1, kThreads, 0, st>>>(peaks, blocks, scale_out);
  return launch_status();
}

XGB_API int xgb_fp8_quantize_with_scale(const void* x, int dtype, int64_t n, const float* scale,
                                        uint8_t* out, void* stream) {
  if (!x || !out || !scale) return XGB_ERR_ARG;
  if (dtype != XGB_BF16 && dtype != XGB_F16) return XGB_ERR_ARG;
  if (n <= 0) return XGB_ERR_SHAPE;
  cudaStream_t st = as_stream(stream);
  const unsigned grid = static_cast<unsigned>(cdiv(cdiv(n, 8), kThreads));
  if (dtype == XGB_BF16)
    pack_kernel<<<grid, kThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(x), n, scale, out);
  else
    pack_kernel<<<grid, kThreads, 0, st>>>(static_cast<const __half*>(x), n, scale, out);
  return launch_status();
}

XGB_API int xgb_fp8_quantize_per_token(const void* x, int dtype, int64_t rows, int64_t cols,
                                       int64_t row_stride, uint8_t* out, float* scales,
                                       void* stream) {
  if (!x || !out || !scales) return XGB_ERR_ARG;
  if (dtype != XGB_BF16 && dtype != XGB_F16) return XGB_ERR_ARG;
  if (rows < 0 || cols <= 0 || row_stride < cols) return XGB_ERR_SHAPE;
  if (rows == 0) return XGB_OK;
  const unsigned grid = static_cast<unsigned>(cdiv(rows, kThreads / 32));
  cudaStream_t st = as_stream(stream);
  const bool by_rows =
      dtype == XGB_BF16
          ? launch_per_token_rows(static_cast<const __nv_bfloat16*>(x), rows, cols, row_stride, out, scales, st)
          : launch_per_token_rows(static_cast<const __half*>(x), rows, cols, row_stride, out, scales, st);
  if (by_rows) return launch_status();
  if (dtype == XGB_BF16)
    per_token_kernel<<<grid, kThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(x), rows, cols,
                                                 row_stride, out, scales);
  else
    per_token_kernel<<<grid, kThreads, 0, st>>>(static_cast<const __half*>(x), rows, cols,
                                                 row_stride, out, scales);
  return launch_status();
}

// ---------------------------------------------------------------- no-allocation variant
// Some callers of this library cannot allocate device memory at call time:
// a plugin embedded in a host runtime that owns every device allocation and
// hands out no workspace, a server that plans all of HBM up front and forbids
// allocation while serving, or a latency-critical path that cannot afford
// cudaMalloc's implicit device-wide synchronisation. For them,
// xgb_fp8_quantize_per_tensor_noalloc takes the per-block peak scratch from
// a fixed array compiled into the library instead of a caller workspace.
//
// The array is a file-scope __device__ symbol: every GPU that loads libxgb.so
// holds its 256 KiB until the process exits. Its address is resolved once per
// device (cudaGetSymbolAddress with that device current) on the entry point's
// first call there, so that first call should come before any stream
// capture. All calls share the one array and it keeps the last call's
// contents; nothing needs clearing (each call writes every peak slot it later
// reads), but calls whose kernels overlap on a device race on it.
namespace xgb {
namespace {

constexpr int64_t kNoAllocMaxBlocks = 65536;  // peaks of 65536 x 8192 elements
constexpr int kMaxDevices = 64;

static __device__ __align__(256) int g_noalloc_peaks[kNoAllocMaxBlocks];

std::mutex g_noalloc_mutex;
int* g_noalloc_scratch[kMaxDevices] = {};

int noalloc_scratch(int** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return XGB_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_scratch[dev] == nullptr) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_noalloc_peaks) != cudaSuccess || addr == nullptr)
      return XGB_ERR_LAUNCH;
    g_noalloc_scratch[dev] = static_cast<int*>(addr);
  }
  *out = g_noalloc_scratch[dev];
  return XGB_OK;
}

}  // namespace
}  // namespace xgb

XGB_API int xgb_fp8_quantize_per_tensor_noalloc(const void* x, int dtype, int64_t n, uint8_t* out,
                                                float* scale_out, void* stream) {
  if (!x || !out || !scale_out) return XGB_ERR_ARG;
  if (dtype != XGB_BF16 && dtype != XGB_F16) return XGB_ERR_ARG;
  if (n <= 0 || cdiv(n, kPeakBlock) > kNoAllocMaxBlocks) return XGB_ERR_SHAPE;
  int* peaks = nullptr;
  const int rc = noalloc_scratch(&peaks);
  if (rc != XGB_OK) return rc;
  const int64_t blocks = cdiv(n, kPeakBlock);
  cudaStream_t st = as_stream(stream);
  const unsigned pack_grid = static_cast<unsigned>(cdiv(cdiv(n, 8), kThreads));
  if (dtype == XGB_BF16) {
    auto xb = static_cast<const __nv_bfloat16*>(x);
    abs_peak_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(xb, n, peaks);
    peak_to_scale_kernel<<<1, kThreads, 0, st>>>(peaks, blocks, scale_out);
    pack_kernel<<<pack_grid, kThreads, 0, st>>>(xb, n, scale_out, out);
  } else {
    auto xh = static_cast<const __half*>(x);
    abs_peak_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(xh, n, peaks);
    peak_to_scale_kernel<<<1, kThreads, 0, st>>>(peaks, blocks, scale_out);
    pack_kernel<<<pack_grid, kThreads, 0, st>>>(xh, n, scale_out, out);
  }
  return launch_status();
}
