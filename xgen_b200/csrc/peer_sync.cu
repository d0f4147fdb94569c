// Flags between ranks for exchanges whose kernels write straight into peer
// GPUs' memory (xgb_fp8_wire_encode_peers): a rank signals a peer by storing
// an epoch number into a word of the peer's buffer (release, system scope,
// after a system fence, so the stores before it land first), and waits for
// its own words to reach an epoch (acquire, system scope). Every wait is
// bounded: after `limit_ns` it records a timeout in the caller's error word
// and returns, so a rank that never signals cannot hang the GPU. Words are
// only ever waited on by the GPU that owns them and written by other GPUs'
// kernels, never by another kernel of the waiting GPU.
#include "sm100.cuh"
#include "xgb_common.cuh"

namespace xgb {
namespace {

constexpr int kMaxFlags = 64;

struct FlagPtrs {
  int* p[kMaxFlags];
};

__global__ void peer_signal_kernel(FlagPtrs f, int n, int value) {
  const int i = threadIdx.x;
  if (i >= n) return;
  __threadfence_system();
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(f.p[i]), "r"(value) : "memory");
}

__global__ void peer_wait_kernel(FlagPtrs f, int n, int value, uint64_t limit_ns, int* err) {
  const int i = threadIdx.x;
  if (i >= n) return;
  const uint64_t t0 = sm100::global_timer_ns();
  for (;;) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(f.p[i]) : "memory");
    if (v >= value) break;
    if (sm100::global_timer_ns() - t0 > limit_ns) {
      if (err) atomicExch(err, sm100::kErrTimeout);
      break;
    }
    __nanosleep(64);
  }
}

int fill(FlagPtrs& f, int* const* flags, int n) {
  if (!flags || n < 0 || n > kMaxFlags) return XGB_ERR_ARG;
  for (int i = 0; i < n; ++i) {
    if (!flags[i] || (reinterpret_cast<uintptr_t>(flags[i]) & 3u)) return XGB_ERR_ARG;
    f.p[i] = flags[i];
  }
  return XGB_OK;
}

}  // namespace
}  // namespace xgb

using namespace xgb;

XGB_API int xgb_peer_signal(int* const* flags, int n, int value, void* stream) {
  FlagPtrs f{};
  if (const int rc = fill(f, flags, n)) return rc;
  if (n == 0) return XGB_OK;
  peer_signal_kernel<<<1, kMaxFlags, 0, as_stream(stream)>>>(f, n, value);
  return launch_status();
}

XGB_API int xgb_peer_wait(int* const* flags, int n, int value, int64_t limit_ns, int* error_flag,
                          void* stream) {
  FlagPtrs f{};
  if (const int rc = fill(f, flags, n)) return rc;
  if (limit_ns <= 0) return XGB_ERR_ARG;
  if (n == 0) return XGB_OK;
  peer_wait_kernel<<<1, kMaxFlags, 0, as_stream(stream)>>>(f, n, value, static_cast<uint64_t>(limit_ns),
                                                          error_flag);
  return launch_status();
}
