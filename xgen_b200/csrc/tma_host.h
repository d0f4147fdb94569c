// Host-side construction of TMA tensor maps (cuTensorMapEncodeTiled reached
// through the runtime's driver entry point, so libxgb.so needs no -lcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace xgb {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  }
  return fn;
}

// Tiled map with 128-byte swizzle and zero fill out of bounds.
// dims/box are innermost-first; strides_bytes has rank-1 entries (dims 1..).
// Returns false if the driver rejects the description (alignment, box).
inline bool make_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank,
                            const void* base, const uint64_t* dims, const uint64_t* strides_bytes,
                            const uint32_t* box) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  uint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, dtype, rank, const_cast<void*>(base), dims, strides_bytes, box,
                   elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace xgb
