// Library-level entry points of libxgb.so (version and status names).
#include "xgb_common.cuh"

XGB_API int xgb_version(void) { return 100; }

XGB_API const char* xgb_status_string(int status) {
  switch (status) {
    case XGB_OK: return "ok";
    case XGB_ERR_ARG: return "invalid argument";
    case XGB_ERR_SHAPE: return "unsupported shape";
    case XGB_ERR_STRIDE: return "unsupported stride";
    case XGB_ERR_ALIGN: return "misaligned pointer or stride";
    case XGB_ERR_LAUNCH: return "CUDA launch error";
    case XGB_ERR_DEVICE: return "device is not an sm_100 GPU";
    case XGB_ERR_WORKSPACE: return "workspace missing or too small";
    default: return "unknown status";
  }
}
