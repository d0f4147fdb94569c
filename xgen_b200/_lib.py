"""ctypes binding of libxgb.so, the C-ABI library of the B200 kernels.

The library is loaded from the package tree (xgen_b200/lib/libxgb.so). There
is no fallback: if it is missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libxgb.so"

XGB_OK = 0
XGB_ERR_ARG = -1
XGB_ERR_SHAPE = -2
XGB_ERR_STRIDE = -3
XGB_ERR_ALIGN = -4
XGB_ERR_LAUNCH = -5
XGB_ERR_DEVICE = -6
XGB_ERR_WORKSPACE = -7

XGB_BF16 = 0
XGB_F16 = 1

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_float = ctypes.c_float
c_vp = ctypes.c_void_p
c_i64p = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); mirrors include/xgb.h
SIGNATURES = {
    "xgb_version": (c_int, []),
    "xgb_status_string": (ctypes.c_char_p, [c_int]),
    "xgb_partial_rope": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64,
                                 c_i64, c_vp]),
    "xgb_qk_rms": (c_int, [c_vp, c_i64p, c_vp, c_i64p, c_vp, c_vp, c_float, c_float, c_vp, c_vp,
                           c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "xgb_indexed_affine": (c_int, [c_vp, c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_i64, c_i64,
                                   c_i64, c_int, c_vp]),
    "xgb_swiglu": (c_int, [c_vp, c_vp, c_i64, c_i64, c_vp, c_vp]),
    "xgb_fp8_wire_encode": (c_int, [ctypes.POINTER(c_vp), c_i64p, c_int, c_i64, c_i64, c_i64,
                                    c_i64, c_i64, c_int, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp]),
    "xgb_fp8_wire_decode": (c_int, [c_vp, ctypes.POINTER(c_vp), c_int, c_i64, c_i64, c_i64,
                                    c_i64, c_int, c_vp]),
    "xgb_fp8_wire_encode_view": (c_int, [ctypes.POINTER(c_vp), c_i64p, c_int, c_i64, c_i64,
                                         c_i64, c_i64, c_i64, c_int, c_vp, c_vp, c_i64, c_i64,
                                         c_i64, c_vp, c_vp]),
    "xgb_fp8_wire_decode_view": (c_int, [c_vp, ctypes.POINTER(c_vp), c_i64p, c_int, c_i64, c_i64,
                                         c_i64, c_i64, c_i64, c_i64, c_i64, c_int, c_vp]),
    "xgb_fp8_wire_encode_peers": (c_int, [ctypes.POINTER(c_vp), c_i64p, c_int, c_i64, c_i64, c_i64,
                                          c_i64, c_vp, c_vp, c_i64, c_i64, ctypes.POINTER(c_vp), c_vp]),
    "xgb_peer_signal": (c_int, [ctypes.POINTER(c_vp), c_int, c_int, c_vp]),
    "xgb_peer_wait": (c_int, [ctypes.POINTER(c_vp), c_int, c_int, c_i64, c_vp, c_vp]),
    "xgb_fp8_quantize_per_tensor_workspace": (c_i64, [c_i64]),
    "xgb_fp8_quantize_per_tensor": (c_int, [c_vp, c_int, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp]),
    "xgb_fp8_abs_peak_scale": (c_int, [c_vp, c_int, c_i64, c_vp, c_vp, c_i64, c_vp]),
    "xgb_fp8_quantize_with_scale": (c_int, [c_vp, c_int, c_i64, c_vp, c_vp, c_vp]),
    "xgb_fp8_quantize_per_tensor_noalloc": (c_int, [c_vp, c_int, c_i64, c_vp, c_vp, c_vp]),
    "xgb_fp8_quantize_per_token": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp]),
    "xgb_fp8_gemm": (c_int, [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_int,
                             c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_i64, c_vp, c_vp]),
    "xgb_norm_modulate_quant": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_float,
                                        c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "xgb_sage_prepare_workspace": (c_i64, [c_i64, c_i64, c_i64]),
    "xgb_sage_prepare": (c_int, [c_vp, c_i64p, c_vp, c_i64p, c_vp, c_i64p, c_int, c_i64, c_i64,
                                 c_i64, c_i64, c_float, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                 c_i64, c_vp, c_vp]),
    "xgb_sage_prepare_rope": (c_int, [c_vp, c_i64p, c_vp, c_i64p, c_vp, c_i64p, c_i64, c_i64, c_i64,
                                      c_i64, c_float, c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp,
                                      c_vp, c_vp, c_i64, c_vp, c_vp]),
    "xgb_sage_prepare_wire": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_float, c_vp,
                                      c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp]),
    "xgb_attention_split_workspace_bytes": (c_i64, []),
    "xgb_sage_wire_stats_workspace": (c_i64, [c_i64, c_i64, c_i64, c_i64]),
    "xgb_sage_wire_stats": (c_int, [c_vp, c_i64p, c_vp, c_i64p, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp,
                                    c_i64, c_vp, c_vp, c_vp, c_i64, c_vp]),
    "xgb_sage_wire_encode": (c_int, [c_vp, c_i64p, c_vp, c_i64p, c_vp, c_i64p, c_i64, c_i64, c_i64,
                                     c_i64, c_vp, c_vp, c_i64, c_float, c_vp, c_vp, c_i64, c_vp,
                                     c_vp, c_vp, c_vp, c_vp, c_vp]),
    "xgb_attention_sage_strided": (c_int, [c_vp, c_i64p, c_vp, c_i64p, c_vp, c_i64p, c_vp, c_i64p,
                                           c_vp, c_i64p, c_vp, c_i64p, c_i64, c_i64, c_i64, c_i64,
                                           c_vp, c_i64p, c_vp, c_i64, c_vp, c_vp]),
    "xgb_attention_sage": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp,
                                   c_i64p, c_vp, c_i64, c_vp, c_vp]),
    "xgb_attention_bf16": (c_int, [c_vp, c_i64p, c_vp, c_i64p, c_vp, c_i64p, c_i64, c_i64, c_i64,
                                   c_i64, c_float, c_vp, c_i64p, c_vp, c_i64, c_vp, c_vp]),
}

_lock = threading.Lock()
_lib = None


class XGBError(RuntimeError):
    """A libxgb.so entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int):
        self.status = status
        super().__init__(f"{fn} failed: {status_string(status)} ({status})")


def lib() -> ctypes.CDLL:
    """The loaded library (loads it on first use; raises if unavailable)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python -m xgen_b200.build` "
                        "(xgen_b200 has no CPU fallback)")
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def status_string(status: int) -> str:
    try:
        return lib().xgb_status_string(status).decode()
    except Exception:  # pragma: no cover - only while the library is broken
        return "unknown status"


def check(fn: str, status: int) -> None:
    if status != XGB_OK:
        if status in (XGB_ERR_ARG, XGB_ERR_SHAPE, XGB_ERR_STRIDE, XGB_ERR_ALIGN):
            raise ValueError(f"{fn}: {status_string(status)} ({status})")
        raise XGBError(fn, status)


def call(name: str, *args) -> None:
    check(name, getattr(lib(), name)(*args))


def i64_array(values) -> ctypes.Array:
    values = list(values)
    return (c_i64 * len(values))(*values)


def ptr_array(values) -> ctypes.Array:
    values = list(values)
    return (c_vp * len(values))(*values)
