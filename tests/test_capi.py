"""The C-ABI library loads and exports every entry point include/xgb.h
declares (no GPU needed: nothing here launches a kernel)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "xgb.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(xgb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "xgb_attention_sage" in names and "xgb_fp8_wire_encode" in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol():
    from xgen_b200 import _lib

    handle = _lib.lib()
    missing = [n for n in declared_symbols() if not hasattr(handle, n)]
    assert not missing, missing


def test_ctypes_table_matches_header():
    from xgen_b200 import _lib

    assert set(_lib.SIGNATURES) == set(declared_symbols())


def test_version_and_status_strings():
    from xgen_b200 import _lib

    h = _lib.lib()
    assert h.xgb_version() >= 100
    assert _lib.status_string(-2) == "unsupported shape"
    assert _lib.status_string(0) == "ok"


def test_argument_errors_without_gpu():
    """Null pointers and bad sizes are rejected before any CUDA call."""
    from xgen_b200 import _lib

    h = _lib.lib()
    assert h.xgb_partial_rope(None, None, None, None, None, None, 1, 1, 1, 128, 96, None) == -1
    dummy = ctypes.c_void_p(16)
    assert h.xgb_partial_rope(dummy, dummy, dummy, dummy, dummy, dummy, 1, 1, 1, 128, 95, None) == -2
    assert h.xgb_fp8_quantize_per_tensor(dummy, 0, 100, dummy, dummy, None, 0, None) == -7
    assert h.xgb_fp8_quantize_per_tensor_workspace(8193) == 8
    strides = _lib.i64_array([0, 0, 0, 1])
    assert h.xgb_attention_sage(dummy, dummy, dummy, dummy, dummy, dummy, 1, 1, 0, dummy, strides,
                                None, 0, None, None) == -2
    # Sage preparation from the FP8 wire: pointers, layout and alignment
    prep = lambda *a: h.xgb_sage_prepare_wire(*a)  # noqa: E731
    ok = (dummy, 2, 64, 1, 3, 100, 0, ctypes.c_float(0.088), dummy, dummy, dummy, dummy, dummy, dummy,
          dummy, 1 << 20, None, None)
    assert prep(None, *ok[1:]) == -1                                   # null payload
    assert prep(*ok[:5], 129, *ok[6:]) == -2                           # valid_seq > peers * seq
    assert prep(*ok[:6], 2, *ok[7:]) == -1                             # padding not a multiple of 4
    assert prep(ctypes.c_void_p(18), *ok[1:]) == -4                    # payload not 4-byte aligned
    assert prep(*ok[:14], dummy, 16, None, None) == -7                 # workspace too small


def test_fused_rope_prepare_argument_errors_without_gpu():
    """xgb_sage_prepare_rope rejects bad RoPE widths, strides, alignment and
    a short workspace before any CUDA call."""
    from xgen_b200 import _lib

    h = _lib.lib()
    d = ctypes.c_void_p(1 << 20)  # 16-byte aligned stand-in pointer (never dereferenced)
    st = _lib.i64_array([300 * 2 * 128, 128, 2 * 128, 1])
    f = ctypes.c_float(0.088)

    def call(*, cos=d, rotary=96, strides=st, ws_bytes=1 << 30, q=d):
        return h.xgb_sage_prepare_rope(q, strides, d, strides, d, strides, 1, 2, 300, 128, f, cos, d,
                                       rotary, d, d, d, d, d, d, d, ws_bytes, None, None)

    assert call(q=None) == -1                                  # null input
    assert call(rotary=90) == -2                               # rotary/2 not a multiple of 8
    assert call(rotary=144) == -2                              # wider than the head
    assert call(strides=_lib.i64_array([300 * 256, 128, 256, 2])) == -3  # channel stride
    assert call(cos=ctypes.c_void_p((1 << 20) + 4)) == -4      # cos table not 16-byte aligned
    assert call(ws_bytes=16) == -7                             # workspace too small


def test_ops_refuse_cpu_tensors():
    torch = pytest.importorskip("torch")
    from xgen_b200 import ops

    x = torch.zeros(2, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.indexed_affine(x, x[0], x[0], torch.zeros(4, dtype=torch.long), modulation=True)
    with pytest.raises(ValueError, match="CUDA"):
        ops.quantize_activation(x)
