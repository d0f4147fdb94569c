"""The allocation-free per-tensor FP8 quantiser, checked through the C ABI.

xgb_fp8_quantize_per_tensor_noalloc serves callers that cannot allocate
device memory when they call in (a plugin whose host runtime owns every
allocation, a server that plans all of HBM ahead, a latency-critical path
that cannot take cudaMalloc's device synchronisation): it keeps its scratch
in a fixed array inside libxgb.so instead of a caller workspace. This test
compares it with the workspace entry point, bit for bit, on two calls in a
row (the second call reuses the array the first one left behind). It lives
in its own file, named to be collected last."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _with_workspace(lib, x):
    n = x.numel()
    out = torch.empty(n, dtype=torch.uint8, device=x.device)
    scale = torch.empty(1, dtype=torch.float32, device=x.device)
    ws_bytes = lib.xgb_fp8_quantize_per_tensor_workspace(n)
    ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=x.device)
    rc = lib.xgb_fp8_quantize_per_tensor(x.data_ptr(), 0, n, out.data_ptr(), scale.data_ptr(),
                                         ws.data_ptr(), ws_bytes, _stream())
    assert rc == 0
    return out, scale


def _no_alloc(lib, x):
    n = x.numel()
    out = torch.empty(n, dtype=torch.uint8, device=x.device)
    scale = torch.empty(1, dtype=torch.float32, device=x.device)
    rc = lib.xgb_fp8_quantize_per_tensor_noalloc(x.data_ptr(), 0, n, out.data_ptr(),
                                                 scale.data_ptr(), _stream())
    assert rc == 0, lib.xgb_status_string(rc)
    return out, scale


def test_no_alloc_matches_workspace_entry_point(cuda_device):
    from xgen_b200 import _lib

    lib = _lib.lib()
    g = torch.Generator(device=cuda_device).manual_seed(11)
    # two calls in a row: a large tensor, then a smaller one with a larger
    # peak, so stale peaks from the first call would show in the second
    first = torch.randn(3000, 5376, device=cuda_device, generator=g).bfloat16()
    second = (torch.randn(997, 1000, device=cuda_device, generator=g) * 40).bfloat16()
    for x in (first, second):
        ref_q, ref_s = _with_workspace(lib, x)
        got_q, got_s = _no_alloc(lib, x)
        torch.cuda.synchronize()
        assert torch.equal(got_s, ref_s)
        assert torch.equal(got_q, ref_q)


def test_no_alloc_rejects_sizes_beyond_its_scratch(cuda_device):
    from xgen_b200 import _lib

    lib = _lib.lib()
    dummy = ctypes.c_void_p(16)
    too_many = 65536 * 8192 + 1
    assert lib.xgb_fp8_quantize_per_tensor_noalloc(dummy, 0, too_many, dummy, dummy,
                                                   _stream()) == _lib.XGB_ERR_SHAPE
