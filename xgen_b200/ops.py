"""torch-facing wrappers of the libxgb.so elementwise and FP8 operators.

Each function mirrors a reference operator (same name where the reference
exposes one, same argument meaning and error behaviour) and runs the
sm_100a kernel on the caller's current CUDA stream. There is no CPU path:
non-CUDA tensors raise ValueError (or return None where the reference's
`try_*` contract does so to select its own eager fallback).
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import call, i64_array

_DTYPE_CODE = {torch.bfloat16: _lib.XGB_BF16, torch.float16: _lib.XGB_F16}


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(*tensors: torch.Tensor, what: str) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise ValueError(f"{what} requires CUDA tensors")


def try_h3_partial_rope(query: torch.Tensor, key: torch.Tensor, cos: torch.Tensor,
                        sin: torch.Tensor):
    """Rotate-half RoPE over the first cos.shape[-1] channels of contiguous
    bf16 Q/K [B, S, H, D]; returns None for inputs the fused kernel does not
    take (the caller then runs its eager RoPE), exactly as
    x_base/x_base/operator/h3_partial_rope.py:32-47."""
    if (torch.is_grad_enabled() or not query.is_cuda or query.dtype != torch.bfloat16
            or query.ndim != 4 or query.shape != key.shape or key.dtype != query.dtype
            or cos.ndim != 2 or cos.shape != sin.shape or cos.shape[0] != query.shape[1]
            or cos.shape[-1] <= 0 or cos.shape[-1] % 2 or cos.shape[-1] > query.shape[-1]
            or cos.dtype != torch.float32 or sin.dtype != torch.float32
            or any(t.device != query.device or not t.is_contiguous()
                   for t in (query, key, cos, sin))):
        return None
    b, s, h, w = query.shape
    q_out, k_out = torch.empty_like(query), torch.empty_like(key)
    call("xgb_partial_rope", query.data_ptr(), key.data_ptr(), cos.data_ptr(), sin.data_ptr(),
         q_out.data_ptr(), k_out.data_ptr(), b, s, h, w, cos.shape[-1], _stream(query))
    return q_out, k_out


def try_h3_qk_rms(query: torch.Tensor, key: torch.Tensor, norm_q, norm_k, rotary_emb=None):
    """Per-head RMSNorm (times weight) of strided bf16 Q/K views [B, S, H, D],
    optionally fused with the partial RoPE; None when unsupported, as
    x_base/x_base/operator/h3_qk_rms.py:48-84."""
    if (torch.is_grad_enabled() or not query.is_cuda or query.ndim != 4 or query.numel() == 0
            or query.shape != key.shape or query.dtype != torch.bfloat16
            or key.dtype != query.dtype or query.stride(-1) != 1 or key.stride(-1) != 1
            or query.device != key.device or type(norm_q) is not torch.nn.RMSNorm
            or type(norm_k) is not torch.nn.RMSNorm or norm_q.eps is None or norm_k.eps is None):
        return None
    b, s, h, w = query.shape
    if w > 256:
        return None
    rotary, cos, sin = 0, None, None
    if rotary_emb is not None:
        cos, sin = rotary_emb
        if (cos.ndim != 2 or cos.shape != sin.shape or cos.shape[0] != s
                or not 0 < cos.shape[-1] <= w or cos.shape[-1] % 2
                or cos.dtype != torch.float32 or sin.dtype != torch.float32
                or any(t.device != query.device or not t.is_contiguous() for t in (cos, sin))):
            return None
        rotary = cos.shape[-1]
    weights = (norm_q.weight, norm_k.weight)
    if any(wt is None or wt.shape != (w,) or wt.dtype != query.dtype
           or wt.device != query.device or not wt.is_contiguous() for wt in weights):
        return None
    q_out = torch.empty(query.shape, device=query.device, dtype=query.dtype)
    k_out = torch.empty_like(q_out)
    call("xgb_qk_rms", query.data_ptr(), i64_array(query.stride()[:3]), key.data_ptr(),
         i64_array(key.stride()[:3]), weights[0].data_ptr(), weights[1].data_ptr(),
         float(norm_q.eps), float(norm_k.eps), cos.data_ptr() if cos is not None else None,
         sin.data_ptr() if sin is not None else None, rotary, q_out.data_ptr(), k_out.data_ptr(),
         b, s, h, w, _stream(query))
    return q_out, k_out


def indexed_affine(x: torch.Tensor, table: torch.Tensor, addend: torch.Tensor,
                   indices: torch.Tensor, *, modulation: bool) -> torch.Tensor:
    """AdaLN modulate (`modulation=True`: x*(1+table[idx]) + addend[idx]) or
    gated residual (`modulation=False`: addend + table[idx]*x) with the
    reference's bf16 rounding after each op; the CUDA branch of `_apply`,
    x_base/x_base/operator/h3_indexed_affine.py:32-49. Raises ValueError for
    layouts that branch does not take."""
    _require_cuda(x, table, addend, indices, what="H3 indexed affine")
    if not (x.ndim == 3 and x.is_contiguous() and indices.is_contiguous() and indices.ndim == 1
            and indices.numel() == x.shape[1] and indices.dtype == torch.int64
            and x.dtype == table.dtype == addend.dtype == torch.bfloat16
            and table.ndim == 2 and table.stride(-1) == 1 and table.shape[-1] == x.shape[-1]
            and (addend.stride(-1) == 1 if modulation else
                 (addend.is_contiguous() and addend.shape == x.shape))):
        raise ValueError("H3 indexed affine requires contiguous bf16 [B,S,H] input, int64 "
                         "indices [S] and row-strided bf16 tables")
    out = torch.empty_like(x)
    b, s, w = x.shape
    call("xgb_indexed_affine", x.data_ptr(), table.data_ptr(), table.stride(0), addend.data_ptr(),
         addend.stride(0) if modulation else 0, indices.data_ptr(), out.data_ptr(), b, s, w,
         int(modulation), _stream(x))
    return out


def gate_first_swiglu(x: torch.Tensor, *, with_amax: bool = False):
    """silu(gate) * value over a packed [..., 2F] bf16 tensor with eager bf16
    rounding; x_base/x_base/operator/h3_swiglu.py:31-41."""
    _require_cuda(x, what="H3 SwiGLU")
    if x.dtype != torch.bfloat16 or x.shape[-1] % 2 or not x.is_contiguous():
        raise ValueError("H3 SwiGLU requires a contiguous bf16 [..., 2F] tensor")
    width = x.shape[-1] // 2
    out = torch.empty((*x.shape[:-1], width), device=x.device, dtype=x.dtype)
    rows = out.numel() // width if width else 0
    amax = torch.zeros((), device=x.device, dtype=torch.float32) if with_amax else None
    call("xgb_swiglu", x.data_ptr(), out.data_ptr(), rows, width,
         amax.data_ptr() if amax is not None else None, _stream(x))
    return (out, amax) if with_amax else out


def quantize_activation(x: torch.Tensor, group=None):
    """Per-tensor dynamic e4m3 (scale = max(amax/448, FLT_MIN)); bit-exact
    with quantize_activation / quantize_per_tensor of
    x_base/x_base/operator/h3_fp8_quant.py:18-25 and h3_fp8.py:9-12. With a
    process group the scale is all-reduced with MAX before packing, so every
    rank of a tensor-parallel group packs with the same scale."""
    _require_cuda(x, what="H3 FP8 quantization")
    if x.dtype not in _DTYPE_CODE:
        raise ValueError("H3 FP8 quantization requires a bf16/fp16 tensor")
    x = x.contiguous()
    out = torch.empty(x.shape, device=x.device, dtype=torch.float8_e4m3fn)
    scale = torch.empty((), device=x.device, dtype=torch.float32)
    n = x.numel()
    if n == 0:
        scale.fill_(torch.finfo(torch.float32).tiny)
        if group is not None:
            import torch.distributed as dist

            dist.all_reduce(scale, op=dist.ReduceOp.MAX, group=group)
        return out, scale
    ws_bytes = _lib.lib().xgb_fp8_quantize_per_tensor_workspace(n)
    ws = torch.empty(max(ws_bytes, 4), device=x.device, dtype=torch.uint8)
    if group is None:
        call("xgb_fp8_quantize_per_tensor", x.data_ptr(), _DTYPE_CODE[x.dtype], n, out.data_ptr(),
             scale.data_ptr(), ws.data_ptr(), ws_bytes, _stream(x))
        return out, scale
    import torch.distributed as dist

    call("xgb_fp8_abs_peak_scale", x.data_ptr(), _DTYPE_CODE[x.dtype], n, scale.data_ptr(),
         ws.data_ptr(), ws_bytes, _stream(x))
    dist.all_reduce(scale, op=dist.ReduceOp.MAX, group=group)
    call("xgb_fp8_quantize_with_scale", x.data_ptr(), _DTYPE_CODE[x.dtype], n, scale.data_ptr(),
         out.data_ptr(), _stream(x))
    return out, scale


def norm_modulate_quant(x: torch.Tensor, norm: str, weight, eps: float, scale: torch.Tensor,
                        shift: torch.Tensor, indices: torch.Tensor, *, return_bf16: bool = False):
    """Fused AdaLN prologue: per-token e4m3 of
    bf16(bf16(norm(x) * bf16(1 + scale[idx])) + shift[idx]) for x [B, S, H]
    (norm "layernorm" without affine or "rmsnorm" x weight); returns
    (codes [B*S, H], scales [B*S]) and, with return_bf16, the modulated bf16."""
    _require_cuda(x, scale, shift, indices, what="H3 norm/modulate")
    if (x.ndim != 3 or x.dtype != torch.bfloat16 or x.stride(-1) != 1 or x.stride(0) != x.shape[1] * x.stride(1)
            or scale.dtype != torch.bfloat16 or shift.dtype != torch.bfloat16
            or scale.stride(-1) != 1 or shift.stride(-1) != 1 or indices.dtype != torch.int64
            or indices.numel() != x.shape[1] or norm not in ("layernorm", "rmsnorm")):
        raise ValueError("norm_modulate_quant needs bf16 [B,S,H] rows, bf16 tables, int64 [S] indices")
    b, s, h = x.shape
    rows = b * s
    codes = torch.empty((rows, h), device=x.device, dtype=torch.float8_e4m3fn)
    scales = torch.empty((rows,), device=x.device, dtype=torch.float32)
    mod = torch.empty((b, s, h), device=x.device, dtype=torch.bfloat16) if return_bf16 else None
    call("xgb_norm_modulate_quant", x.data_ptr(), x.stride(1), rows, h, s,
         1 if norm == "rmsnorm" else 0, weight.data_ptr() if weight is not None else None,
         float(eps), scale.data_ptr(), scale.stride(0), shift.data_ptr(), shift.stride(0),
         indices.contiguous().data_ptr(), codes.data_ptr(), scales.data_ptr(),
         mod.data_ptr() if mod is not None else None, _stream(x))
    return (codes, scales, mod) if return_bf16 else (codes, scales)


def output_adaln(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor,
                 indices: torch.Tensor, *, norm: str = "layernorm", weight=None,
                 eps: float = 1e-6, fused: bool = False) -> torch.Tensor:
    """Final-layer output AdaLN of the H3 transformer (`norm_out`,
    x_diffusers/x_diffusers/framework/transformer/minimax_h3.py:672-696):
    bf16(bf16(norm(x) * bf16(1 + scale[idx])) + shift[idx]); scale/shift are
    the [M, H] tables of lookup_final().

    Default: the reference's own LayerNorm followed by the bit-exact
    indexed-affine kernel, bitwise equal to the reference's fused output path
    (x_base/tests/test_h3_output_adaln.py:29-45). fused=True runs norm and
    modulation in one pass (xgb_norm_modulate_quant without the e4m3
    output), whose fp32 statistics can round a value one bf16 ulp apart."""
    _require_cuda(x, scale, shift, indices, what="H3 output AdaLN")
    if (x.ndim != 3 or x.dtype != torch.bfloat16 or x.stride(-1) != 1 or x.stride(0) != x.shape[1] * x.stride(1)
            or scale.dtype != torch.bfloat16 or shift.dtype != torch.bfloat16
            or scale.stride(-1) != 1 or shift.stride(-1) != 1 or indices.dtype != torch.int64
            or indices.numel() != x.shape[1] or norm not in ("layernorm", "rmsnorm")):
        raise ValueError("output_adaln needs bf16 [B,S,H] rows, bf16 tables, int64 [S] indices")
    b, s, h = x.shape
    if not fused:
        if norm == "layernorm":
            n = torch.nn.functional.layer_norm(x, (h,), eps=eps)
        else:
            n = torch.nn.functional.rms_norm(x, (h,), weight, eps=eps)
        return indexed_affine(n, scale, shift, indices, modulation=True)
    out = torch.empty((b, s, h), device=x.device, dtype=torch.bfloat16)
    call("xgb_norm_modulate_quant", x.data_ptr(), x.stride(1), b * s, h, s,
         1 if norm == "rmsnorm" else 0, weight.data_ptr() if weight is not None else None,
         float(eps), scale.data_ptr(), scale.stride(0), shift.data_ptr(), shift.stride(0),
         indices.contiguous().data_ptr(), None, None, out.data_ptr(), _stream(x))
    return out


def quantize_per_token(x: torch.Tensor):
    """Per-row dynamic e4m3 of a 2-D bf16/fp16 matrix: (codes, scales[rows])."""
    _require_cuda(x, what="H3 FP8 quantization")
    if x.dtype not in _DTYPE_CODE or x.ndim != 2 or x.stride(-1) != 1:
        raise ValueError("per-token FP8 quantization requires a row-major 2-D bf16/fp16 matrix")
    rows, cols = x.shape
    out = torch.empty((rows, cols), device=x.device, dtype=torch.float8_e4m3fn)
    scales = torch.empty((rows,), device=x.device, dtype=torch.float32)
    call("xgb_fp8_quantize_per_token", x.data_ptr(), _DTYPE_CODE[x.dtype], rows, cols,
         x.stride(0), out.data_ptr(), scales.data_ptr(), _stream(x))
    return out, scales
