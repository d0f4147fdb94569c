"""numpy restatements of the reference's elementwise Triton kernels.

Test infrastructure only. Inputs/outputs are fp32 arrays holding exact bf16
values (use oracle.numerics to convert bit images). Every operation is fp32
with an explicit bf16 rounding wherever the reference rounds, and no fused
multiply-add (the reference compiles with enable_fp_fusion=False).
"""
from __future__ import annotations

import numpy as np

from .numerics import bf16_round, fdiv

f32 = np.float32


def partial_rope(q: np.ndarray, k: np.ndarray, cos: np.ndarray, sin: np.ndarray):
    """Rotate-half RoPE over the first R = cos.shape[-1] channels of Q and K
    [batch, seq, heads, width]; x_base/x_base/operator/h3_partial_rope.py:9-29."""
    return _rope(q, cos, sin), _rope(k, cos, sin)


def _rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    r = cos.shape[-1]
    half = r // 2
    x = x.astype(f32)
    c = bf16_round(cos.astype(f32))[None, :, None, :]  # [1, S, 1, R]
    s = bf16_round(sin.astype(f32))[None, :, None, :]
    rot = x[..., :r]
    partner = np.concatenate([-rot[..., half:], rot[..., :half]], axis=-1)
    left = bf16_round(rot * c)
    right = bf16_round(partner * s)
    out = x.copy()
    out[..., :r] = bf16_round(left + right)
    return out


def qk_rms(q: np.ndarray, k: np.ndarray, q_weight: np.ndarray, k_weight: np.ndarray,
           q_eps: float, k_eps: float, cos=None, sin=None):
    """Per-head RMSNorm times weight, then optional RoPE;
    x_base/x_base/operator/h3_qk_rms.py:9-45. Q/K [batch, seq, heads, width]."""
    return (_rms(q, q_weight, q_eps, cos, sin), _rms(k, k_weight, k_eps, cos, sin))


def _rms(x, w, eps, cos, sin):
    x = x.astype(f32)
    width = x.shape[-1]
    ss = np.sum(x * x, axis=-1, dtype=f32)
    scale = (f32(1.0) / np.sqrt(fdiv(ss, f32(width)) + f32(eps))).astype(f32)[..., None]
    normed = bf16_round((x * scale).astype(f32) * w.astype(f32))
    if cos is None:
        return normed
    r = cos.shape[-1]
    half = r // 2
    c = bf16_round(cos.astype(f32))[None, :, None, :]
    s = bf16_round(sin.astype(f32))[None, :, None, :]
    rot = normed[..., :r]
    partner = np.concatenate([-rot[..., half:], rot[..., :half]], axis=-1)
    out = normed.copy()
    out[..., :r] = bf16_round(bf16_round(rot * c) + bf16_round(partner * s))
    return out


def indexed_affine(x: np.ndarray, table: np.ndarray, addend: np.ndarray, indices: np.ndarray,
                   modulation: bool) -> np.ndarray:
    """modulation: bf16(bf16(x*bf16(1+table[idx])) + addend[idx]);
    gate: bf16(bf16(x*table[idx]) + addend);
    x_base/x_base/operator/h3_indexed_affine.py:9-49. x [batch, seq, width]."""
    factor = table[indices].astype(f32)[None]
    if modulation:
        factor = bf16_round(f32(1.0) + factor)
        bias = addend[indices].astype(f32)[None]
    else:
        bias = addend.astype(f32)
    return bf16_round(bf16_round(x.astype(f32) * factor) + bias)


def swiglu(x: np.ndarray):
    """Gate-first packed SwiGLU with the reference's rounding and its
    NaN-propagating abs-peak; x_base/x_base/operator/h3_swiglu.py:15-41."""
    width = x.shape[-1] // 2
    g = x[..., :width].astype(f32)
    v = x[..., width:].astype(f32)
    act = bf16_round(fdiv(g, f32(1.0) + np.exp(-g).astype(f32)))
    out = bf16_round(act * v)
    peak = f32(np.nan) if np.isnan(out).any() else f32(np.abs(out).max(initial=0.0))
    return out, peak
