"""fp32 restatement of the H3 DiT block (test infrastructure only).

Restates h3_block_forward (x_diffusers/x_diffusers/framework/transformer/
h3_npu_fusion.py:339-356) with unquantised fp32 math: AdaLN rows by index,
norm (LayerNorm without affine, or RMSNorm x weight), modulation, fused QKV
projection, optional per-head Q/K RMSNorm, rotate-half RoPE on the first R
channels (minimax_h3.py:72-114), non-causal attention, output projection,
gated residual, and the FFN (GELU, or the gate-first SwiGLU of
h3_swiglu.py:16-41). It is the reference's BF16/FP32 path that the FP8 +
Sage block is compared against.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def _norm(x, kind, weight, eps):
    if kind == "layernorm":
        return F.layer_norm(x, (x.shape[-1],), eps=eps)
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return y * weight if weight is not None else y


def _rope(x, cos, sin):
    r = cos.shape[-1]
    half = r // 2
    rot = x[..., :r]
    partner = torch.cat([-rot[..., half:], rot[..., :half]], dim=-1)
    out = x.clone()
    out[..., :r] = rot * cos[None, :, None, :] + partner * sin[None, :, None, :]
    return out


def block_forward(x, weights, table, indices, cos, sin, cfg):
    """x [B, S, H] fp32 (the full sequence), weights as H3DiTBlockB200.random_weights,
    table [rows, 6H]; returns the block output in fp32."""
    w = {k: v.float() for k, v in weights.items()}
    b, s, h = x.shape
    t = table.float()[indices]  # [S, 6H]
    shift, scale, gate, shift_ff, scale_ff, gate_ff = t.chunk(6, dim=-1)
    n = _norm(x, cfg.norm, w.get("norm1.weight"), cfg.eps) * (1 + scale) + shift
    qkv = n @ w["to_qkv"].T
    q, k, v = (z.unflatten(-1, (cfg.heads, cfg.head_dim)) for z in qkv.chunk(3, dim=-1))
    if cfg.qk_norm:
        q = _norm(q, "rmsnorm", w["norm_q.weight"], cfg.eps)
        k = _norm(k, "rmsnorm", w["norm_k.weight"], cfg.eps)
    q, k = _rope(q, cos, sin), _rope(k, cos, sin)
    att = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
    att = att.transpose(1, 2).flatten(2)
    x = x + gate * (att @ w["to_out"].T)
    n = _norm(x, cfg.norm, w.get("norm2.weight"), cfg.eps) * (1 + scale_ff) + shift_ff
    u = n @ w["ff_up"].T
    if cfg.activation == "gelu":
        u = F.gelu(u)
    else:
        g_, v_ = u.chunk(2, dim=-1)
        u = F.silu(g_) * v_
    return x + gate_ff * (u @ w["ff_down"].T)
