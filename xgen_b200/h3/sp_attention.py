"""The H3 self-attention core between the QKV projection and `to_out`.

`sp_self_attention` is the part of AscendMiniMaxH3AttnProcessor.__call__
(x_diffusers/x_diffusers/framework/transformer/minimax_h3.py:165-247) that
runs after Q/K normalisation: partial RoPE, the Ulysses/PHAA redistribution
when SP > 1, the attention backend, and the return redistribution. With the
FP8 wire the RoPE is fused into the wire encode; at SP = 1 a Sage backend
applies it inside its quantisation kernels (a standalone RoPE kernel runs
otherwise), and the backend writes straight into the (B, S, H, D) output.
"""
from __future__ import annotations

import torch

from ..ops import try_h3_partial_rope
from ..phaa.phaa_attention import run_phaa_attention
from ..sp.comm import all_to_all_after_attn, all_to_all_before_attn


def sp_self_attention(query, key, value, rotary_emb, *, backend, heads: int, head_dim: int = 128,
                      sp_group=None, sp_size: int = 1, phaa_num: int = 2,
                      fp8_transport: bool = True, comm_stream=None, pad_key: str = "mmh3_seq",
                      device_join: bool = True, use_phaa: bool = True, int8_transport: bool = False,
                      attention_mask=None):
    """query/key/value (B, S_loc, heads*head_dim) bf16 -> (B, S_loc, heads*head_dim).
    int8_transport: Sage-quantise before the exchange (xgen_b200.phaa.sage_wire)
    and return the output over the FP8 wire. attention_mask goes to the
    backend, which takes its masked path for it (as the reference's
    attention backends do)."""
    b, s, _ = query.shape
    with torch.no_grad():
        if sp_size > 1 and int8_transport and attention_mask is None:
            return run_phaa_attention(
                query, key, value, comm_stream=comm_stream, sp_group=sp_group, sp_size=sp_size,
                heads=heads, phaa_split_num=1, head_dim=head_dim, rotary_emb=rotary_emb,
                pad_key=pad_key, attention_fn=backend, fp8_transport=True,
                device_join=device_join, int8_transport=True)
        if sp_size > 1 and use_phaa:
            if not fp8_transport and rotary_emb is not None:
                query, key = _rope(query, key, rotary_emb, heads, head_dim)
            return run_phaa_attention(
                query, key, value, comm_stream=comm_stream, sp_group=sp_group, sp_size=sp_size,
                heads=heads, phaa_split_num=phaa_num, head_dim=head_dim,
                rotary_emb=rotary_emb if fp8_transport else None, pad_key=pad_key,
                attention_fn=backend, fp8_transport=fp8_transport, device_join=device_join,
                fuse_rope=fp8_transport and rotary_emb is not None, attention_mask=attention_mask)
        fuse = (rotary_emb is not None and sp_size == 1 and attention_mask is None
                and callable(getattr(backend, "fuses_rope", None)) and backend.fuses_rope(query))
        if rotary_emb is not None and not fuse:
            query, key = _rope(query, key, rotary_emb, heads, head_dim)
        q4 = query.unflatten(-1, (heads, head_dim))
        k4 = key.unflatten(-1, (heads, head_dim))
        v4 = value.unflatten(-1, (heads, head_dim))
        if sp_size > 1:
            q4, k4, v4 = (all_to_all_before_attn(t, sp_group, 2, 1, pad_key) for t in (q4, k4, v4))
        out = torch.empty(q4.shape, device=q4.device, dtype=q4.dtype)
        extra = {"rotary_emb": rotary_emb} if fuse else {}
        res = backend(q4.transpose(1, 2), k4.transpose(1, 2), v4.transpose(1, 2),
                      attn_mask=attention_mask, out=out.transpose(1, 2), **extra)
        if res.data_ptr() != out.data_ptr():
            out.copy_(res.transpose(1, 2))
        if sp_size > 1:
            out = all_to_all_after_attn(out, sp_group, 1, 2, pad_key)
        return out.flatten(2)


def _rope(query, key, rotary_emb, heads, head_dim):
    q4 = query.unflatten(-1, (heads, head_dim))
    k4 = key.unflatten(-1, (heads, head_dim))
    if not q4.is_contiguous():
        q4 = q4.contiguous()
    if not k4.is_contiguous():
        k4 = k4.contiguous()
    rotated = try_h3_partial_rope(q4, k4, *rotary_emb)
    if rotated is None:
        raise ValueError("H3 RoPE tables must be fp32 [S, R] with even R <= head_dim")
    return rotated[0].flatten(2), rotated[1].flatten(2)
