"""Drop-in H3 attention processor and the recipe installer for the B200 path.

`H3AttnProcessorB200` takes the place of the reference's SP attention
processor, `AscendMiniMaxH3AttnProcessor.__call__(attn, hidden_states,
rotary_emb=None, attention_mask=None)` (x_diffusers/x_diffusers/framework/
transformer/minimax_h3.py:129-251). It reads the same attributes from the
attention module:

  attn.to_qkv (fused) or to_q/to_k/to_v, attn.heads, attn.norm_q/norm_k,
  attn.to_out[0] / to_out[1], attn.parallel_manager (.sp_group, .sp_size),
  attn._h3_attention_backend, attn._h3_fused_qk_rms, attn._h3_phaa_fp8,
  attn._h3_tp_cp (picks the 'mmh3_seq' pad key for plain Ulysses).

and runs QKV -> Q/K RMSNorm -> RoPE -> SP redistribution -> attention ->
return -> to_out on this library's kernels (`sp_self_attention`).

`install(transformer, precision, ...)` is the switch the reference flips with
`--h3_cuda_precision {fp8-sage, fp8-bf16}` and XGEN_PHAA_FP8:
`prepare_transformer` (x_diffusers/x_diffusers/adaptor/h3_cuda_precision.py
:213-311) swaps the four projections of every block for FP8 Linears and sets
one shared attention backend; `configure_parallelism`
(x_diffusers/x_diffusers/adaptor/h3_cuda.py:82-181) sets the PHAA FP8
transport flags; `install_dit_fusions` (h3_cuda.py:32-52) enables the fused
Q/K RMSNorm and RoPE and replaces the block forward. Here the replaced block
forward runs the whole block on the fused B200 kernels (`H3DiTBlockB200`,
sharing the installed modules) and falls back to the module-by-module
composition of the reference's fused_h3_block_forward
(x_base/x_base/operator/h3_indexed_affine.py:52-61) for masks, autograd or a
layout the fused block does not cover.
"""
from __future__ import annotations

import os
from types import MethodType

import torch
from torch import nn

from ..attention import H3AttentionBackendB200
from ..fp8_linear import H3FP8Linear
from ..ops import indexed_affine, try_h3_qk_rms
from .block import H3BlockConfig, H3DiTBlockB200
from .sp_attention import sp_self_attention

PRECISIONS = {"fp8-sage": "sage", "fp8-bf16": "bf16"}


def _sp(attn):
    manager = getattr(attn, "parallel_manager", None)
    if manager is None:
        return None, 1
    return manager.sp_group, manager.sp_size


class H3AttnProcessorB200:
    """SP self-attention of one H3 attention module on the B200 kernels.

    The PHAA exchange runs on `comm_stream` (one per processor and device,
    created on first use), as the reference processor's own comm stream."""

    def __init__(self):
        self._streams: dict[int, torch.cuda.Stream] = {}

    def comm_stream(self, device: torch.device):
        idx = device.index if device.index is not None else torch.cuda.current_device()
        stream = self._streams.get(idx)
        if stream is None:
            stream = self._streams[idx] = torch.cuda.Stream(device=device)
        return stream

    def __call__(self, attn, hidden_states, rotary_emb=None, attention_mask=None):
        heads = attn.heads
        if getattr(attn, "fused_projections", False):
            query, key, value = attn.to_qkv(hidden_states).chunk(3, dim=-1)
        else:
            query, key, value = attn.to_q(hidden_states), attn.to_k(hidden_states), attn.to_v(hidden_states)
        head_dim = query.shape[-1] // heads
        q4, k4 = query.unflatten(-1, (heads, head_dim)), key.unflatten(-1, (heads, head_dim))
        norm_q, norm_k = getattr(attn, "norm_q", None), getattr(attn, "norm_k", None)
        if norm_q is not None:
            normed = None
            if getattr(attn, "_h3_fused_qk_rms", False):
                normed = try_h3_qk_rms(q4, k4, norm_q, norm_k)
            q4, k4 = normed if normed is not None else (norm_q(q4), norm_k(k4))
        sp_group, sp_size = _sp(attn)
        backend = getattr(attn, "_h3_attention_backend", None)
        if backend is None:
            backend = attn._h3_attention_backend = H3AttentionBackendB200("bf16")
        phaa_num = getattr(attn, "_h3_phaa_num", 0)
        fp8_wire = bool(getattr(attn, "_h3_phaa_fp8", False))
        use_phaa = sp_size > 1 and phaa_num >= 1
        pad_key = "mmh3_seq" if use_phaa or getattr(attn, "_h3_tp_cp", False) else "pad"
        out = sp_self_attention(
            q4.flatten(2), k4.flatten(2), value, rotary_emb, backend=backend, heads=heads,
            head_dim=head_dim, sp_group=sp_group, sp_size=sp_size,
            phaa_num=min(max(phaa_num, 1), max(1, heads // max(sp_size, 1))),
            fp8_transport=fp8_wire, use_phaa=use_phaa,
            comm_stream=self.comm_stream(hidden_states.device) if sp_size > 1 else None,
            pad_key=pad_key, attention_mask=attention_mask)
        out = out.type_as(hidden_states)
        out = attn.to_out[0](out)
        return attn.to_out[1](out)


# ---------------------------------------------------------------- installer
def _linear(module: nn.Module, scaling: str, device) -> H3FP8Linear:
    return H3FP8Linear(module.weight.detach(), module.bias.detach() if module.bias is not None else None,
                       scaling=scaling).to(device)


def _norm_kind(norm):
    """(kind, weight, eps) of a block norm the fused prologue computes, or
    None: LayerNorm without affine parameters, or RMSNorm (weight optional)."""
    if isinstance(norm, nn.LayerNorm) and not norm.elementwise_affine:
        return "layernorm", None, float(norm.eps)
    if isinstance(norm, nn.RMSNorm):
        # eps None: torch uses the input dtype's epsilon (the block runs in bf16)
        eps = norm.eps if norm.eps is not None else torch.finfo(torch.bfloat16).eps
        weight = norm.weight.detach().to(torch.bfloat16) if norm.weight is not None else None
        return "rmsnorm", weight, float(eps)
    return None


def _activation(act):
    """FFN activation module -> H3BlockConfig.activation, or None."""
    if "swiglu" in type(act).__name__.lower():
        return "swiglu"
    approximate = getattr(act, "approximate", None)
    if approximate == "none":
        return "gelu"
    if approximate == "tanh":
        return "gelu_tanh"
    return None


def _fused_block(block, precision, scaling, device):
    """An H3DiTBlockB200 over the installed modules, or None when the
    block's layout has no fused equivalent (the installed forward then runs
    module by module)."""
    attn, ff = block.attn, block.ff
    n1, n2 = _norm_kind(getattr(block, "norm1", None)), _norm_kind(getattr(block, "norm2", None))
    act = _activation(ff.net[0])
    if n1 is None or n2 is None or n1[0] != n2[0] or act is None:
        return None
    if len(ff.net) != 3 or not isinstance(ff.net[2], H3FP8Linear):
        return None
    norm_q, norm_k = getattr(attn, "norm_q", None), getattr(attn, "norm_k", None)
    qk = isinstance(norm_q, nn.RMSNorm) and isinstance(norm_k, nn.RMSNorm)
    if (norm_q is not None or norm_k is not None) and not qk:
        return None
    hidden = attn.to_qkv.in_features
    config = H3BlockConfig(hidden=hidden, heads=attn.heads, head_dim=hidden // attn.heads,
                           ffn=ff.net[2].in_features, activation=act, norm=n1[0], qk_norm=qk,
                           eps=n1[2], precision=precision, fp8_scaling=scaling)
    return H3DiTBlockB200.from_modules(
        config, device, to_qkv=attn.to_qkv, to_out=attn.to_out[0], ff_up=ff.net[0].proj,
        ff_down=ff.net[2], norm1_weight=n1[1], norm2_weight=n2[1],
        norm_q=attn.norm_q if qk else None, norm_k=attn.norm_k if qk else None,
        attention=attn._h3_attention_backend)


def h3_block_forward_b200(self, hidden_states, temb, adaln_indices, rotary_emb, attention_mask=None):
    """The installed H3 block forward (same signature as the reference's
    block forward): the fused B200 block when it applies, else the
    module-by-module composition of fused_h3_block_forward."""
    tables = self.adaln_proj(temb)
    fused = getattr(self, "_h3_b200_block", None)
    if (fused is not None and attention_mask is None and not torch.is_grad_enabled()
            and hidden_states.dtype == torch.bfloat16 and hidden_states.ndim == 3):
        attn = self.attn
        processor = getattr(attn, "processor", None)
        sp_group, sp_size = _sp(attn)
        phaa_num = getattr(attn, "_h3_phaa_num", 0)
        comm = (processor.comm_stream(hidden_states.device)
                if sp_size > 1 and isinstance(processor, H3AttnProcessorB200) else None)
        table = torch.cat([t.to(torch.bfloat16) for t in tables], dim=-1)
        return fused.forward(hidden_states, table, adaln_indices, rotary_emb, sp_group=sp_group,
                             sp_size=sp_size, phaa_num=min(max(phaa_num, 1), max(1, attn.heads // sp_size)),
                             fp8_transport=bool(getattr(attn, "_h3_phaa_fp8", False)),
                             comm_stream=comm, use_phaa=sp_size > 1 and phaa_num >= 1)
    shift, scale, gate, shift_ff, scale_ff, gate_ff = tables
    normed = indexed_affine(self.norm1(hidden_states), scale, shift, adaln_indices, modulation=True)
    branch = self.attn(normed, rotary_emb, attention_mask)
    hidden_states = indexed_affine(branch, gate, hidden_states, adaln_indices, modulation=False)
    normed = indexed_affine(self.norm2(hidden_states), scale_ff, shift_ff, adaln_indices, modulation=True)
    return indexed_affine(self.ff(normed), gate_ff, hidden_states, adaln_indices, modulation=False)


def _set_processor(attn, processor):
    if callable(getattr(attn, "set_processor", None)):
        attn.set_processor(processor)
    else:
        attn.processor = processor


def install(transformer, precision: str = "fp8-sage", *, parallel_manager=None,
            phaa_num: int | None = None, fp8_transport: bool | None = None,
            scaling: str = "per_token", device=None):
    """Install the B200 SP attention path on an H3 transformer in place.

    precision      "fp8-sage" (INT8/FP8 Sage attention) or "fp8-bf16" (BF16
                   attention); the projections become FP8 Linears either way.
    parallel_manager  attached to the transformer and every block's attention
                   (its .sp_group / .sp_size drive the SP redistribution).
    phaa_num       PHAA head chunks per attention call (the reference's
                   --phaa_num); 0 or None at SP > 1 uses plain Ulysses unless
                   the FP8 transport is on, which needs a valid value.
    fp8_transport  the PHAA FP8 wire; None reads XGEN_PHAA_FP8 == "1".
    scaling        FP8 activation scaling of the projections: "per_token"
                   (B200 default) or "per_tensor" (the reference's).
    Returns the shared attention backend."""
    if precision not in PRECISIONS:
        raise ValueError(f"Unsupported H3 CUDA precision {precision!r}; use fp8-sage or fp8-bf16")
    blocks = list(getattr(transformer, "transformer_blocks", []))
    if not blocks:
        raise ValueError("H3 transformer has no transformer_blocks")
    if parallel_manager is not None:
        if callable(getattr(transformer, "set_parallel_manager", None)):
            transformer.set_parallel_manager(parallel_manager)
        else:
            transformer.parallel_manager = parallel_manager
            for block in blocks:
                block.attn.parallel_manager = parallel_manager
    sp_size = getattr(parallel_manager, "sp_size", None) or getattr(
        getattr(blocks[0].attn, "parallel_manager", None), "sp_size", 1)
    if fp8_transport is None:
        fp8_transport = os.environ.get("XGEN_PHAA_FP8") == "1"
    local_heads = blocks[0].attn.heads // max(1, sp_size)
    if fp8_transport and (sp_size < 2 or phaa_num is None or not 1 <= phaa_num <= local_heads):
        raise ValueError("XGEN_PHAA_FP8=1 requires H3, SP > 1, and a valid --phaa_num")
    if phaa_num is not None and phaa_num > max(1, local_heads):
        raise ValueError(f"--phaa_num {phaa_num} exceeds the {local_heads} local heads")
    # validate every block before converting any
    for block in blocks:
        attn = block.attn
        if getattr(attn, "fused_projections", False) or not all(
                isinstance(getattr(attn, name, None), nn.Linear) for name in ("to_q", "to_k", "to_v")):
            raise ValueError("FP8 recipe expects original unfused BF16 H3 projections")
        has_bias = [getattr(attn, name).bias is not None for name in ("to_q", "to_k", "to_v")]
        if any(has_bias) and not all(has_bias):
            raise ValueError("H3 QKV biases must either all exist or all be absent")
    device = torch.device(device) if device is not None else blocks[0].attn.to_q.weight.device
    backend = H3AttentionBackendB200(PRECISIONS[precision])
    processor = H3AttnProcessorB200()
    for block in blocks:
        attn = block.attn
        q, k, v = attn.to_q, attn.to_k, attn.to_v
        qkv = nn.Linear(q.in_features, 3 * q.out_features, bias=q.bias is not None)
        qkv.weight = nn.Parameter(torch.cat([q.weight.detach(), k.weight.detach(), v.weight.detach()]),
                                  requires_grad=False)
        if q.bias is not None:
            qkv.bias = nn.Parameter(torch.cat([q.bias.detach(), k.bias.detach(), v.bias.detach()]),
                                    requires_grad=False)
        attn.to_qkv = _linear(qkv, scaling, device)
        attn.to_q = attn.to_k = attn.to_v = None
        attn.fused_projections = True
        attn.to_out[0] = _linear(attn.to_out[0], scaling, device)
        block.ff.net[0].proj = _linear(block.ff.net[0].proj, scaling, device)
        block.ff.net[2] = _linear(block.ff.net[2], scaling, device)
        for norm in (getattr(attn, "norm_q", None), getattr(attn, "norm_k", None),
                     getattr(block, "norm1", None), getattr(block, "norm2", None)):
            if norm is not None:
                norm.to(device)
        attn._h3_attention_backend = backend
        attn._h3_fused_qk_rms = True
        attn._h3_fused_partial_rope = True
        attn._h3_phaa_fp8 = bool(fp8_transport)
        attn._h3_phaa_num = int(phaa_num or 0)
        _set_processor(attn, processor)
        if not hasattr(block, "_h3_eager_forward"):
            block._h3_eager_forward = block.forward
        block._h3_b200_block = _fused_block(block, PRECISIONS[precision], scaling, device)
        block.forward = MethodType(h3_block_forward_b200, block)
    transformer._h3_cuda_precision = precision
    setattr(transformer, "_h3_sage_cuda" if precision == "fp8-sage" else "_h3_dense_cuda", backend)
    return backend
