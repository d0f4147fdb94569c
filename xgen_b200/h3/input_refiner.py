"""Opt-in SP path for the H3 input token refiner (the text-conditioning
transformer ahead of the DiT), on the B200 attention and FP8 linears.

Same interface and behaviour as x_diffusers/x_diffusers/adaptor/
h3_input_refiner.py:13-148:
- `install_input_refiner(model, profile)` with profile "cudnn-sp" (BF16
  attention, BF16 FFN), "cudnn-sp-fp8" (FP8 FFN projections) or "custom";
- the refiner's forward splits the tokens over the SP group (pad key
  "h3_input_refiner", so the DiT's "mmh3_seq" pad is untouched), runs its
  blocks on the local tokens and gathers the result;
- every block's attention exchanges Q/K/V seq->head and back with the
  Ulysses all-to-all and runs full-context BF16 attention on its heads;
- `convert_ffn` swaps each FFN Linear for an H3FP8Linear whose activation
  scale is MAX-reduced over the SP group, so every rank packs with the
  scale the unsharded tokens would give.

The "cudnn" attention of the reference (H3DenseCUDA) is the tcgen05 BF16
kernel here (H3AttentionBackendB200("bf16")). Inference only.
"""
from __future__ import annotations

import logging
from functools import wraps

import torch
import torch.distributed as dist

from ..attention import H3AttentionBackendB200
from ..fp8_linear import H3FP8Linear
from ..sp.comm import all_to_all_after_attn, all_to_all_before_attn, gather_sequence, split_sequence
from ..sp.padding import set_pad

logger = logging.getLogger(__name__)
PAD_KEY = "h3_input_refiner"
PROFILES = ("none", "cudnn-sp", "cudnn-sp-fp8")


class RefinerSPAttention:
    """BF16 full-context attention with heads distributed over the SP group
    (a diffusers attention processor: called with the attention module)."""

    def __init__(self, group, backend, metrics):
        self.group, self.backend, self.metrics = group, backend, metrics

    def __call__(self, attn, hidden_states, rotary_emb=None, attention_mask=None):
        if rotary_emb is not None or attention_mask is not None or attn.fused_projections:
            raise ValueError("H3 input refiner SP expects unfused QKV, no RoPE and no mask")
        query, key, value = (layer(hidden_states).unflatten(-1, (attn.heads, attn.head_dim))
                             for layer in (attn.to_q, attn.to_k, attn.to_v))
        query, key = attn.norm_q(query), attn.norm_k(key)
        if any(t.dtype != torch.bfloat16 for t in (query, key, value)):
            raise ValueError("H3 input refiner attention requires BF16 QKV")
        self.metrics["attention_calls"] += 1
        if self.group is not None:
            self.metrics["logical_sp_payload_bytes"] += 4 * query.numel() * query.element_size()
            # the tail pad is removed before attention and restored after it
            query, key, value = (all_to_all_before_attn(t, self.group, pad_key=PAD_KEY)
                                 for t in (query, key, value))
        query, key, value = (t.transpose(1, 2) for t in (query, key, value))
        output = self.backend(query, key, value).transpose(1, 2).contiguous()
        if self.group is not None:
            output = all_to_all_after_attn(output, self.group, pad_key=PAD_KEY)
        return attn.to_out[1](attn.to_out[0](output.flatten(2, 3)))


def convert_ffn(refiner, group=None) -> int:
    """Replace each block's FFN projections (ff.net[0].proj, ff.net[2]) by
    H3FP8Linear with the activation scale shared over `group`."""
    converted = 0
    for block in refiner.refiner_blocks:
        for parent, name in ((block.ff.net[0], "proj"), (block.ff.net, "2")):
            original = getattr(parent, name)
            if not isinstance(original, torch.nn.Linear):
                raise ValueError("H3 input refiner FP8 expects original FFN Linear modules")
            packed = H3FP8Linear(original.weight, original.bias).to(original.weight.device)
            packed.activation_group = group
            setattr(parent, name, packed)
            converted += 1
    return converted


def install_input_refiner(model, profile, *, sp=None, attention=None, ffn=None):
    """Install the SP refiner on `model.token_refiner`. The SP group is bound
    at the first forward from `model._h3_condition_parallel_manager` or
    `model.parallel_manager` (created after weight preparation)."""
    if profile not in (*PROFILES[1:], "custom"):
        raise ValueError("Unknown H3 input refiner profile")
    sp = True if sp is None else sp
    attention = "cudnn" if attention is None else attention
    ffn = ("fp8" if profile == "cudnn-sp-fp8" else "bf16") if ffn is None else ffn
    if attention != "cudnn":
        raise ValueError("H3 input refiner: only the B200 BF16 attention ('cudnn') is built")
    refiner = model.token_refiner
    if hasattr(refiner, "_h3_sp_metrics"):
        raise ValueError("H3 input refiner SP is already installed")
    world = dist.get_world_size()
    if world not in (2, 4, 8) or (sp and any(b.attn.heads % world for b in refiner.refiner_blocks)):
        raise ValueError("H3 input refiner SP requires 2/4/8 ranks and divisible attention heads")
    if any(p.dtype != torch.bfloat16 for p in refiner.parameters()):
        raise ValueError("H3 input refiner SP expects original BF16 parameters")
    metrics = dict(profile=profile, sp_size=world if sp else 1,
                   communication_dtype="bfloat16" if sp else "none", attention_backend=attention,
                   ffn_precision=ffn, calls=0, completed=0, attention_calls=0, max_input_tokens=0,
                   local_tokens=0, last_input_tokens=0, last_padding=0, fp8_ffn_projections=0,
                   logical_sp_payload_bytes=0)
    if ffn == "fp8":
        metrics["fp8_ffn_projections"] = convert_ffn(refiner)
    backend = H3AttentionBackendB200("bf16")
    processors = []
    for block in refiner.refiner_blocks:
        processor = RefinerSPAttention(None, backend, metrics)
        block.attn.set_processor(processor)
        processors.append(processor)
    original = refiner.forward
    state = {"group": None, "bound": False}

    @wraps(original)
    def forward(hidden_states):
        if torch.is_grad_enabled():
            raise ValueError("H3 input refiner SP is inference-only")
        if hidden_states.device.type != "cuda" or hidden_states.dtype != torch.bfloat16 or hidden_states.ndim != 3:
            raise ValueError("H3 input refiner SP expects CUDA BF16 batch/token/channel inputs")
        tokens = hidden_states.shape[1]
        if tokens < 1:
            raise ValueError("H3 input refiner cannot have an empty context")
        if sp and not state["bound"]:
            manager = getattr(model, "_h3_condition_parallel_manager", getattr(model, "parallel_manager", None))
            if (manager is None or manager.sp_group is None
                    or dist.get_world_size(manager.sp_group) != world
                    or getattr(manager, "tp_size", 1) != 1):
                raise ValueError(f"H3 input refiner requires an initialized SP{world} group")
            group = state["group"] = manager.sp_group
            for processor in processors:
                processor.group = group
            if ffn == "fp8":
                for block in refiner.refiner_blocks:
                    block.ff.net[0].proj.activation_group = group
                    block.ff.net[2].activation_group = group
            state["bound"] = True
        group = state["group"]
        pad = set_pad(PAD_KEY, tokens, group) if sp else 0
        metrics["calls"] += 1
        metrics["last_input_tokens"] = tokens
        metrics["last_padding"] = pad
        metrics["max_input_tokens"] = max(tokens, metrics["max_input_tokens"])
        local = split_sequence(hidden_states, group, dim=1, pad=pad) if sp else hidden_states
        metrics["local_tokens"] = local.shape[1]
        local = original(local)
        result = gather_sequence(local, group, dim=1, pad=pad) if sp else local
        metrics["completed"] += 1
        return result

    refiner.forward = forward
    refiner._h3_sp_metrics = metrics
    refiner._h3_cudnn_backend = backend
    model._h3_input_refiner_profile = profile
    logger.info("H3 input token refiner: profile=%s SP=%d attention=%s FFN=%s FP8 projections=%d",
                profile, metrics["sp_size"], attention, ffn, metrics["fp8_ffn_projections"])
    return metrics
