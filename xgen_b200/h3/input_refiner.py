"""Opt-in SP path for the H3 input token refiner (the text-conditioning
transformer ahead of the DiT), on the B200 attention and FP8 linears.

Interface of x_diffusers/x_diffusers/adaptor/h3_input_refiner.py:13-148:
`install_input_refiner(model, profile, *, sp, attention, ffn)` with the
profiles "cudnn-sp" (BF16 attention and FFN), "cudnn-sp-fp8" (FP8 FFN
projections) and "custom", returning the metrics dict it keeps updating;
`RefinerSPAttention`, the per-block attention processor; `convert_ffn`.

Design here: one `_RefinerSP` object per installed refiner owns everything
the install sets up, the metrics, the attention backend, the processors and
the SP group. It binds the group lazily (the loader creates the SP group
after weight preparation) and stands in for the refiner's forward:

  tokens [B, T, C] --split over SP (pad key "h3_input_refiner", so the
  DiT's "mmh3_seq" pad is untouched)--> local tokens --original forward-->
  --gather--> [B, T, C]

Inside, each block's attention moves Q/K/V from token shards to head shards
with the Ulysses all-to-all (pad rows dropped before the softmax), runs
full-context attention on the B200 BF16 kernel (the reference's cuDNN
backend, H3DenseCUDA), and moves the output back. With the FP8 FFN every
rank quantises its activations with the scale that the whole (unsharded)
token set gives: a MAX all-reduce of the abs-peak over the SP group.
Inference only.
"""
from __future__ import annotations

import logging

import torch
import torch.distributed as dist

from ..attention import H3AttentionBackendB200
from ..fp8_linear import H3FP8Linear
from ..sp.comm import all_to_all_after_attn, all_to_all_before_attn, gather_sequence, split_sequence
from ..sp.padding import set_pad

logger = logging.getLogger(__name__)
PAD_KEY = "h3_input_refiner"
PROFILES = ("none", "cudnn-sp", "cudnn-sp-fp8")
_METRIC_COUNTERS = ("calls", "completed", "attention_calls", "max_input_tokens", "local_tokens",
                    "last_input_tokens", "last_padding", "fp8_ffn_projections", "logical_sp_payload_bytes")


class RefinerSPAttention:
    """Attention processor of one refiner block: heads spread over the SP
    group (none when `group` is None), BF16 full-context attention."""

    def __init__(self, group, backend, metrics):
        self.group, self.backend, self.metrics = group, backend, metrics

    def _project(self, attn, hidden_states):
        heads = attn.heads
        q, k, v = (proj(hidden_states).unflatten(-1, (heads, attn.head_dim))
                   for proj in (attn.to_q, attn.to_k, attn.to_v))
        q, k = attn.norm_q(q), attn.norm_k(k)
        if {q.dtype, k.dtype, v.dtype} != {torch.bfloat16}:
            raise ValueError("H3 input refiner attention requires BF16 QKV")
        return q, k, v

    def __call__(self, attn, hidden_states, rotary_emb=None, attention_mask=None):
        if attn.fused_projections or rotary_emb is not None or attention_mask is not None:
            raise ValueError("H3 input refiner SP expects unfused QKV, no RoPE and no mask")
        qkv = self._project(attn, hidden_states)
        self.metrics["attention_calls"] += 1
        if self.group is not None:
            # Q, K, V out and the attention output back, as logical bytes
            self.metrics["logical_sp_payload_bytes"] += 4 * qkv[0].numel() * qkv[0].element_size()
            qkv = [all_to_all_before_attn(t, self.group, pad_key=PAD_KEY) for t in qkv]
        heads_major = [t.transpose(1, 2) for t in qkv]           # [B, H, T, D] views
        out = self.backend(*heads_major).transpose(1, 2).contiguous()  # [B, T, H, D]
        if self.group is not None:
            out = all_to_all_after_attn(out, self.group, pad_key=PAD_KEY)
        return attn.to_out[1](attn.to_out[0](out.flatten(2)))


def _ffn_slots(block):
    """(parent, attribute) of the two FFN projections of a refiner block."""
    return (block.ff.net[0], "proj"), (block.ff.net, "2")


def convert_ffn(refiner, group=None) -> int:
    """Swap every block's FFN projections for per-tensor H3FP8Linear whose
    activation scale is MAX-reduced over `group`; returns how many."""
    slots = [slot for block in refiner.refiner_blocks for slot in _ffn_slots(block)]
    for parent, attr in slots:
        if not isinstance(getattr(parent, attr), torch.nn.Linear):
            raise ValueError("H3 input refiner FP8 expects original FFN Linear modules")
    for parent, attr in slots:
        linear = getattr(parent, attr)
        fp8 = H3FP8Linear(linear.weight, linear.bias).to(linear.weight.device)
        fp8.activation_group = group
        setattr(parent, attr, fp8)
    return len(slots)


class _RefinerSP:
    def __init__(self, model, profile, sp, attention, ffn):
        self.model, self.refiner = model, model.token_refiner
        self.sp, self.ffn = sp, ffn
        self.world = dist.get_world_size()
        self.group = None
        self.bound = not sp
        self.metrics = dict(profile=profile, sp_size=self.world if sp else 1,
                            communication_dtype="bfloat16" if sp else "none",
                            attention_backend=attention, ffn_precision=ffn)
        self.metrics.update(dict.fromkeys(_METRIC_COUNTERS, 0))
        self.backend = H3AttentionBackendB200("bf16")
        self.processors = [RefinerSPAttention(None, self.backend, self.metrics)
                           for _ in self.refiner.refiner_blocks]
        self.inner = self.refiner.forward

    def validate(self):
        blocks = self.refiner.refiner_blocks
        if self.world not in (2, 4, 8) or (self.sp and any(b.attn.heads % self.world for b in blocks)):
            raise ValueError("H3 input refiner SP requires 2/4/8 ranks and divisible attention heads")
        if any(p.dtype != torch.bfloat16 for p in self.refiner.parameters()):
            raise ValueError("H3 input refiner SP expects original BF16 parameters")

    def apply(self):
        if self.ffn == "fp8":
            self.metrics["fp8_ffn_projections"] = convert_ffn(self.refiner)
        for block, processor in zip(self.refiner.refiner_blocks, self.processors):
            block.attn.set_processor(processor)
        self.refiner.forward = self.forward
        self.refiner._h3_sp_metrics = self.metrics
        self.refiner._h3_cudnn_backend = self.backend
        self.model._h3_input_refiner_profile = self.metrics["profile"]

    def _bind(self):
        """Attach the SP group that exists by the first forward."""
        model = self.model
        manager = getattr(model, "_h3_condition_parallel_manager", None) or getattr(model, "parallel_manager", None)
        usable = (manager is not None and manager.sp_group is not None
                  and dist.get_world_size(manager.sp_group) == self.world
                  and getattr(manager, "tp_size", 1) == 1)
        if not usable:
            raise ValueError(f"H3 input refiner requires an initialized SP{self.world} group")
        self.group = manager.sp_group
        for processor in self.processors:
            processor.group = self.group
        if self.ffn == "fp8":
            for block in self.refiner.refiner_blocks:
                for parent, attr in _ffn_slots(block):
                    getattr(parent, attr).activation_group = self.group
        self.bound = True

    def forward(self, hidden_states):
        if torch.is_grad_enabled():
            raise ValueError("H3 input refiner SP is inference-only")
        if not (hidden_states.is_cuda and hidden_states.dtype == torch.bfloat16 and hidden_states.ndim == 3):
            raise ValueError("H3 input refiner SP expects CUDA BF16 batch/token/channel inputs")
        tokens = hidden_states.shape[1]
        if tokens == 0:
            raise ValueError("H3 input refiner cannot have an empty context")
        if not self.bound:
            self._bind()
        m = self.metrics
        m["calls"] += 1
        m["last_input_tokens"] = tokens
        m["max_input_tokens"] = max(m["max_input_tokens"], tokens)
        if not self.sp:
            m["last_padding"] = 0
            m["local_tokens"] = tokens
            out = self.inner(hidden_states)
        else:
            pad = m["last_padding"] = set_pad(PAD_KEY, tokens, self.group)
            shard = split_sequence(hidden_states, self.group, dim=1, pad=pad)
            m["local_tokens"] = shard.shape[1]
            out = gather_sequence(self.inner(shard), self.group, dim=1, pad=pad)
        m["completed"] += 1
        return out


def install_input_refiner(model, profile, *, sp=None, attention=None, ffn=None):
    """Install the SP refiner on `model.token_refiner`; returns its metrics.
    The SP group is taken at the first forward from
    `model._h3_condition_parallel_manager` or `model.parallel_manager`."""
    if profile not in PROFILES[1:] and profile != "custom":
        raise ValueError("Unknown H3 input refiner profile")
    sp = True if sp is None else sp
    attention = attention or "cudnn"
    if ffn is None:
        ffn = "fp8" if profile == "cudnn-sp-fp8" else "bf16"
    if attention != "cudnn":
        raise ValueError("H3 input refiner: only the B200 BF16 attention ('cudnn') is built")
    if hasattr(model.token_refiner, "_h3_sp_metrics"):
        raise ValueError("H3 input refiner SP is already installed")
    state = _RefinerSP(model, profile, sp, attention, ffn)
    state.validate()
    state.apply()
    logger.info("H3 input token refiner: profile=%s SP=%d attention=%s FFN=%s FP8 projections=%d",
                profile, state.metrics["sp_size"], attention, ffn, state.metrics["fp8_ffn_projections"])
    return state.metrics
