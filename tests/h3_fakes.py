"""A stand-in for the reference's H3 transformer modules (the diffusers
fork is not installed): the attribute layout that prepare_transformer and
the SP attention processor read (x_diffusers/x_diffusers/adaptor/
h3_cuda_precision.py:229-261, framework/transformer/minimax_h3.py:129-251).
Test infrastructure only."""
from __future__ import annotations

import torch
from torch import nn


class FakeAttention(nn.Module):
    def __init__(self, hidden, heads, bias=False, eps=1e-6):
        super().__init__()
        self.heads = heads
        self.to_q = nn.Linear(hidden, hidden, bias=bias)
        self.to_k = nn.Linear(hidden, hidden, bias=bias)
        self.to_v = nn.Linear(hidden, hidden, bias=bias)
        self.to_out = nn.ModuleList([nn.Linear(hidden, hidden, bias=bias), nn.Dropout(0.0)])
        self.norm_q = nn.RMSNorm(hidden // heads, eps=eps)
        self.norm_k = nn.RMSNorm(hidden // heads, eps=eps)
        self.fused_projections = False
        self.processor = None

    def set_processor(self, processor):
        self.processor = processor

    def forward(self, hidden_states, rotary_emb=None, attention_mask=None):
        return self.processor(self, hidden_states, rotary_emb, attention_mask)


class FakeGELU(nn.Module):
    def __init__(self, dim_in, dim_out, approximate="none"):
        super().__init__()
        self.proj = nn.Linear(dim_in, dim_out, bias=False)
        self.approximate = approximate

    def forward(self, x):
        return torch.nn.functional.gelu(self.proj(x), approximate=self.approximate)


class FakeFeedForward(nn.Module):
    def __init__(self, hidden, ffn):
        super().__init__()
        self.net = nn.ModuleList([FakeGELU(hidden, ffn), nn.Dropout(0.0), nn.Linear(ffn, hidden, bias=False)])

    def forward(self, x):
        for layer in self.net:
            x = layer(x)
        return x


class FakeAdaLN(nn.Module):
    """adaln_proj(temb) -> the six [rows, hidden] tables (shift, scale,
    gate, shift_ff, scale_ff, gate_ff) of a cached table."""

    def __init__(self, table):
        super().__init__()
        self.register_buffer("table", table)

    def forward(self, temb):
        return self.table.chunk(6, dim=-1)


class FakeBlock(nn.Module):
    def __init__(self, hidden, heads, ffn, table, eps=1e-6):
        super().__init__()
        self.norm1 = nn.LayerNorm(hidden, elementwise_affine=False, eps=eps)
        self.norm2 = nn.LayerNorm(hidden, elementwise_affine=False, eps=eps)
        self.attn = FakeAttention(hidden, heads, eps=eps)
        self.ff = FakeFeedForward(hidden, ffn)
        self.adaln_proj = FakeAdaLN(table)

    def forward(self, hidden_states, temb, adaln_indices, rotary_emb, attention_mask=None):
        raise NotImplementedError("the BF16 eager block is not part of these tests")


class FakeTransformer(nn.Module):
    def __init__(self, blocks):
        super().__init__()
        self.transformer_blocks = nn.ModuleList(blocks)
        self.parallel_manager = None

    def set_parallel_manager(self, manager):
        self.parallel_manager = manager
        for block in self.transformer_blocks:
            block.attn.parallel_manager = manager


def fake_h3(weights: dict, config, table: torch.Tensor, blocks: int = 1) -> FakeTransformer:
    """A FakeTransformer whose blocks carry `weights` (H3DiTBlockB200
    .random_weights layout, bf16): to_qkv is split into to_q/to_k/to_v."""
    h = config.hidden
    out = []
    for _ in range(blocks):
        blk = FakeBlock(h, config.heads, config.ffn, table, eps=config.eps).to(torch.bfloat16)
        a = blk.attn
        with torch.no_grad():
            a.to_q.weight.copy_(weights["to_qkv"][:h])
            a.to_k.weight.copy_(weights["to_qkv"][h:2 * h])
            a.to_v.weight.copy_(weights["to_qkv"][2 * h:])
            a.to_out[0].weight.copy_(weights["to_out"])
            blk.ff.net[0].proj.weight.copy_(weights["ff_up"])
            blk.ff.net[2].weight.copy_(weights["ff_down"])
            if "norm_q.weight" in weights:
                a.norm_q.weight.copy_(weights["norm_q.weight"])
                a.norm_k.weight.copy_(weights["norm_k.weight"])
        out.append(blk)
    return FakeTransformer(out)
