"""A small module with the structure of the H3 input token refiner (what
install_input_refiner touches): `refiner_blocks`, each with a diffusers-style
attention (`to_q/to_k/to_v`, `norm_q/norm_k`, `to_out`, `heads`, `head_dim`,
`fused_projections`, `set_processor`) and an FFN `ff.net = [GELU(proj),
Dropout, Linear]`. Test helper only."""
import torch
import torch.nn.functional as F


class PlainProcessor:
    """The refiner block's own attention (torch SDPA on its bf16 tensors):
    the unsharded reference."""

    def __call__(self, attn, x, rotary_emb=None, attention_mask=None):
        q, k, v = (layer(x).unflatten(-1, (attn.heads, attn.head_dim)) for layer in (attn.to_q, attn.to_k, attn.to_v))
        q, k = attn.norm_q(q), attn.norm_k(k)
        out = F.scaled_dot_product_attention(*(t.transpose(1, 2) for t in (q, k, v)))
        return attn.to_out[1](attn.to_out[0](out.transpose(1, 2).flatten(2)))


class FakeAttention(torch.nn.Module):
    def __init__(self, hidden, heads):
        super().__init__()
        self.heads, self.head_dim = heads, hidden // heads
        self.to_q, self.to_k, self.to_v = (torch.nn.Linear(hidden, hidden) for _ in range(3))
        self.norm_q = torch.nn.RMSNorm(self.head_dim, eps=1e-5)
        self.norm_k = torch.nn.RMSNorm(self.head_dim, eps=1e-5)
        self.to_out = torch.nn.ModuleList([torch.nn.Linear(hidden, hidden), torch.nn.Dropout(0.0)])
        self.fused_projections = False
        self.processor = PlainProcessor()

    def set_processor(self, processor):
        self.processor = processor

    def forward(self, x):
        return self.processor(self, x)


class GELUProj(torch.nn.Module):
    def __init__(self, i, o):
        super().__init__()
        self.proj = torch.nn.Linear(i, o)

    def forward(self, x):
        return F.gelu(self.proj(x))


class FakeFF(torch.nn.Module):
    def __init__(self, hidden, ffn):
        super().__init__()
        self.net = torch.nn.ModuleList([GELUProj(hidden, ffn), torch.nn.Dropout(0.0), torch.nn.Linear(ffn, hidden)])

    def forward(self, x):
        for layer in self.net:
            x = layer(x)
        return x


class FakeBlock(torch.nn.Module):
    def __init__(self, hidden, heads, ffn):
        super().__init__()
        self.attn, self.ff = FakeAttention(hidden, heads), FakeFF(hidden, ffn)

    def forward(self, x):
        x = x + self.attn(x)
        return x + self.ff(x)


class FakeRefiner(torch.nn.Module):
    def __init__(self, hidden=256, heads=2, ffn=512, blocks=2, seed=0):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.refiner_blocks = torch.nn.ModuleList([FakeBlock(hidden, heads, ffn) for _ in range(blocks)])
        with torch.no_grad():
            for p in self.parameters():
                p.copy_(torch.randn(p.shape, generator=g) * (0.05 if p.ndim > 1 else 0.01) + (1.0 if p.ndim == 1 and p.numel() == hidden // heads else 0.0))
        self.to(torch.bfloat16)

    def forward(self, x):
        for block in self.refiner_blocks:
            x = block(x)
        return x
