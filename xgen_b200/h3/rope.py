"""RoPE tables for the H3 packed audio/video/text sequence.

The RoPE kernels consume fp32 cos/sin tables [S, R] in the rotate-half
convention (the reference's contract, x_base/x_base/operator/h3_partial_rope.py
:32-47): channel c < R/2 pairs with c + R/2 and both share one frequency.
`rope_3d` builds the 3-D table of BASELINE's synthetic configs (head dims
split across t/h/w, theta 10000); `rope_partial` the reference model's
partial table (rotary_channels = 6 * rope_freq_dim over the first 96 of 128
channels, minimax_h3.py:78-114).
"""
from __future__ import annotations

import torch


def _axis_freqs(dim: int, theta: float) -> torch.Tensor:
    return theta ** (-torch.arange(0, dim, 2, dtype=torch.float64) / dim)


def rope_3d(grid: tuple[int, int, int], extra_tokens: int = 0, head_dim: int = 128,
            split: tuple[int, int, int] = (32, 48, 48), theta: float = 10000.0):
    """cos, sin fp32 [T*H*W + extra_tokens, head_dim]: video tokens at their
    (t, h, w) grid position, then `extra_tokens` (text/audio) continuing
    along t after the last frame."""
    t, h, w = grid
    if sum(split) != head_dim:
        raise ValueError("axis split must cover the head dim")
    tt, hh, ww = torch.meshgrid(torch.arange(t), torch.arange(h), torch.arange(w), indexing="ij")
    pos = [tt.reshape(-1), hh.reshape(-1), ww.reshape(-1)]
    if extra_tokens:
        pos[0] = torch.cat([pos[0], t + torch.arange(extra_tokens)])
        pos[1] = torch.cat([pos[1], torch.zeros(extra_tokens, dtype=torch.long)])
        pos[2] = torch.cat([pos[2], torch.zeros(extra_tokens, dtype=torch.long)])
    angles = torch.cat([p.double()[:, None] * _axis_freqs(d, theta)[None, :]
                        for p, d in zip(pos, split)], dim=1)  # [S, head_dim/2]
    angles = torch.cat([angles, angles], dim=1)
    return torch.cos(angles).float(), torch.sin(angles).float()


def rope_partial(seq: int, rotary: int = 96, theta: float = 10000.0):
    """1-D rotate-half table over the first `rotary` channels."""
    freqs = _axis_freqs(rotary, theta)
    angles = torch.arange(seq, dtype=torch.float64)[:, None] * freqs[None, :]
    angles = torch.cat([angles, angles], dim=1)
    return torch.cos(angles).float(), torch.sin(angles).float()
