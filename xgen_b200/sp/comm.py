"""Ulysses sequence-parallel redistribution (seq-sharded <-> head-sharded).

Same contracts as x_base/x_base/sequence_parallelism/comm.py:
  all_to_all_before_attn  (:853-901)  [B, S/P, H(, D)] -> [B, S - pad, H/P(, D)]
  all_to_all_after_attn   (:904-952)  [B, S - pad, H/P(, D)] -> [B, S/P, H(, D)]
  split_sequence / gather_sequence (:667-800)
with the 4-D A2A of _all_to_all_4d_impl (:308-371): one NCCL
`all_to_all_single` per tensor over the SP group, contiguous S/P spans per
rank, heads [r*H/P, (r+1)*H/P) on rank r after the exchange.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .padding import get_pad_manager


def _world(group) -> int:
    return dist.get_world_size(group) if dist.is_initialized() else 1


def all_to_all_4d(tensor: torch.Tensor, scatter_dim: int, gather_dim: int, group) -> torch.Tensor:
    """(bs, S/P, h) -> (bs, S, h/P) for (2, 1); (bs, S, h/P) -> (bs, S/P, h) for (1, 2)."""
    world = _world(group)
    if world == 1:
        return tensor
    if scatter_dim == 2 and gather_dim == 1:
        bs, shard_s, h = tensor.shape
        send = tensor.reshape(bs, shard_s, world, h // world).transpose(0, 2).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=group)
        return recv.reshape(shard_s * world, bs, h // world).transpose(0, 1).contiguous()
    if scatter_dim == 1 and gather_dim == 2:
        bs, s, shard_h = tensor.shape
        send = (tensor.reshape(bs, world, s // world, shard_h).transpose(0, 3).transpose(0, 1)
                .contiguous().reshape(world, shard_h, s // world, bs))
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=group)
        return (recv.reshape(shard_h * world, s // world, bs).transpose(0, 2).contiguous()
                .reshape(bs, s // world, shard_h * world))
    raise ValueError(
        f"Invalid dimensions: scatter_dim={scatter_dim}, gather_dim={gather_dim}. "
        "Must be (scatter_dim=1, gather_dim=2) or (scatter_dim=2, gather_dim=1).")


def all_to_all_before_attn(tensor, process_group=None, scatter_dim=2, gather_dim=1, pad_key="pad"):
    pad = get_pad_manager().get_or_default(pad_key, 0)
    orig = tensor.shape
    if tensor.ndim > 3:
        tensor = tensor.reshape(orig[0], orig[1], -1)
    out = all_to_all_4d(tensor, scatter_dim, gather_dim, process_group)
    if pad > 0:
        out = out.narrow(gather_dim, 0, out.size(gather_dim) - pad)
    if len(orig) > 3:
        out = out.reshape(out.shape[0], out.shape[1], orig[2] // _world(process_group), *orig[3:])
    return out


def all_to_all_after_attn(tensor, process_group=None, scatter_dim=1, gather_dim=2, pad_key="pad"):
    pad = get_pad_manager().get_or_default(pad_key, 0)
    if pad > 0:
        shape = list(tensor.shape)
        shape[scatter_dim] = pad
        tensor = torch.cat([tensor, tensor.new_zeros(shape)], dim=scatter_dim)
    orig = tensor.shape
    if tensor.ndim > 3:
        tensor = tensor.reshape(orig[0], orig[1], -1)
    out = all_to_all_4d(tensor, scatter_dim, gather_dim, process_group)
    if len(orig) > 3:
        out = out.reshape(out.shape[0], out.shape[1], orig[2] * _world(process_group), *orig[3:])
    return out


def split_sequence(x: torch.Tensor, group, dim: int = 1, pad: int = 0) -> torch.Tensor:
    """This rank's contiguous span of `x` along `dim` after zero-padding by `pad`."""
    world = _world(group)
    if world == 1:
        return x
    if pad > 0:
        shape = list(x.shape)
        shape[dim] = pad
        x = torch.cat([x, x.new_zeros(shape)], dim=dim)
    rank = dist.get_rank(group)
    return x.chunk(world, dim=dim)[rank].contiguous()


def gather_sequence(x: torch.Tensor, group, dim: int = 1, pad: int = 0) -> torch.Tensor:
    """Inverse of split_sequence (all-gather, concatenate, drop the pad)."""
    world = _world(group)
    if world == 1:
        return x
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x.contiguous(), group=group)
    out = torch.cat(parts, dim=dim)
    if pad > 0:
        out = out.narrow(dim, 0, out.size(dim) - pad)
    return out
