"""Process-wide tensor-parallel group, as x_base/x_base/tensor_parallelism/
state.py:14-40 keeps it: `ParallelManager` writes it when tp_size > 1, and a
TP linear whose own `tp_group` is None reads its group, size and rank here
(size 1 and rank 0 until something registers a group)."""
from __future__ import annotations

from typing import Optional

_tp_group = None
_tp_world_size: int = 1
_tp_rank: int = 0


def set_tp_group(group, world_size: int, rank: int) -> None:
    global _tp_group, _tp_world_size, _tp_rank
    _tp_group, _tp_world_size, _tp_rank = group, int(world_size), int(rank)


def clear_tp_group() -> None:
    set_tp_group(None, 1, 0)


def get_tp_group():
    if _tp_group is None:
        raise ValueError("TP group not initialized. Call ParallelManager with tp_size > 1 first.")
    return _tp_group


def get_tp_world_size() -> int:
    return _tp_world_size


def get_tp_rank() -> int:
    return _tp_rank


def resolve(group) -> tuple[Optional[object], int, int]:
    """(group, size, rank) a TP layer communicates over: its own group when
    it has one, else the registered one (x_base/x_base/tensor_parallelism/
    layers.py:17-27)."""
    if group is not None:
        import torch.distributed as dist

        return group, dist.get_world_size(group), dist.get_rank(group)
    if _tp_world_size > 1:
        return get_tp_group(), _tp_world_size, _tp_rank
    return None, 1, 0
