"""Process-group mesh over (dp, cp, sp, tp) and the parallel manager the
attention modules read their SP group from.

Same interface and rank layout as x_base/x_base/sequence_parallelism/mesh.py:
  ProcessGroupMesh (:32-152)  an N-D row-major grid of the world's ranks;
                              the group "along axis a" of a rank holds the
                              ranks that differ from it only in axis a
  ParallelConfig  (:158-180)  dp*cp*sp*tp == world, ulysses*ring == sp
  ParallelManager (:183-264)  dp/cp/sp/tp groups on axes 0-3, size-1 axes
                              (except dp) leave `<axis>_group/_rank` None;
                              tp_size > 1 registers the process-wide TP group
  initialize      (:271-291)  init_process_group when not yet initialised

The ranks of one group are consecutive in the innermost axes, so with
torchrun's one process per GPU the TP and SP groups of an 8-GPU node are
runs of adjacent GPUs. `dist.new_group` is collective over the world: every
rank creates every group of an axis, in the same row-major order of the
other axes' coordinates, and keeps the one it belongs to.

USP (Ulysses x ring through the yunchang package) is outside the B200 hot
path: a config naming both degrees raises BackendNotAvailableError when
yunchang is not importable, as the reference does.
"""
from __future__ import annotations

import gc
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Sequence, Tuple, Union

import torch
import torch.distributed as dist

from .errors import BackendNotAvailableError, ParallelConfigError

Coord = Tuple[int, ...]


def _prod(nums: Iterable[int]) -> int:
    out = 1
    for n in nums:
        out *= int(n)
    return out


def _strides(shape: Sequence[int]) -> Tuple[int, ...]:
    out, acc = [], 1
    for n in reversed(shape):
        out.append(acc)
        acc *= n
    return tuple(reversed(out))


class ProcessGroupMesh:
    """The world's ranks as a row-major grid of the given shape: rank r sits
    at the coordinate whose dot product with the row-major strides is r."""

    def __init__(self, *size: int) -> None:
        if not dist.is_initialized():
            raise RuntimeError("torch.distributed is not initialized.")
        world = dist.get_world_size()
        if _prod(size) != world:
            raise RuntimeError(f"Product of mesh sizes ({_prod(size)}) must equal world_size ({world}).")
        self._shape: Coord = tuple(int(s) for s in size)
        self._rank: int = dist.get_rank()
        self._coord: Coord = self._unravel(self._rank, self._shape)
        self._ranks_to_group: Dict[Coord, object] = {}
        self._group_to_ranks: Dict[object, Coord] = {}

    @property
    def shape(self) -> Coord:
        return self._shape

    @property
    def rank(self) -> int:
        return self._rank

    @property
    def coord(self) -> Coord:
        return self._coord

    @staticmethod
    def _unravel(rank: int, shape: Sequence[int]) -> Coord:
        if not 0 <= rank < _prod(shape):
            raise ValueError(f"rank {rank} outside a mesh of shape {tuple(shape)}")
        return tuple(int(rank // st % n) for st, n in zip(_strides(shape), shape))

    @staticmethod
    def _ravel(coord: Sequence[int], shape: Sequence[int]) -> int:
        if len(coord) != len(shape) or any(not 0 <= c < n for c, n in zip(coord, shape)):
            raise ValueError(f"coordinate {tuple(coord)} outside a mesh of shape {tuple(shape)}")
        return sum(int(c) * st for c, st in zip(coord, _strides(shape)))

    def _get_coords_along_axis(self, base: Coord, axis: List[int],
                               indices: List[List[int]]) -> List[Coord]:
        """Every coordinate equal to `base` outside `axis`, taking the listed
        indices on each axis in `axis` (the first axis varies slowest)."""
        for ax in axis:
            if not 0 <= ax < len(base):
                raise ValueError(f"Axis {ax} out of bounds for coordinate of dimension {len(base)}")
        coords = [tuple(base)]
        for ax, idxs in zip(axis, indices):
            coords = [c[:ax] + (int(i),) + c[ax + 1:] for c in coords for i in idxs]
        return coords

    def _get_group(self, ranks: Sequence[int], backend: Optional[str] = None):
        key = tuple(sorted(ranks))
        if key not in self._ranks_to_group:
            group = dist.new_group(list(key), backend=backend)
            self._ranks_to_group[key] = group
            if group is not dist.GroupMember.NON_GROUP_MEMBER:
                self._group_to_ranks[group] = key
        return self._ranks_to_group[key]

    def _normalise(self, axis, indices_at_axis):
        if isinstance(axis, int):
            axis = [axis]
            if indices_at_axis is not None and indices_at_axis and isinstance(indices_at_axis[0], int):
                indices_at_axis = [indices_at_axis]
        axis = [int(a) for a in axis]
        for ax in axis:
            if not 0 <= ax < len(self._shape):
                raise ValueError(f"Axis {ax} out of bounds for coordinate of dimension {len(self._shape)}")
        if indices_at_axis is None:
            indices_at_axis = [list(range(self._shape[ax])) for ax in axis]
        return axis, [list(i) for i in indices_at_axis]

    def ranks_along_axis(self, axis: Union[int, List[int]],
                         indices_at_axis: Optional[List] = None) -> Coord:
        """Sorted ranks of this rank's group along `axis`."""
        axis, indices = self._normalise(axis, indices_at_axis)
        coords = self._get_coords_along_axis(self._coord, axis, indices)
        return tuple(sorted(self._ravel(c, self._shape) for c in coords))

    def get_group_along_axis(self, axis: Union[int, List[int]],
                             indices_at_axis: Optional[List] = None,
                             backend: Optional[str] = None):
        """This rank's process group along `axis`; the first request for an
        axis creates the groups of every rank along it (collective)."""
        axis, indices = self._normalise(axis, indices_at_axis)
        mine = self.ranks_along_axis(axis, indices)
        if mine in self._ranks_to_group:
            return self._ranks_to_group[mine]
        return self._create_group_along_axis(axis, indices, backend)

    def _create_group_along_axis(self, axis: List[int], indices: List[List[int]],
                                 backend: Optional[str]):
        others = [1 if d in axis else n for d, n in enumerate(self._shape)]
        target = None
        for flat in range(_prod(others)):
            base = self._unravel(flat, others)
            ranks = [self._ravel(c, self._shape) for c in self._get_coords_along_axis(base, axis, indices)]
            group = self._get_group(ranks, backend=backend)
            if self._rank in ranks:
                target = group
        return target

    def destroy_mesh_process_groups(self) -> None:
        for group in self._ranks_to_group.values():
            if group is not dist.GroupMember.NON_GROUP_MEMBER:
                dist.destroy_process_group(group)
        self._ranks_to_group.clear()
        self._group_to_ranks.clear()
        gc.collect()


@dataclass
class ParallelConfig:
    dp_size: int = 1
    cp_size: int = 1
    sp_size: int = 1
    tp_size: int = 1
    sp_ulysses_size: Optional[int] = None
    sp_ring_size: Optional[int] = None

    def validate(self, world_size: int) -> None:
        sizes = (self.dp_size, self.cp_size, self.sp_size, self.tp_size)
        if any(int(s) < 1 for s in sizes):
            raise ParallelConfigError(f"parallel sizes must be >= 1, got dp/cp/sp/tp = {sizes}")
        total = _prod(sizes)
        if total != world_size:
            raise ParallelConfigError(
                f"dp({self.dp_size}) * cp({self.cp_size}) * sp({self.sp_size}) * tp({self.tp_size}) "
                f"= {total}, but world_size = {world_size}")
        if self.sp_ulysses_size and self.sp_ring_size \
                and self.sp_ulysses_size * self.sp_ring_size != self.sp_size:
            raise ParallelConfigError(
                f"ulysses({self.sp_ulysses_size}) * ring({self.sp_ring_size}) != sp({self.sp_size})")


class ParallelManager:
    """dp/cp/sp/tp groups over a (dp, cp, sp, tp) mesh. The H3 attention
    reads `sp_group`/`sp_size`/`sp_rank` from it (x_comfyui/x_comfyui/
    framework/transformer/minimax_h3.py:143-147)."""

    def __init__(self, dp_size: int, cp_size: int, sp_size: int, tp_size: int = 1,
                 sp_ulysses_size: Optional[int] = None, sp_ring_size: Optional[int] = None,
                 register_tp_global: bool = True) -> None:
        self._register_tp_global = register_tp_global
        self._config = ParallelConfig(dp_size, cp_size, sp_size, tp_size, sp_ulysses_size, sp_ring_size)
        self._config.validate(dist.get_world_size())
        self._mesh = ProcessGroupMesh(dp_size, cp_size, sp_size, tp_size)
        self._init_groups()

    def _axis(self, axis: int, size: int, always: bool = False):
        if size > 1 or always:
            group = self._mesh.get_group_along_axis(axis)
            return group, dist.get_rank(group)
        return None, None

    def _init_groups(self) -> None:
        c = self._config
        self.dp_size, self.cp_size, self.sp_size, self.tp_size = c.dp_size, c.cp_size, c.sp_size, c.tp_size
        self.dp_group, self.dp_rank = self._axis(0, c.dp_size, always=True)
        self.cp_group, self.cp_rank = self._axis(1, c.cp_size)
        self.enable_usp = False
        self.sp_group, self.sp_rank = self._axis(2, c.sp_size)
        if c.sp_size > 1:
            self._init_ulysses_sp()
        self.tp_group, self.tp_rank = self._axis(3, c.tp_size)
        if c.tp_size > 1 and self._register_tp_global:
            from ..tp_state import set_tp_group

            set_tp_group(group=self.tp_group, world_size=self.tp_size, rank=self.tp_rank)

    def _init_ulysses_sp(self) -> None:
        ulysses, ring = self._config.sp_ulysses_size, self._config.sp_ring_size
        if not (ulysses and ring):
            return
        try:
            from yunchang import set_seq_parallel_pg
        except ImportError:
            raise BackendNotAvailableError("yunchang", "pip install yunchang") from None
        set_seq_parallel_pg(sp_ulysses_degree=ulysses, sp_ring_degree=ring,
                            rank=dist.get_rank(), world_size=dist.get_world_size())
        self.enable_usp = True

    @property
    def config(self) -> ParallelConfig:
        return self._config

    @property
    def mesh(self) -> ProcessGroupMesh:
        return self._mesh

    def destroy(self) -> None:
        if self.tp_size > 1 and self._register_tp_global:
            from ..tp_state import clear_tp_group

            clear_tp_group()
        self._mesh.destroy_mesh_process_groups()


def initialize(rank: int = 0, world_size: int = 1, init_method: Optional[str] = None,
               backend: str = "nccl") -> None:
    """init_process_group once per process and bind the process to GPU `rank`
    (x_base/x_base/sequence_parallelism/mesh.py:271-291)."""
    if dist.is_initialized():
        return
    dist.init_process_group(backend=backend, init_method=init_method, world_size=world_size, rank=rank)
    if torch.cuda.is_available():
        torch.cuda.set_device(rank % torch.cuda.device_count())
