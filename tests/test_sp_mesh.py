"""Process-group mesh and parallel manager (xgen_b200/sp/mesh.py) against
the behaviour x_base/tests/test_sp_mesh.py pins for
x_base/x_base/sequence_parallelism/mesh.py, plus a real 4-rank gloo run that
checks every group's membership against numpy's row-major unravel and the
registered TP state."""
import os
import socket
from unittest.mock import MagicMock, patch

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from xgen_b200.sp.errors import BackendNotAvailableError, ParallelConfigError, SequenceParallelError
from xgen_b200.sp.mesh import ParallelConfig, ParallelManager, ProcessGroupMesh, _prod, initialize

MESH_DIST = "xgen_b200.sp.mesh.dist"


def _fake_dist(world, rank, initialized=True):
    fake = MagicMock()
    fake.is_initialized.return_value = initialized
    fake.get_world_size.return_value = world
    fake.get_rank.return_value = rank
    fake.new_group.side_effect = lambda ranks, backend=None: ("group", tuple(ranks))
    fake.GroupMember = dist.GroupMember
    return fake


def _mesh(shape, rank):
    with patch(MESH_DIST, _fake_dist(_prod(shape), rank)):
        return ProcessGroupMesh(*shape)


def test_prod():
    assert _prod([]) == 1 and _prod([5]) == 5 and _prod([2, 3, 4]) == 24


def test_mesh_needs_initialised_world_of_matching_size():
    with patch(MESH_DIST, _fake_dist(8, 0, initialized=False)):
        with pytest.raises(RuntimeError, match="not initialized"):
            ProcessGroupMesh(2, 2)
    with patch(MESH_DIST, _fake_dist(8, 0)):
        with pytest.raises(RuntimeError, match="Product of mesh sizes"):
            ProcessGroupMesh(2, 2)
    m = _mesh((2, 2, 2), 3)
    assert m.shape == (2, 2, 2) and m.rank == 3 and m.coord == (0, 1, 1)


@pytest.mark.parametrize("shape", [(2, 2, 2), (1, 2, 1, 4), (3, 1, 2, 2), (8,)])
def test_ravel_unravel_row_major(shape):
    for r in range(_prod(shape)):
        c = ProcessGroupMesh._unravel(r, shape)
        assert c == tuple(int(i) for i in np.unravel_index(r, shape))
        assert ProcessGroupMesh._ravel(c, shape) == r
    assert ProcessGroupMesh._unravel(5, (2, 2, 2)) == (1, 0, 1)
    assert ProcessGroupMesh._ravel((1, 0, 1), (2, 2, 2)) == 5
    with pytest.raises(ValueError):
        ProcessGroupMesh._unravel(_prod(shape), shape)


def test_coords_along_axis():
    m = _mesh((2, 2, 2), 0)
    assert set(m._get_coords_along_axis((1, 0, 1), [2], [[0, 1]])) == {(1, 0, 0), (1, 0, 1)}
    assert len(m._get_coords_along_axis((0, 0, 0), [0, 2], [[0, 1], [0, 1]])) == 4
    with pytest.raises(ValueError, match="out of bounds"):
        m._get_coords_along_axis((0, 0, 0), [3], [[0]])


def test_group_along_axis_creates_every_group_once_in_row_major_order():
    fake = _fake_dist(8, 5)  # coordinate (1, 0, 1) of a (2, 2, 2) mesh
    with patch(MESH_DIST, fake):
        m = ProcessGroupMesh(2, 2, 2)
        g = m.get_group_along_axis(2)
        again = m.get_group_along_axis(2)
    assert g == ("group", (4, 5)) and again is g
    created = [c.args[0] for c in fake.new_group.call_args_list]
    assert created == [[0, 1], [2, 3], [4, 5], [6, 7]]  # every rank makes the same calls
    cached = MagicMock()
    m._ranks_to_group[(1, 5)] = cached
    with patch(MESH_DIST, fake):
        assert m.get_group_along_axis(0) is cached


def test_destroy_clears_caches():
    fake = _fake_dist(4, 0)
    with patch(MESH_DIST, fake):
        m = ProcessGroupMesh(2, 2)
        m.get_group_along_axis(0)
        m.destroy_mesh_process_groups()
    assert fake.destroy_process_group.call_count == 2
    assert not m._ranks_to_group and not m._group_to_ranks


def test_parallel_config_validate():
    ParallelConfig(dp_size=2, cp_size=1, sp_size=4).validate(8)
    ParallelConfig(dp_size=1, cp_size=1, sp_size=4, sp_ulysses_size=2, sp_ring_size=2).validate(4)
    with pytest.raises(ParallelConfigError, match="dp.*cp.*sp"):
        ParallelConfig(dp_size=2, cp_size=2, sp_size=4).validate(8)
    with pytest.raises(ParallelConfigError, match="ulysses"):
        ParallelConfig(dp_size=1, cp_size=1, sp_size=4, sp_ulysses_size=2, sp_ring_size=3).validate(4)
    with pytest.raises(ParallelConfigError):
        ParallelConfig(dp_size=0, cp_size=1, sp_size=8).validate(0)
    assert issubclass(ParallelConfigError, SequenceParallelError)


def test_manager_dp_only_leaves_other_axes_none():
    group = MagicMock()
    with patch(MESH_DIST, _fake_dist(4, 0)), \
         patch.object(ProcessGroupMesh, "get_group_along_axis", return_value=group):
        mgr = ParallelManager(dp_size=4, cp_size=1, sp_size=1)
    assert mgr.dp_size == 4 and mgr.dp_group is group and mgr.dp_rank == 0
    assert mgr.cp_group is None and mgr.sp_group is None and mgr.tp_group is None
    assert mgr.sp_rank is None and mgr.sp_size == 1 and not mgr.enable_usp


def test_manager_usp_needs_yunchang():
    with patch(MESH_DIST, _fake_dist(4, 0)), \
         patch.object(ProcessGroupMesh, "get_group_along_axis", return_value=MagicMock()), \
         patch.dict("sys.modules", {"yunchang": None}):
        with pytest.raises(BackendNotAvailableError, match="yunchang"):
            ParallelManager(dp_size=1, cp_size=1, sp_size=4, sp_ulysses_size=2, sp_ring_size=2)


def test_manager_rejects_bad_config_before_making_groups():
    fake = _fake_dist(8, 0)
    with patch(MESH_DIST, fake):
        with pytest.raises(ParallelConfigError):
            ParallelManager(dp_size=2, cp_size=2, sp_size=4)
    fake.new_group.assert_not_called()


def test_initialize():
    fake = _fake_dist(4, 0, initialized=False)
    with patch(MESH_DIST, fake):
        initialize(rank=0, world_size=4, backend="nccl")
    fake.init_process_group.assert_called_once()
    fake = _fake_dist(4, 0)
    with patch(MESH_DIST, fake):
        initialize(rank=0, world_size=4)
    fake.init_process_group.assert_not_called()


def _members(shape, rank, axis):
    """Ranks that share every coordinate of `rank` except `axis` (numpy)."""
    c = np.unravel_index(rank, shape)
    return sorted(int(r) for r in range(int(np.prod(shape)))
                  if all(np.unravel_index(r, shape)[d] == c[d] for d in range(len(shape)) if d != axis))


def _mesh_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    out = {}
    try:
        from xgen_b200 import tp_state

        for sizes in ((2, 1, 2, 1), (1, 1, 2, 2), (1, 2, 1, 2), (1, 1, 4, 1)):
            mgr = ParallelManager(*sizes)
            row = {}
            for axis, name in enumerate(("dp", "cp", "sp", "tp")):
                group = getattr(mgr, name + "_group")
                if group is None:
                    row[name] = None
                    continue
                t = torch.tensor([float(rank)])
                dist.all_reduce(t, group=group)  # the group really connects its members
                row[name] = (sorted(dist.get_process_group_ranks(group)),
                             getattr(mgr, name + "_rank"), float(t))
                row[name + "_expect"] = _members(sizes, rank, axis)
            row["tp_state"] = (tp_state.get_tp_world_size(), tp_state.get_tp_rank())
            mgr.destroy()
            row["tp_after"] = tp_state.get_tp_world_size()
            out[sizes] = row
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_manager_groups_four_gloo_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    procs = [ctx.Process(target=_mesh_worker, args=(r, 4, port, results)) for r in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    for rank in range(4):
        for sizes, row in results[rank].items():
            for name in ("dp", "cp", "sp", "tp"):
                size = sizes[("dp", "cp", "sp", "tp").index(name)]
                if size == 1 and name != "dp":
                    assert row[name] is None, (sizes, name)
                    continue
                ranks, my_rank, total = row[name]
                assert ranks == row[name + "_expect"], (sizes, name)
                assert my_rank == ranks.index(rank)
                assert total == float(sum(ranks))
            tp = sizes[3]
            assert row["tp_state"] == ((tp, row["tp"][1]) if tp > 1 else (1, 0))
            assert row["tp_after"] == 1
    # the H3 layout: SP over the inner ranks of each DP replica
    assert results[3][(2, 1, 2, 1)]["sp"][0] == [2, 3]
    assert results[3][(2, 1, 2, 1)]["dp"][0] == [1, 3]
