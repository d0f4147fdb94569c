"""AdaLN sources on CPU: the safetensors table format, the schedule cache
(x_base/x_base/adaln_cache/cache.py:47-296) including int8 tables,
conditioning prefixes and constant-row merging, modality row indices
(minimax_h3.py:410-415), LocalSpan (h3_local_io.py:14-38) and the rank-owner
projection (h3_adaln_owner.py:9-41) over 2 gloo ranks."""
import os
import socket
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from xgen_b200.h3.adaln import (AdalnScheduleCache, H3OwnedAdaLN, LocalSpan, SafetensorsFile,
                                adaln_indices, write_safetensors)

H, M, BLOCKS = 8, 2, 3


def _tables(seed, steps=2, const=True, prefix="", quant=False):
    g = torch.Generator().manual_seed(seed)
    t, raw = {}, {}

    def put(key, value):
        raw[key] = value
        if quant:
            scale = value.abs().amax().clamp_min(1e-6) / 127.0
            t[key + "_int8"] = torch.round(value / scale).clamp(-127, 127).to(torch.int8)
            t[key + "_scale"] = scale.reshape(1)
        else:
            t[key] = value.bfloat16()

    for s in range(steps):
        t[f"{prefix}step{s}_timesteps"] = torch.tensor([0.9 - 0.1 * s, 0.5 - 0.1 * s])
        for b in range(BLOCKS):
            put(f"{prefix}step{s}_block{b}", torch.randn(M, 3 * 6 * H, generator=g))
        put(f"{prefix}step{s}_final", torch.randn(M, 2 * H, generator=g))
    if const:
        t["const_timesteps"] = torch.tensor([0.999, 1.0])
        for b in range(BLOCKS):
            put(f"const_block{b}", torch.randn(2, 3 * 6 * H, generator=g))
        put("const_final", torch.randn(2, 2 * H, generator=g))
    return t, raw


def _expect(value, quant):
    if quant:
        scale = value.abs().amax().clamp_min(1e-6) / 127.0
        codes = torch.round(value / scale).clamp(-127, 127).to(torch.int8)
        return (codes.float() * scale.reshape(1)).bfloat16()
    return value.bfloat16()


def test_safetensors_round_trip(tmp_path):
    path = str(tmp_path / "t.safetensors")
    data = {"a": torch.randn(3, 5).bfloat16(), "b": torch.arange(7, dtype=torch.int8),
            "c": torch.randn(2, 2, 2)}
    write_safetensors(path, data, {"num_steps": 3, "x": "y"})
    f = SafetensorsFile(path)
    assert set(f.keys()) == set(data) and f.metadata() == {"num_steps": "3", "x": "y"}
    for k, v in data.items():
        assert torch.equal(f.get_tensor(k), v)
    with open(path, "rb") as fh:  # header padded to 8 bytes, as the format requires
        assert int.from_bytes(fh.read(8), "little") % 8 == 0


@pytest.mark.parametrize("quant", [False, True])
def test_schedule_cache_lookup(tmp_path, quant):
    tensors, raw = _tables(1, quant=quant)
    path = str(tmp_path / "adaln.safetensors")
    write_safetensors(path, tensors, {"num_steps": 3, "num_blocks": BLOCKS,
                                      "quantization": "int8" if quant else "none"})
    cache = AdalnScheduleCache(cache_file=path, device="cpu")
    assert not cache.has_current
    for s in range(2):
        cache.maybe_install(tensors[f"step{s}_timesteps"])
        assert cache.has_current
        for b in range(BLOCKS):
            table = _expect(raw[f"step{s}_block{b}"], quant).view(-1, 6 * H)
            parts = cache.lookup_block(b)
            assert len(parts) == 6 and parts[0].shape == (M * 3, H)
            for j in range(6):
                assert torch.equal(parts[j], table[:, j * H:(j + 1) * H])
            assert torch.equal(cache.lookup_block_table(b), table)
        shift, scale = cache.lookup_final()
        final = _expect(raw[f"step{s}_final"], quant)
        assert torch.equal(shift, final[:, :H]) and torch.equal(scale, final[:, H:])
    with pytest.raises(KeyError):
        cache.maybe_install(torch.tensor([0.123, 0.456]))


@pytest.mark.parametrize("conditioning,const_idx", [("video", [0]), ("audio", [1]), ("both", [0, 1])])
def test_constant_rows_are_merged(tmp_path, conditioning, const_idx):
    tensors, raw = _tables(2)
    path = str(tmp_path / "adaln.safetensors")
    write_safetensors(path, tensors, {"num_steps": 3, "num_blocks": BLOCKS})
    cache = AdalnScheduleCache(cache_file=path, conditioning_type=conditioning, device="cpu")
    ts = torch.cat([tensors["step1_timesteps"], tensors["const_timesteps"][const_idx]])
    cache.maybe_install(ts)
    rows = torch.tensor([3 * i + m for i in const_idx for m in range(3)])
    for b in range(BLOCKS):
        step = raw[f"step1_block{b}"].bfloat16().view(-1, 6 * H)
        const = raw[f"const_block{b}"].bfloat16().view(-1, 6 * H).index_select(0, rows)
        expect = torch.cat([step, const])
        assert torch.equal(cache.lookup_block_table(b), expect)
        assert torch.equal(cache.lookup_block(b)[2], expect[:, 2 * H:3 * H])
    shift, scale = cache.lookup_final()
    fin, cfin = raw["step1_final"].bfloat16(), raw["const_final"].bfloat16()[const_idx]
    assert torch.equal(shift, torch.cat([fin[:, :H], cfin[:, :H]]))
    assert torch.equal(scale, torch.cat([fin[:, H:], cfin[:, H:]]))


def test_conditioned_tables_and_errors(tmp_path):
    tensors, raw = _tables(3, const=False, prefix="audio_")
    path = str(tmp_path / "adaln.safetensors")
    write_safetensors(path, tensors, {"num_eval_steps": 2, "num_blocks": BLOCKS,
                                      "conditioning_tables": "audio"})
    cache = AdalnScheduleCache(cache_file=path, conditioning_type="audio", device="cpu")
    cache.maybe_install(tensors["audio_step0_timesteps"])
    assert torch.equal(cache.lookup_block_table(1), raw["audio_step0_block1"].bfloat16().view(-1, 6 * H))
    with pytest.raises(ValueError, match="conditioning=video"):
        AdalnScheduleCache(cache_file=path, conditioning_type="video", device="cpu")
    plain, _ = _tables(4, const=False)
    path2 = str(tmp_path / "plain.safetensors")
    write_safetensors(path2, plain, {"num_steps": 3, "num_blocks": BLOCKS})
    with pytest.raises(RuntimeError, match="requires constant"):
        AdalnScheduleCache(cache_file=path2, conditioning_type="video", device="cpu")


def test_adaln_indices():
    t = torch.tensor([0, 0, 1, 1, 2])
    tags = torch.tensor([0, 1, 2, -1, 0])
    idx, mask = adaln_indices(t, tags)
    assert idx.tolist() == [0, 1, 5, 3, 6]
    assert mask is not None and mask[3, 3] and not mask[3, 0] and mask[0, 4]
    idx, mask = adaln_indices(t, tags.clamp(min=0))
    assert mask is None


def test_local_span():
    spans = [LocalSpan.for_rank(10, 4, r) for r in range(4)]
    assert [(s.start, s.length, s.valid) for s in spans] == [(0, 3, 3), (3, 3, 3), (6, 3, 3), (9, 3, 1)]
    x = torch.arange(10)
    assert spans[3].slice_padded(x, value=-1).tolist() == [9, -1, -1]
    src, dst = spans[1].indices(torch.tensor([8, 3, 5, 1, 4]))
    assert src.tolist() == [1, 2, 4] and dst.tolist() == [0, 2, 1]
    with pytest.raises(ValueError):
        LocalSpan.for_rank(10, 4, 4)


def _owner_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)  # identical weights on both ranks; only the owner uses them
        hidden = 4
        original = SimpleNamespace(hidden_size=hidden, linear=torch.nn.Linear(8, 6 * hidden))
        mod = H3OwnedAdaLN(original, index=1, exact_cache=True)
        temb = torch.randn(3, 8, generator=torch.Generator().manual_seed(5))
        with torch.no_grad():
            first = mod(temb)
            second = mod(temb)
            expect = original.linear(torch.nn.functional.silu(temb)).reshape(-1, 6 * hidden).chunk(6, dim=-1)
        results[rank] = (all(torch.equal(a, b) for a, b in zip(first, expect)),
                         all(torch.equal(a, b) for a, b in zip(second, expect)),
                         mod.owner, mod.projection_calls, mod.cache_hits, mod.linear is None)
    finally:
        dist.destroy_process_group()


def test_owned_adaln_two_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    procs = [ctx.Process(target=_owner_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    # rank 1 owns block index 1: it projects once and hits its cache once;
    # rank 0 holds no weights and receives the broadcast
    assert results[1] == (True, True, 1, 1, 1, False)
    assert results[0] == (True, True, 1, 0, 0, True)
