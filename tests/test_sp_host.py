"""Host-side SP/PHAA logic on CPU: layouts against the reference's own
run_phaa_attention (golden fixture), padding rules, and a real 2-rank gloo
exchange against the single-rank result."""
import os
import socket
from unittest.mock import patch

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from conftest import golden
from xgen_b200.phaa import phaa_attention as phaa
from xgen_b200.sp import comm
from xgen_b200.sp.padding import PadManager, PadNotSetError, get_pad_manager


def _bf16(bits):
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def _sdpa(q, k, v, **kwargs):
    return F.scaled_dot_product_attention(q.float(), k.float(), v.float()).to(q.dtype)


def test_phaa_matches_reference_layout():
    """Same inputs, same local-copy exchange and attention as the fixture made
    by the reference's run_phaa_attention (phaa_attention.py:38-366)."""
    g = golden("phaa_local")
    for i in range(int(g["ncases"])):
        b, s, heads, d, sp, split, pad, calls = (int(x) for x in g[f"c{i}_meta"])
        qkv = [_bf16(g[f"c{i}_{n}"]).reshape(b, s, heads * d) for n in "qkv"]
        get_pad_manager()._pads["mmh3_seq"] = pad

        def local_copy(output, tensor, **kwargs):
            output.copy_(tensor)

        with patch.object(dist, "get_world_size", return_value=sp), \
             patch.object(dist, "all_to_all_single", side_effect=local_copy) as ex:
            out = phaa.run_phaa_attention(*qkv, comm_stream=phaa._HostStreams._Stream(),
                                          sp_group=None, sp_size=sp, heads=heads,
                                          phaa_split_num=split, head_dim=d, attention_fn=_sdpa,
                                          pad_key="mmh3_seq")
            assert ex.call_count == calls
        ref = _bf16(g[f"c{i}_out"]).reshape(out.shape)
        assert torch.equal(out, ref), i
    get_pad_manager().clear()


def test_chunk_sizes_follow_reference():
    # 7 heads per device, 2 chunks -> [4, 3] (phaa_attention.py:113-118)
    assert phaa.chunk_sizes(7, 2) == [4, 3]
    assert phaa.chunk_sizes(3, 2) == [2, 1]
    assert phaa.chunk_sizes(12, 4) == [3, 3, 3, 3]


def test_pad_manager_contract():
    m = PadManager()
    assert m.set("mmh3_seq", 126754, 8) == 6
    assert m.get("mmh3_seq") == 6 and m.is_set("mmh3_seq")
    assert m.set("x", 16, 8) == 0
    with pytest.raises(PadNotSetError):
        m.get("missing")
    assert m.get_or_default("missing", 3) == 3


def test_phaa_option_validation():
    q = torch.zeros(1, 4, 2 * 64, dtype=torch.bfloat16)
    common = dict(comm_stream=None, sp_group=None, sp_size=1, heads=2, phaa_split_num=1,
                  head_dim=64, attention_fn=_sdpa)
    with pytest.raises(ValueError, match="gather priority"):
        phaa.run_phaa_attention(q, q, q, gather_priority=True, **common)
    with pytest.raises(ValueError, match="tail-first"):
        phaa.run_phaa_attention(q, q, q, tail_first=True, **common)
    with pytest.raises(ValueError, match="FP8 transport requires CUDA"):
        phaa.run_phaa_attention(q, q, q, fp8_transport=True, **common)
    from xgen_b200.phaa.fp8_async_transport import AsyncFP8Options
    with pytest.raises(ValueError, match="fused return pack requires direct return"):
        AsyncFP8Options(fused_return_pack=True)
    with pytest.raises(ValueError, match="async exchange requires device join"):
        phaa.run_phaa_attention(q, q, q, fp8_transport=True, async_options=AsyncFP8Options(),
                                **common)
    with pytest.raises(ValueError, match="device join requires single-stream FP8"):
        phaa.run_phaa_attention(q, q, q, device_join=True, async_options=AsyncFP8Options(),
                                **common)


# ------------------------------------------------------------------ 2 gloo ranks
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, k, v, heads, d, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s = q.shape[1]
        pad = (world - s % world) % world
        get_pad_manager().set("mmh3_seq", s, world)
        shards = [comm.split_sequence(t, dist.group.WORLD, dim=1, pad=pad) for t in (q, k, v)]
        # plain Ulysses
        q4, k4, v4 = (comm.all_to_all_before_attn(t.unflatten(-1, (heads, d)), None, 2, 1, "mmh3_seq")
                      for t in shards)
        att = _sdpa(q4.transpose(1, 2), k4.transpose(1, 2), v4.transpose(1, 2)).transpose(1, 2)
        uly = comm.all_to_all_after_attn(att, None, 1, 2, "mmh3_seq").flatten(2)
        # PHAA with the bf16 exchange
        ph = phaa.run_phaa_attention(*shards, comm_stream=phaa._HostStreams._Stream(),
                                     sp_group=None, sp_size=world, heads=heads, phaa_split_num=2,
                                     head_dim=d, attention_fn=_sdpa, pad_key="mmh3_seq")
        results[rank] = (comm.gather_sequence(uly, None, 1, pad), comm.gather_sequence(ph, None, 1, pad))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("s,heads", [(24, 4), (23, 4), (21, 6)])
def test_two_rank_sp_matches_single_rank(s, heads):
    # heads=6 on 2 ranks gives 3 local heads in PHAA chunks [2, 1], the
    # uneven split of 24 heads at SP8
    d = 32
    g = torch.Generator().manual_seed(s)
    q, k, v = (torch.randn(1, s, heads * d, generator=g).bfloat16() for _ in range(3))
    expect = _sdpa(*(t.unflatten(-1, (heads, d)).transpose(1, 2) for t in (q, k, v)))
    expect = expect.transpose(1, 2).flatten(2)
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, k, v, heads, d, results))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    for r in range(2):
        uly, ph = results[r]
        assert torch.equal(uly, expect)
        assert torch.equal(ph, expect)


def test_tail_split_switch(monkeypatch):
    """XGB_ATTN_TAIL_SPLIT=0 hands the attention kernels no split workspace
    (so they run unsplit); the lookup happens before any device work."""
    from xgen_b200 import attention

    monkeypatch.setenv("XGB_ATTN_TAIL_SPLIT", "0")
    assert attention._ws_args(torch.device("cuda", 0)) == (None, 0)
