"""H3 local packed input/output (xgen_b200/h3/local_io.py) against the
contract of x_diffusers/x_diffusers/framework/transformer/h3_local_io.py:
41-92, on CPU: one rank against a direct computation, and two gloo ranks
against the one-rank result."""
import os
import socket
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from xgen_b200.h3.local_io import gather_local_output, prepare_local

HID = 8


class FakeH3(torch.nn.Module):
    def __init__(self):
        super().__init__()
        g = torch.Generator().manual_seed(0)
        lin = lambda i, o: torch.nn.Linear(i, o).requires_grad_(False)  # noqa: E731
        self.proj_in, self.audio_proj_in = lin(6, HID), lin(5, HID)
        self.context_embedder, self.token_refiner = lin(4, HID), lin(HID, HID)
        self.proj_out, self.audio_proj_out = lin(HID, 3), lin(HID, 2)
        for p in self.parameters():
            p.copy_(torch.randn(p.shape, generator=g))
        self.parallel_manager = None

    def rope(self, positions):
        ang = positions.float()[:, None] * torch.arange(1, 5).float()[None]
        return ang.cos(), ang.sin()

    def norm_out(self, hidden, temb, indices):
        return torch.nn.functional.layer_norm(hidden, (HID,)) * (1 + temb[indices][None, :, None])


def _inputs():
    g = torch.Generator().manual_seed(1)
    s = 13
    perm = torch.randperm(s, generator=g)
    text_idx, video_idx, audio_idx = perm[:3], perm[3:11], perm[11:]
    video = torch.randn(1, 8, 6, generator=g)
    audio = torch.randn(1, 2, 5, generator=g)
    text = torch.randn(1, 3, 4, generator=g)
    positions = torch.arange(s) * 3
    temb = torch.randn(s, generator=g)
    return video, audio, text, positions, text_idx, video_idx, audio_idx, temb


def _full(model, video, audio, text, positions, text_idx, video_idx, audio_idx, temb):
    with torch.no_grad():
        hidden, rotary, span = prepare_local(model, video, audio, text, positions, text_idx,
                                             video_idx, audio_idx)
        out = gather_local_output(model, hidden, temb, span, torch.arange(len(positions)),
                                  video_idx, audio_idx)
    return hidden, rotary, span, out


def test_one_rank_scatters_every_modality_to_its_position():
    model = FakeH3()
    video, audio, text, positions, ti, vi, ai, temb = _inputs()
    hidden, rotary, span, (pv, pa) = _full(model, video, audio, text, positions, ti, vi, ai, temb)
    assert (span.start, span.length, span.valid) == (0, 13, 13)
    with torch.no_grad():
        expect = torch.zeros(1, 13, HID)
        expect[0, ti] = model.token_refiner(model.context_embedder(text))[0]
        expect[0, vi] = model.proj_in(video)[0]
        expect[0, ai] = model.audio_proj_in(audio)[0]
        assert torch.equal(hidden, expect)
        assert torch.equal(rotary[0], model.rope(positions)[0])
        normed = model.norm_out(expect, temb, torch.arange(13))
        assert torch.equal(pv, model.proj_out(normed)[:, vi])
        assert torch.equal(pa, model.audio_proj_out(normed)[:, ai])


def test_index_checks():
    model = FakeH3()
    video, audio, text, positions, ti, vi, ai, _ = _inputs()
    with pytest.raises(ValueError, match="indices must match"):
        prepare_local(model, video, audio, text, positions, ti[:2], vi, ai)
    bad = ti.clone()
    bad[0] = 99
    with pytest.raises(RuntimeError, match="outside the sequence"):
        prepare_local(model, video, audio, text, positions, bad, vi, ai)
    model._h3_cuda_precision = "fp8-sage"
    model.proj_out.to(torch.bfloat16)
    hidden, _, span = prepare_local(model, video, audio, text, positions, ti, vi, ai)
    with pytest.raises(ValueError, match="FP32"):
        gather_local_output(model, hidden.bfloat16(), torch.zeros(13), span, torch.arange(13), vi, ai)


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = FakeH3()
        args = _inputs()
        single = _full(model, *args)
        model.parallel_manager = SimpleNamespace(sp_size=world, sp_rank=rank, sp_group=dist.group.WORLD)
        hidden, rotary, span, out = _full(model, *args)
        from xgen_b200.sp.padding import get_pad
        # the projections see fewer rows per rank, which moves the last bit of
        # CPU matmul results: the layout is checked to fp32 accuracy
        close = lambda a, b: a.shape == b.shape and torch.allclose(a, b, rtol=1e-5, atol=1e-6)  # noqa: E731
        own = single[0][:, span.start:span.start + span.valid]
        own = torch.cat([own, torch.zeros(1, span.length - span.valid, HID)], 1)
        results[rank] = (span.start, span.length, span.valid, get_pad("mmh3_seq"), close(hidden, own),
                         close(out[0], single[3][0]), close(out[1], single[3][1]))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_match_one():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    # 13 rows over 2 ranks: spans of 7, the second holding 6 rows and 1 pad
    assert results[0] == (0, 7, 7, 1, True, True, True)
    assert results[1] == (7, 7, 6, 1, True, True, True)
