"""SP=2 Q/K/V gather over NVLink peer memory (xgb_fp8_wire_encode_peers +
bounded epoch flags) on two GPUs:

- the receive buffer holds, byte for byte, what the encode + NCCL
  all_to_all_single path receives, for several exchanges in a row (both
  slots, and a slot reused after its "freed" flags), with and without the
  fused RoPE;
- the returned attention output decodes to the NCCL path's values;
- the SP attention layer over it (gather and return, 1, 2 or 4 PHAA chunks,
  so slots are reused within a layer) equals the NCCL path bit for bit.

Skips when fewer than two GPUs are visible."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

D = 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    return dev


def _wire_worker(rank, world, port, results):
    import torch.distributed as dist

    from xgen_b200.attention import kernel_errors
    from xgen_b200.h3.rope import rope_partial
    from xgen_b200.phaa import fp8_transport as fp8
    from xgen_b200.phaa import peer_wire

    dev = _init(rank, world, port)
    try:
        s_loc, hp = 512, 4  # local tokens, heads per peer
        ok = []
        for step in range(4):
            g = torch.Generator(device=dev).manual_seed(100 * step + rank)
            qkv = [torch.randn(1, s_loc, world * hp * D, device=dev, generator=g).bfloat16() for _ in range(3)]
            chunks = tuple(t.unflatten(-1, (world, hp, D)).permute(2, 1, 0, 3, 4) for t in qkv)
            rope = None
            if step % 2:
                cos, sin = rope_partial(world * s_loc, 96 if step == 1 else 128)
                rope = tuple(x[rank * s_loc:(rank + 1) * s_loc].contiguous().to(dev) for x in (cos, sin))
            assert peer_wire.eligible(chunks, D, dist.group.WORLD)
            expect, peers, pad = fp8.fp8_exchange_wire(chunks, D, dist.group.WORLD, rotary_emb=rope)
            got, peers2, pad2, ticket = peer_wire.exchange_wire(chunks, D, dist.group.WORLD, rotary_emb=rope)
            torch.cuda.synchronize()
            ok.append((peers, pad) == (peers2, pad2) and torch.equal(got, expect))
            peer_wire.release(ticket)
            # the return direction: one attention output [peers, seq, batch, heads*D]
            out = torch.randn(world, s_loc, 1, hp * D, device=dev, generator=g).bfloat16()
            back_nccl, back_peer = torch.empty_like(out), torch.empty_like(out)
            fp8.fp8_all_to_all(back_nccl, out, D, dist.group.WORLD)
            wire, peers3, _, ticket = peer_wire.exchange_wire((out.unflatten(-1, (hp, D)),), D, dist.group.WORLD)
            fp8.decode(wire, [back_peer], D, peers3)
            peer_wire.release(ticket)
            torch.cuda.synchronize()
            ok.append(torch.equal(back_peer, back_nccl))
        torch.cuda.synchronize()
        results[rank] = (ok, kernel_errors(dev))
    finally:
        dist.destroy_process_group()


def _layer_worker(rank, world, port, results):
    import torch.distributed as dist

    from xgen_b200.attention import H3AttentionBackendB200, kernel_errors
    from xgen_b200.h3.rope import rope_partial
    from xgen_b200.h3.sp_attention import sp_self_attention
    from xgen_b200.sp import comm
    from xgen_b200.sp.padding import get_pad_manager

    dev = _init(rank, world, port)
    try:
        heads, s = 8, 2048
        g = torch.Generator().manual_seed(7)
        q, k, v = (torch.randn(1, s, heads * D, generator=g).bfloat16() for _ in range(3))
        cos, sin = rope_partial(s, 96)
        pad = get_pad_manager().set("mmh3_seq", s, world)
        shard = [comm.split_sequence(t, dist.group.WORLD, dim=1, pad=pad).to(dev) for t in (q, k, v)]
        cs = tuple(comm.split_sequence(t, dist.group.WORLD, dim=0, pad=pad).to(dev) for t in (cos, sin))
        backend = H3AttentionBackendB200("sage")
        comm_stream = torch.cuda.Stream(device=dev)
        outs = {}
        for mode in ("0", "1", "1", "0", "1"):
            os.environ["XGB_SP_PEER_WIRE"] = mode
            for phaa in (1, 2, 4):
                out = sp_self_attention(*shard, cs, backend=backend, heads=heads, head_dim=D,
                                        sp_group=dist.group.WORLD, sp_size=world, phaa_num=phaa,
                                        fp8_transport=True, comm_stream=comm_stream)
                outs.setdefault((mode, phaa), []).append(out.cpu())
        torch.cuda.synchronize()
        same = all(torch.equal(o, outs[("0", phaa)][0]) for (mode, phaa), lst in outs.items() for o in lst)
        results[rank] = (same, backend.kernel_calls, kernel_errors(dev))
    finally:
        dist.destroy_process_group()


def _run(target):
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    return results


def test_peer_wire_equals_nccl_exchange(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    results = _run(_wire_worker)
    for r in range(2):
        ok, errors = results[r]
        assert all(ok), (r, ok)
        assert errors == 0, r


def test_sp2_layer_over_peer_wire_matches_nccl(cuda_device, monkeypatch):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    monkeypatch.setenv("XGB_ATTN_TAIL_SPLIT", "0")
    results = _run(_layer_worker)
    for r in range(2):
        same, calls, errors = results[r]
        assert same, r
        assert calls > 0 and errors == 0, r
